"""The fused full-array sum + cross-GPU combine (emmy_xchg_*,
emmy_sum_f32_allreduce): one kernel per GPU sums the shard and exchanges
the per-GPU totals over NVLink peer memory.

* one rank: the result is the shard's sum (rtol 1e-5 against float64) and
  the same bits on every call;
* a peer that never arrives: the bounded wait runs out, the call writes NaN
  and raises status bit 0, and the context stays usable;
* two GPUs, one process each: every rank gets the same bits, equal to the
  two ranks' totals added in rank order.
"""

from __future__ import annotations

import sys

import numpy as np
import pytest

from conftest import REPO

pytestmark = pytest.mark.gpu


def _f32_sum_ref(x) -> float:
    return float(x.double().sum().item())


def test_one_rank_is_the_shard_sum(cuda_device):
    import torch
    from emmy_ptx_compiler_b200 import runtime
    ex = runtime.Exchange(cuda_device, 1, 0)
    ex.connect([ex.handle])
    g = torch.Generator(device=f"cuda:{cuda_device}").manual_seed(11)
    for n in (1, 1000, (1 << 22) + 5, (1 << 26) + 3):
        x = torch.empty(n, dtype=torch.float32, device=f"cuda:{cuda_device}").uniform_(-1, 1, generator=g)
        a = torch.zeros(1, dtype=torch.float32, device=f"cuda:{cuda_device}")
        b = torch.zeros(1, dtype=torch.float32, device=f"cuda:{cuda_device}")
        s = torch.cuda.current_stream(cuda_device).cuda_stream
        ex.sum_allreduce(x, n, a, stream=s)
        ex.sum_allreduce(x, n, b, stream=s)
        torch.cuda.synchronize(cuda_device)
        assert a.item() == b.item(), (n, a.item(), b.item())
        np.testing.assert_allclose(a.item(), _f32_sum_ref(x), rtol=1e-5, atol=1e-4)
    assert ex.status() == 0
    ex.close()


def test_missing_peer_times_out_and_the_context_stays_usable(cuda_device):
    """Rank 0 of 2 whose 'peer' is its own buffer: nothing ever publishes
    rank 1's flag, so the wait (50 ms limit) runs out."""
    import torch
    from emmy_ptx_compiler_b200 import runtime
    ex = runtime.Exchange(cuda_device, 2, 0)
    ex.connect([ex.handle, ex.handle])
    x = torch.ones(4096, dtype=torch.float32, device=f"cuda:{cuda_device}")
    out = torch.zeros(1, dtype=torch.float32, device=f"cuda:{cuda_device}")
    ex.sum_allreduce(x, 4096, out, timeout_ms=50)
    torch.cuda.synchronize(cuda_device)
    assert np.isnan(out.item())
    assert ex.status() & 1
    assert ex.status() == 0, "status is cleared by reading it"
    ex.close()
    ok = runtime.Exchange(cuda_device, 1, 0)
    ok.connect([ok.handle])
    ok.sum_allreduce(x, 4096, out)
    torch.cuda.synchronize(cuda_device)
    assert out.item() == 4096.0
    ok.close()


def _worker(rank: int, world: int, q_hs, q_out) -> None:
    sys.path.insert(0, str(REPO))
    import torch
    from emmy_ptx_compiler_b200 import runtime
    torch.cuda.set_device(rank)
    ex = runtime.Exchange(rank, world, rank)
    for dst in range(world):  # every rank's inbox gets this rank's handle
        q_hs[dst].put((rank, ex.handle))
    handles = {}
    while len(handles) < world:
        r, h = q_hs[rank].get(timeout=60)
        handles[r] = h
    ex.connect([handles[r] for r in range(world)])
    res = []
    g = torch.Generator(device=f"cuda:{rank}").manual_seed(100 + rank)
    for call in range(3):
        n = (1 << 24) + 17 * call
        x = torch.empty(n, dtype=torch.float32, device=f"cuda:{rank}").uniform_(-1, 1, generator=g)
        out = torch.zeros(1, dtype=torch.float32, device=f"cuda:{rank}")
        mine = torch.zeros(1, dtype=torch.float32, device=f"cuda:{rank}")
        s = torch.cuda.current_stream(rank).cuda_stream
        solo = runtime.Exchange(rank, 1, 0)  # this GPU's own total, same kernel and order
        solo.connect([solo.handle])
        solo.sum_allreduce(x, n, mine, stream=s)
        ex.sum_allreduce(x, n, out, timeout_ms=5000, stream=s)
        torch.cuda.synchronize(rank)
        solo.close()
        res.append((float(mine.item()), float(out.item())))
    st = ex.status()
    ex.close()
    q_out.put((rank, res, st))


def test_two_gpus_get_the_same_bits():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q_hs, q_out = [ctx.Queue() for _ in range(2)], ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, q_hs, q_out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    got = dict((r, (res, st)) for r, res, st in (q_out.get(timeout=10) for _ in range(2)))
    assert got[0][1] == 0 and got[1][1] == 0
    for call in range(3):
        s0, o0 = got[0][0][call]
        s1, o1 = got[1][0][call]
        want = float(np.float32(np.float32(s0) + np.float32(s1)))
        assert o0 == o1 == want, (call, o0, o1, want)

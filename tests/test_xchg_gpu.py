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


def test_a_failed_group_stays_failed_until_reset(cuda_device):
    """After a wait runs out, later calls on that GPU publish nothing and
    return at once (NaN, status bit 0), so the GPU can never run two calls
    ahead of a late peer; emmy_xchg_reset clears the state.  Rank 0 of 2 whose
    'peer' is its own buffer: nothing ever publishes rank 1's word."""
    import torch
    from emmy_ptx_compiler_b200 import runtime
    ex = runtime.Exchange(cuda_device, 2, 0)
    ex.connect([ex.handle, ex.handle])
    x = torch.ones(4096, dtype=torch.float32, device=f"cuda:{cuda_device}")
    s = torch.cuda.current_stream(cuda_device).cuda_stream
    times = []
    for _ in range(3):
        out = torch.zeros(1, dtype=torch.float32, device=f"cuda:{cuda_device}")
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        ex.sum_allreduce(x, 4096, out, timeout_ms=100, stream=s)
        e1.record()
        torch.cuda.synchronize(cuda_device)
        times.append(e0.elapsed_time(e1))
        assert np.isnan(out.item())
        assert ex.status() & 1
    assert times[0] >= 90.0, times            # the first call waited out its limit
    assert max(times[1:]) < 20.0, times       # later calls returned at once
    ex.reset()
    out = torch.zeros(1, dtype=torch.float32, device=f"cuda:{cuda_device}")
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    ex.sum_allreduce(x, 4096, out, timeout_ms=100, stream=s)
    e1.record()
    torch.cuda.synchronize(cuda_device)
    assert e0.elapsed_time(e1) >= 90.0, "after reset the group waits again"
    assert np.isnan(out.item()) and ex.status() & 1
    ex.close()


def _exchange(rank: int, world: int, q_hs):
    from emmy_ptx_compiler_b200 import runtime
    ex = runtime.Exchange(rank, world, rank)
    for dst in range(world):
        q_hs[dst].put((rank, ex.handle))
    handles = {}
    while len(handles) < world:
        r, h = q_hs[rank].get(timeout=60)
        handles[r] = h
    ex.connect([handles[r] for r in range(world)])
    return ex


def _late_worker(rank: int, q_hs, q_sig, q_out) -> None:
    """Rank 1 stays away while rank 0 makes two calls (both fail: the first
    waits out, the second returns at once); rank 1's first call then finds
    rank 0's first total and succeeds, and its second call finds nothing
    (rank 0 published nothing for call 2) and fails; after a reset on both
    ranks the next call succeeds on both with the same bits."""
    sys.path.insert(0, str(REPO))
    import torch
    torch.cuda.set_device(rank)
    ex = _exchange(rank, 2, q_hs)
    s = torch.cuda.current_stream(rank).cuda_stream
    x = torch.full((1 << 20,), float(rank + 1), dtype=torch.float32, device=f"cuda:{rank}")
    res = []

    def call(timeout_ms):
        out = torch.zeros(1, dtype=torch.float32, device=f"cuda:{rank}")
        ex.sum_allreduce(x, x.numel(), out, timeout_ms=timeout_ms, stream=s)
        torch.cuda.synchronize(rank)
        return float(out.item()), ex.status()

    if rank == 0:
        res.append(call(200))
        res.append(call(200))
        q_sig[1].put("go")
        assert q_sig[0].get(timeout=120) == "done"
    else:
        assert q_sig[1].get(timeout=120) == "go"
        res.append(call(5000))
        res.append(call(200))
        q_sig[0].put("done")
    ex.reset()
    q_sig[1 - rank].put("reset")
    assert q_sig[rank].get(timeout=120) == "reset"
    res.append(call(5000))
    q_sig[1 - rank].put("finished")
    assert q_sig[rank].get(timeout=120) == "finished"
    ex.close()
    q_out.put((rank, res))


def test_a_late_rank_never_sees_a_run_ahead():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q_hs, q_sig, q_out = [ctx.Queue() for _ in range(2)], [ctx.Queue() for _ in range(2)], ctx.Queue()
    procs = [ctx.Process(target=_late_worker, args=(r, q_hs, q_sig, q_out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    got = dict(q_out.get(timeout=10) for _ in range(2))
    n = float(1 << 20)
    (a1, st_a1), (a2, st_a2), (a3, st_a3) = got[0]
    (b1, st_b1), (b2, st_b2), (b3, st_b3) = got[1]
    assert np.isnan(a1) and st_a1 & 1 and np.isnan(a2) and st_a2 & 1
    assert b1 == n * 1 + n * 2 and st_b1 == 0          # rank 0's first total was there
    assert np.isnan(b2) and st_b2 & 1                  # rank 0 published nothing for call 2
    assert a3 == b3 == n * 3 and st_a3 == 0 and st_b3 == 0


def _module_worker(rank: int, q_hs, q_out) -> None:
    """A compiled full-array reduction KernelOp with its cross-GPU entry: each
    GPU reduces its own data and every GPU gets the rank-order sum."""
    sys.path.insert(0, str(REPO))
    import torch
    from emmy_ptx_compiler_b200 import harness
    torch.cuda.set_device(rank)
    from conftest import CASES
    ex = _exchange(rank, 2, q_hs)
    res = []
    for cid in ("c4_sum_1048579", "c4_sum_chunk_2p28", "r_max_1024"):
        case = harness.DeviceCase(CASES / cid, rank)
        assert case.bundle["notes"]["cross_gpu_entry"]
        bufs = harness._seeded_device_inputs(case.spec, rank, seed=7 + rank)
        out = case.spec.outputs[0]
        case.launch(bufs)
        torch.cuda.synchronize(rank)
        mine = float(bufs[out].item())
        bufs[out].zero_()
        ex.launch(case.module, [bufs[n] for n in case.spec.arg_order], timeout_ms=5000,
                  stream=torch.cuda.current_stream(rank).cuda_stream)
        torch.cuda.synchronize(rank)
        res.append((cid, mine, float(bufs[out].item())))
        case.module.close()
    st = ex.status()
    q_out.put((rank, res, st))
    torch.cuda.synchronize(rank)
    import time
    time.sleep(1.0)     # the peer's last exchange has long ended before the buffer goes
    ex.close()


def test_compiled_reduction_combines_across_two_gpus():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q_hs, q_out = [ctx.Queue() for _ in range(2)], ctx.Queue()
    procs = [ctx.Process(target=_module_worker, args=(r, q_hs, q_out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
        assert p.exitcode == 0
    got = dict((r, (res, st)) for r, res, st in (q_out.get(timeout=10) for _ in range(2)))
    assert got[0][1] == 0 and got[1][1] == 0
    for (cid, m0, o0), (_, m1, o1) in zip(got[0][0], got[1][0]):
        if cid.startswith("r_max"):
            want = max(m0, m1)
        else:
            want = float(np.float32(np.float32(m0) + np.float32(m1)))
        assert o0 == o1 == want, (cid, o0, o1, want)


@pytest.mark.parametrize("cid", ["c4_sum_1048579", "r_max_1024", "r_mean_777"])
def test_compiled_reduction_exchange_entry_on_one_gpu(cid, cuda_device):
    """A compiled full-array reduction's <entry>__xchg on a group of one GPU
    (it exchanges with itself): the same bits as its plain entry, twice in a
    row, and a clean status word."""
    import torch
    from conftest import CASES
    from emmy_ptx_compiler_b200 import harness, runtime
    case = harness.DeviceCase(CASES / cid, cuda_device)
    assert case.bundle["notes"]["cross_gpu_entry"]
    bufs = harness._seeded_device_inputs(case.spec, cuda_device, seed=21)
    out = case.spec.outputs[0]
    case.launch(bufs)
    torch.cuda.synchronize(cuda_device)
    want = bufs[out].clone()
    ex = runtime.Exchange(cuda_device, 1, 0)
    ex.connect([ex.handle])
    for _ in range(2):
        bufs[out].fill_(float("nan"))
        ex.launch(case.module, [bufs[n] for n in case.spec.arg_order], timeout_ms=2000,
                  stream=torch.cuda.current_stream(cuda_device).cuda_stream)
        torch.cuda.synchronize(cuda_device)
        assert torch.equal(bufs[out].view(torch.int32), want.view(torch.int32))
    assert ex.status() == 0
    ex.close()
    case.module.close()

"""Two GPUs, one process each: row-sharded full-array sum whose per-GPU
partials are combined through the C ABI's NCCL all-reduce
(emmy_comm_init / emmy_allreduce_f32).  Skipped with fewer than 2 GPUs (two
ranks that wait on each other never share one GPU)."""

from __future__ import annotations

import sys

import pytest

from conftest import CASES, REPO

pytestmark = pytest.mark.gpu


def _worker(rank: int, world: int, q_id, q_out) -> None:
    sys.path.insert(0, str(REPO))
    import torch
    from emmy_ptx_compiler_b200 import harness, runtime
    torch.cuda.set_device(rank)
    runtime.init(rank)
    case = harness.DeviceCase(CASES / "c4_sum_1048579", rank)
    n = int(case.spec.args["x"]["shape"][0])
    g = torch.Generator(device=f"cuda:{rank}")
    g.manual_seed(100 + rank)
    x = torch.empty(n, dtype=torch.float32, device=f"cuda:{rank}").uniform_(-1, 1, generator=g)
    part = torch.zeros(1, dtype=torch.float32, device=f"cuda:{rank}")
    case.launch({"x": x, "sum_1": part})
    torch.cuda.synchronize(rank)
    if rank == 0:
        uid = runtime.Comm.unique_id()
        for _ in range(world - 1):
            q_id.put(uid)
    else:
        uid = q_id.get(timeout=60)
    comm = runtime.Comm(rank, world, rank, uid, timeout_ms=60000)
    total = torch.zeros(1, dtype=torch.float32, device=f"cuda:{rank}")
    comm.allreduce_f32(part.data_ptr(), total.data_ptr(), 1,
                       stream=torch.cuda.current_stream(rank).cuda_stream, timeout_ms=60000)
    ref = float(x.double().sum().item())
    q_out.put((rank, float(part.item()), ref, float(total.item())))
    comm.close()
    case.module.close()


def test_sharded_sum_with_nccl_combine():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q_id, q_out = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, q_id, q_out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    res = sorted(q_out.get(timeout=10) for _ in range(2))
    want = sum(r[2] for r in res)
    for rank, part, ref, total in res:
        assert abs(part - ref) <= 1e-5 * abs(ref) + 1e-3
        assert abs(total - want) <= 1e-5 * abs(want) + 2e-3
    assert res[0][3] == res[1][3], "every rank sees the same combined sum"

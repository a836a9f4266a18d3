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


@pytest.mark.parametrize("cid", ["c2_gelu_256x4096", "c5_gemm_384x1024x768", "c5_gemm_200x136x300",
                                 "f_softmax_64x1000", "a_attn_100x48"])
def test_sharded_launch_matches_one_gpu(cid):
    """emmy_launch_sharded over 2 GPUs from one process: each device holds only
    its shard of the streamed parameters (rows of x / y, rows of A / C) and a
    full copy of the rest; the gathered result is bit-identical to one launch
    on one GPU."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    sys.path.insert(0, str(REPO))
    from emmy_ptx_compiler_b200 import harness, runtime
    case = harness.DeviceCase(CASES / cid, 0)
    bufs = harness._seeded_device_inputs(case.spec, 0, seed=3)
    case.launch(bufs)
    torch.cuda.synchronize(0)
    want = {n: bufs[n].clone() for n in case.spec.outputs}
    mods = [case.module, runtime.Module(case.bundle["cubin"], case.spec.entry, 1)]
    total, align, per_unit = case.module.unit_range()
    args, outs = [], []
    for d in range(2):
        b, e = runtime.shard_range(mods[d], 2, d)
        row = []
        shard_out = {}
        for k, n in enumerate(case.spec.arg_order):
            full = bufs[n] if n not in case.spec.outputs else torch.zeros_like(bufs[n])
            flat = full.reshape(-1)
            if per_unit[k]:
                per = per_unit[k] // full.element_size()
                t = flat[b * per:e * per].to(f"cuda:{d}").clone()
            else:
                t = full.to(f"cuda:{d}").clone()
            if n in case.spec.outputs:
                shard_out[n] = (t, per_unit[k] // full.element_size() if per_unit[k] else None)
            row.append(t)
        args.append(row)
        outs.append(shard_out)
    runtime.launch_sharded(mods, args)
    for d in range(2):
        torch.cuda.synchronize(d)
    for n in case.spec.outputs:
        parts = [outs[d][n][0].reshape(-1).to("cuda:0") for d in range(2)]
        got = torch.cat(parts)
        assert torch.equal(got.view(torch.uint8), want[n].reshape(-1).view(torch.uint8)), \
            f"{cid}.{n}: sharded launch differs from the one-GPU launch"
    assert mods[0].status() == 0 and mods[1].status() == 0
    mods[1].close()
    case.module.close()

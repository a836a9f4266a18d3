"""Device helpers that restate a correctly rounded operation another way must
give CUDA's own results bit for bit.

``emmy_div_by(x, y, RN(1/y), ok)`` (the row-fused kernels' division by a
per-row value, Markstein's correction) against ``__fdiv_rn(x, y)``: random
bit patterns of every sign and exponent (NaN, infinity, zero and subnormals
included), softmax-like operands, divisors with all-ones mantissas and powers
of two, quotients near underflow and overflow, and dividends with all-ones
mantissas.
"""

from __future__ import annotations

import pytest

pytestmark = pytest.mark.gpu

CHECK_SRC = r"""
extern "C" __global__ void div_check(const float *a, const float *b, unsigned long long n,
                                     unsigned long long *bad, float *example) {
    for (unsigned long long i = blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x; i < n;
         i += (unsigned long long)gridDim.x * blockDim.x) {
        const float x = a[i], y = b[i];
        const float p = __fdiv_rn(x, y);
        const float q = emmy_div_by(x, y, __frcp_rn(y), emmy_div_ok(y));
        if (__float_as_uint(p) != __float_as_uint(q) && !(p != p && q != q)) {
            const unsigned long long k = atomicAdd(bad, 1ull);
            if (k < 4) { example[3 * k] = x; example[3 * k + 1] = y; example[3 * k + 2] = q; }
        }
    }
}
"""


def _operands(kind: int, n: int, g):
    import torch
    dev = "cuda:0"
    bits_a = torch.randint(0, 1 << 32, (n,), device=dev, generator=g, dtype=torch.int64)
    bits_b = torch.randint(0, 1 << 32, (n,), device=dev, generator=g, dtype=torch.int64)
    as_f32 = lambda t: (t & 0xFFFFFFFF).to(torch.int64).sub(((t & 0x80000000) != 0).to(torch.int64) << 32) \
        .to(torch.int32).view(torch.float32)  # noqa: E731
    if kind == 0:
        return as_f32(bits_a), as_f32(bits_b)
    if kind == 1:
        return torch.rand(n, device=dev, generator=g), 1 + 8191 * torch.rand(n, device=dev, generator=g)
    if kind == 2:
        mant = torch.where(bits_b % 2 == 0, torch.full_like(bits_b, 0x7FFFFF), torch.zeros_like(bits_b))
        expo = 1 + (bits_b >> 1) % 253
        return torch.randn(n, device=dev, generator=g), as_f32((expo << 23) | mant)
    if kind == 3:
        return (torch.randn(n, device=dev, generator=g) * 1e-30, torch.randn(n, device=dev, generator=g) * 1e8)
    if kind == 4:
        return (torch.randn(n, device=dev, generator=g) * 1e30, torch.randn(n, device=dev, generator=g) * 1e-8)
    expo = 64 + (bits_a >> 8) % 128
    return as_f32((expo << 23) | (0x7FFFFF - bits_a % 4)), 1 + torch.rand(n, device=dev, generator=g)


@pytest.mark.parametrize("kind", range(6))
def test_div_by_reciprocal_matches_fdiv_rn(kind, cuda_device):
    import torch
    from emmy_ptx_compiler_b200 import cgen, runtime, toolchain
    mod = runtime.Module(toolchain.build(cgen.DEVICE_PRELUDE + CHECK_SRC, kind="cubin", name="div_check"),
                         "div_check", cuda_device)
    g = torch.Generator(device="cuda:0")
    g.manual_seed(100 + kind)
    n = 1 << 24
    a, b = (t.contiguous() for t in _operands(kind, n, g))
    bad = torch.zeros(1, dtype=torch.int64, device="cuda:0")
    example = torch.zeros(12, device="cuda:0")
    mod.launch([a, b, n, bad, example], grid=(592, 1, 1), block=(256, 1, 1))
    torch.cuda.synchronize(cuda_device)
    assert int(bad.item()) == 0, f"{int(bad.item())} mismatches, e.g. (x, y, got) {example[:3].tolist()}"
    mod.close()

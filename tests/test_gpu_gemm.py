"""tcgen05 GEMM layouts (K-major / MN-major operands, bf16 / fp16, ragged shapes) against torch."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _run(dtype, a_mn, b_mn, M, N, K, seed=0, pair=False, wide=False):
    from orda_ce_kernel import _native

    lib = _native.load()
    g = torch.Generator(device="cuda").manual_seed(seed)
    A = torch.randn(M, K, device="cuda", generator=g).to(dtype)
    B = torch.randn(N, K, device="cuda", generator=g).to(dtype)
    # storage in the requested major-ness: MN-major stores the transpose contiguously
    a_store = A.t().contiguous() if a_mn else A.contiguous()
    b_store = B.t().contiguous() if b_mn else B.contiguous()
    out = torch.full((M, N), float("nan"), device="cuda", dtype=torch.float32)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    code = {torch.bfloat16: _native.BF16, torch.float16: _native.F16}[dtype]
    fn = lib.orda_debug_gemm_wide if wide else (lib.orda_debug_gemm_pair if pair else lib.orda_debug_gemm)
    rc = fn(code, int(a_mn), int(b_mn), a_store.data_ptr(), a_store.stride(0),
                             b_store.data_ptr(), b_store.stride(0), M, N, K, out.data_ptr(), out.stride(0),
                             status.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _native.status_string(rc)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    ref = A.float() @ B.float().t()
    return out, ref


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, True), (True, False)])
def test_gemm_layouts_exact_tiles(dtype, a_mn, b_mn):
    out, ref = _run(dtype, a_mn, b_mn, 256, 512, 256)
    torch.testing.assert_close(out, ref, rtol=1e-3, atol=1e-3)


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, True)])
@pytest.mark.parametrize("shape", [(130, 300, 72), (1, 40, 8), (300, 257, 1000), (1000, 1000, 520)])
def test_gemm_layouts_ragged(a_mn, b_mn, shape):
    M, N, K = shape
    if a_mn and M % 8:
        M += 8 - M % 8  # MN-major rows of 16-bit data need 16-byte strides
    if b_mn and N % 8:
        N += 8 - N % 8
    if not a_mn and K % 8:
        K += 8 - K % 8
    out, ref = _run(torch.bfloat16, a_mn, b_mn, M, N, K, seed=1)
    torch.testing.assert_close(out, ref, rtol=2e-3, atol=2e-3)


def test_gemm_many_tiles_persistent():
    out, ref = _run(torch.bfloat16, False, False, 2048, 4096, 512, seed=2)
    torch.testing.assert_close(out, ref, rtol=2e-3, atol=2e-3)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, True), (True, False)])
@pytest.mark.parametrize("shape", [(512, 512, 256), (300, 264, 1000), (1, 40, 8), (2048, 4096, 512)])
def test_pair_gemm_layouts(dtype, a_mn, b_mn, shape):
    """CTA-pair (cta_group::2) kernel: every operand layout, exact and ragged shapes."""
    M, N, K = shape
    if a_mn and M % 8:
        M += 8 - M % 8
    if b_mn and N % 8:
        N += 8 - N % 8
    if not a_mn and K % 8:
        K += 8 - K % 8
    out, ref = _run(dtype, a_mn, b_mn, M, N, K, seed=5, pair=True)
    torch.testing.assert_close(out, ref, rtol=2e-3, atol=2e-3)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, True), (True, False)])
@pytest.mark.parametrize("shape", [(512, 512, 256), (520, 264, 1000), (1, 40, 8), (2048, 4096, 512), (1536, 768, 64)])
def test_wide_gemm_layouts(dtype, a_mn, b_mn, shape):
    """Wide CTA-pair kernel (512 x 256 tiles, two accumulators, split accumulator release): every
    operand layout; ragged shapes; K shorter than the pipeline (a single k block)."""
    M, N, K = shape
    if a_mn and M % 8:
        M += 8 - M % 8
    if b_mn and N % 8:
        N += 8 - N % 8
    if not a_mn and K % 8:
        K += 8 - K % 8
    out, ref = _run(dtype, a_mn, b_mn, M, N, K, seed=7, wide=True)
    torch.testing.assert_close(out, ref, rtol=2e-3, atol=2e-3)

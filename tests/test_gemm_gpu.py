"""The tcgen05 GEMM against an fp32 torch product of the same bf16 operands, in every operand
orientation, at ragged and at step shapes (fp32 accumulation: differences come only from the
summation order and the output rounding)."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(a, b_t, bias=None):
    r = a.float() @ b_t.float().t()
    return r if bias is None else r + bias.float()


def _check(out, ref, out_dtype):
    if out_dtype == torch.float32:
        torch.testing.assert_close(out, ref, rtol=1e-3, atol=1e-3)
    else:
        torch.testing.assert_close(out.float(), ref, rtol=1.6e-2, atol=1e-2)


@pytest.mark.parametrize("a_t", [False, True])
@pytest.mark.parametrize("b_t", [False, True])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_gemm_orientations(cuda, a_t, b_t, out_dtype):
    from hackathon_b200.gemm import device_error, gemm
    torch.manual_seed(0)
    M, N, K = 384, 512, 320
    a = torch.randn(K, M, device=cuda).to(torch.bfloat16).t() if a_t else \
        torch.randn(M, K, device=cuda).to(torch.bfloat16)
    b = torch.randn(K, N, device=cuda).to(torch.bfloat16).t() if b_t else \
        torch.randn(N, K, device=cuda).to(torch.bfloat16)
    out = gemm(a, b, out_dtype=out_dtype)
    device_error()
    _check(out, _ref(a, b), out_dtype)


@pytest.mark.parametrize("shape", [(1, 1, 1), (127, 255, 63), (129, 257, 65), (200, 1000, 96),
                                   (1000, 136, 2048)])
def test_gemm_ragged_edges(cuda, shape):
    from hackathon_b200.gemm import device_error, gemm
    M, N, K = shape
    torch.manual_seed(1)
    # leading dims padded to a multiple of 8 elements (16-byte rows), views cut to the shape
    lda, ldb = (K + 7) // 8 * 8, (K + 7) // 8 * 8
    a = torch.randn(M, lda, device=cuda).to(torch.bfloat16)[:, :K]
    b = torch.randn(N, ldb, device=cuda).to(torch.bfloat16)[:, :K]
    bias = torch.randn(N, device=cuda)
    out = gemm(a, b, out_dtype=torch.float32, bias=bias)
    device_error()
    _check(out, _ref(a, b, bias), torch.float32)


@pytest.mark.parametrize("shape", [(16384, 3584, 3584), (4096, 18944, 3584),
                                   (4096, 3584, 18944)])
def test_gemm_step_shapes(cuda, shape):
    """7B projection shapes (x W^T) against cuBLAS-free fp32 reference on a row sample."""
    from hackathon_b200.gemm import device_error, gemm
    M, N, K = shape
    g = torch.Generator(device=cuda).manual_seed(2)
    a = torch.randn(M, K, device=cuda, generator=g).to(torch.bfloat16)
    b = (torch.randn(N, K, device=cuda, generator=g) * 0.02).to(torch.bfloat16)
    out = gemm(a, b, out_dtype=torch.bfloat16)
    device_error()
    rows = torch.tensor([0, 1, 127, 128, M // 2, M - 1], device=cuda)
    ref = a[rows].float() @ b.float().t()
    torch.testing.assert_close(out[rows].float(), ref, rtol=1.6e-2, atol=2e-2)


def test_gemm_misaligned_rows(cuda):
    """Rows that are not whole 16-byte units: the C-ABI refuses them (a tensor map's row stride),
    the Python wrapper copies such operands into padded rows and computes the product."""
    from hackathon_b200 import _lib
    from hackathon_b200.gemm import device_error, gemm
    a = torch.randn(64, 67, device=cuda).to(torch.bfloat16)   # 134-byte rows
    b = torch.randn(64, 67, device=cuda).to(torch.bfloat16)
    c = torch.empty(64, 64, device=cuda, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="16"):
        _lib.call("qb_gemm_bf16", a.data_ptr(), 67, 0, b.data_ptr(), 67, 0, c.data_ptr(), 64,
                  _lib.tag(c.dtype), None, 64, 64, 67, _lib.stream(a.device))
    out = gemm(a, b)
    device_error()
    torch.testing.assert_close(out.float(), a.float() @ b.float().t(), rtol=1.6e-2, atol=2e-2)


@pytest.mark.parametrize("b_t", [False, True])
@pytest.mark.parametrize("shape", [(384, 512, 320, 64), (129, 257, 200, 16), (1, 300, 64, 8),
                                   (1000, 136, 2048, 100)])
def test_gemm2_two_segments(cuda, shape, b_t):
    """C = A0 B0^T + A1 B1^T in one accumulation (qb_gemm2_bf16): both B layouts, ragged M/N and
    segment lengths that are not multiples of the 64-wide k-block."""
    from hackathon_b200.gemm import device_error, gemm2
    M, N, K0, K1 = shape
    g = torch.Generator(device=cuda).manual_seed(4)

    def pad(n):   # leading dims padded to 16-byte rows, views cut to the shape
        return (n + 7) // 8 * 8

    def b_op(k):
        if b_t:   # transposed view of a row-major [k, N]: read MN-major
            return torch.randn(k, pad(N), device=cuda, generator=g).to(torch.bfloat16)[:, :N].t()
        return torch.randn(N, pad(k), device=cuda, generator=g).to(torch.bfloat16)[:, :k]

    a0 = torch.randn(M, pad(K0), device=cuda, generator=g).to(torch.bfloat16)[:, :K0]
    a1 = torch.randn(M, pad(K1), device=cuda, generator=g).to(torch.bfloat16)[:, :K1]
    b0, b1 = b_op(K0), b_op(K1)
    bias = torch.randn(N, device=cuda, generator=g)
    for out_dtype in (torch.float32, torch.bfloat16):
        out = gemm2(a0, b0, a1, b1, out_dtype=out_dtype, bias=bias)
        device_error()
        _check(out, _ref(a0, b0, bias) + a1.float() @ b1.float().t(), out_dtype)


def test_gemm2_mixed_b_layouts(cuda):
    """A row-major B1 next to a transposed-view B0 is brought to one layout on the host."""
    from hackathon_b200.gemm import device_error, gemm2
    g = torch.Generator(device=cuda).manual_seed(5)
    a0 = torch.randn(256, 128, device=cuda, generator=g).to(torch.bfloat16)
    b0 = torch.randn(128, 384, device=cuda, generator=g).to(torch.bfloat16).t()
    a1 = torch.randn(256, 64, device=cuda, generator=g).to(torch.bfloat16)
    b1 = torch.randn(384, 64, device=cuda, generator=g).to(torch.bfloat16)
    out = gemm2(a0, b0, a1, b1, out_dtype=torch.float32)
    device_error()
    _check(out, _ref(a0, b0) + _ref(a1, b1), torch.float32)


@pytest.mark.parametrize("shape", [(16384, 3584, 3584), (16384, 512, 3584)])
def test_gemm2_projection_step_shape(cuda, shape):
    """A 7B projection with its rank-64 LoRA term at the step's token count, sampled rows."""
    from hackathon_b200.gemm import device_error, gemm2
    M, N, K = shape
    g = torch.Generator(device=cuda).manual_seed(6)
    x = torch.randn(M, K, device=cuda, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device=cuda, generator=g) * 0.02).to(torch.bfloat16)
    u = torch.randn(M, 64, device=cuda, generator=g).to(torch.bfloat16)
    sb = (torch.randn(N, 64, device=cuda, generator=g) * 0.05).to(torch.bfloat16)
    out = gemm2(x, w, u, sb)
    device_error()
    rows = torch.tensor([0, 1, 127, 128, 2047, 2048, M // 2, M - 1], device=cuda)
    ref = x[rows].float() @ w.float().t() + u[rows].float() @ sb.float().t()
    torch.testing.assert_close(out[rows].float(), ref, rtol=1.6e-2, atol=2e-2)


@pytest.mark.parametrize("b_t", [False, True])
@pytest.mark.parametrize("shape", [(2048, 1000, 200), (2560, 1330, 96), (4096, 1800, 136)])
def test_gemm_ragged_bf16_both_b_layouts(cuda, shape, b_t):
    """Multi-wave shapes with a ragged last tile in N and K, for both B layouts, single- and
    two-segment, bf16 output."""
    from hackathon_b200.gemm import device_error, gemm, gemm2
    M, N, K = shape
    g = torch.Generator(device=cuda).manual_seed(7)
    a = torch.randn(M, K, device=cuda, generator=g).to(torch.bfloat16)
    if b_t:
        b = torch.randn(K, (N + 7) // 8 * 8, device=cuda, generator=g).to(torch.bfloat16)[:, :N].t()
    else:
        b = torch.randn(N, K, device=cuda, generator=g).to(torch.bfloat16)
    out = gemm(a, b)
    u = torch.randn(M, 64, device=cuda, generator=g).to(torch.bfloat16)
    if b_t:
        v = torch.randn(64, (N + 7) // 8 * 8, device=cuda, generator=g).to(torch.bfloat16)[:, :N].t()
    else:
        v = torch.randn(N, 64, device=cuda, generator=g).to(torch.bfloat16)
    out2 = gemm2(a, b, u, v)
    device_error()
    _check(out, _ref(a, b), torch.bfloat16)
    _check(out2, _ref(a, b) + _ref(u, v), torch.bfloat16)


@pytest.mark.parametrize("shape", [(300, 1000, 64), (16384, 3584, 64), (129, 200, 16),
                                   (2048, 640, 128), (777, 18944, 64)])
@pytest.mark.parametrize("b_t", [True, False])
def test_gemm_mask_acc(cuda, shape, b_t):
    """C += s * mask .* (A B^T) with the dropout bit words (qb_gemm_bf16_mask_acc): against the
    fp32 product masked on the host from the same bits, one rounding of C + s * acc."""
    from hackathon_b200.gemm import device_error, gemm_mask_acc
    M, N, K = shape
    g = torch.Generator(device=cuda).manual_seed(8)
    a = torch.randn(M, K, device=cuda, generator=g).to(torch.bfloat16)
    if b_t:   # [K, N] row-major, used transposed (the LoRA A matrix [r, in])
        b = (torch.randn(K, (N + 7) // 8 * 8, device=cuda, generator=g) * 0.1).to(torch.bfloat16)[:, :N].t()
    else:
        b = (torch.randn(N, K, device=cuda, generator=g) * 0.1).to(torch.bfloat16)
    words = (N + 31) // 32
    bits = torch.randint(-2**31, 2**31 - 1, (M, words), device=cuda, dtype=torch.int64,
                         generator=g).to(torch.int32)
    c0 = torch.randn(M, (N + 7) // 8 * 8, device=cuda, generator=g).to(torch.bfloat16)[:, :N]
    c = c0.clone()
    gemm_mask_acc(a, b, bits, 1.25, c)
    device_error()
    cols = torch.arange(N, device=cuda)
    mask = ((bits.long()[:, cols // 32] >> (cols % 32)) & 1).bool()
    ref = c0.float() + torch.where(mask, 1.25 * (a.float() @ b.float().t()), 0.0)
    torch.testing.assert_close(c.float(), ref, rtol=1.6e-2, atol=2e-2)
    # masked-out elements are untouched, bit for bit
    assert torch.equal(c.view(torch.int16)[~mask], c0.contiguous().view(torch.int16)[~mask])


@pytest.mark.parametrize("lora", [False, True])
def test_gemm2_residual_epilogue(cuda, lora):
    """out = residual + A0 B0^T (+ A1 B1^T) (+ bias) in one accumulation and one rounding."""
    from hackathon_b200.gemm import device_error, gemm2
    g = torch.Generator(device=cuda).manual_seed(9)
    M, N, K = 1000, 640, 320
    a = torch.randn(M, K, device=cuda, generator=g).to(torch.bfloat16)
    b = (torch.randn(N, K, device=cuda, generator=g) * 0.05).to(torch.bfloat16)
    res = torch.randn(M, N, device=cuda, generator=g).to(torch.bfloat16)
    bias = torch.randn(N, device=cuda, generator=g)
    u = torch.randn(M, 64, device=cuda, generator=g).to(torch.bfloat16) if lora else None
    sb = (torch.randn(N, 64, device=cuda, generator=g) * 0.05).to(torch.bfloat16) if lora else None
    out = gemm2(a, b, u, sb, bias=bias, residual=res)
    device_error()
    ref = res.float() + a.float() @ b.float().t() + bias
    if lora:
        ref = ref + u.float() @ sb.float().t()
    torch.testing.assert_close(out.float(), ref, rtol=1.6e-2, atol=2e-2)


@pytest.mark.parametrize("accumulate", [True, False])
@pytest.mark.parametrize("a_t", [False, True])
@pytest.mark.parametrize("b_t", [False, True])
@pytest.mark.parametrize("shape", [(3584, 64, 16384), (64, 3584, 16384), (512, 64, 16384),
                                   (200, 100, 1000), (129, 130, 200), (1, 64, 64),
                                   (300, 257, 4096)])
def test_gemm_acc_f32_split_k(cuda, shape, a_t, b_t, accumulate):
    """C (fp32) = (C or 0) + alpha A B^T with the tokens split across the SMs (the LoRA weight
    gradients: [in, r] / [r, in] / [out, r] outputs, K = 16384), every orientation, ragged shapes
    and narrow tiles, accumulating into a C that already holds values or overwriting one that
    holds NaN, against fp32 torch; a second run gives the same bits (the splits are summed in a
    fixed order)."""
    from hackathon_b200 import _lib
    from hackathon_b200.gemm import device_error, gemm_acc_f32
    M, N, K = shape
    g = torch.Generator(device=cuda).manual_seed(M + N + K)
    a = torch.randn(K, M, device=cuda, generator=g).to(torch.bfloat16).t() if a_t else \
        torch.randn(M, K, device=cuda, generator=g).to(torch.bfloat16)
    b = torch.randn(K, N, device=cuda, generator=g).to(torch.bfloat16).t() if b_t else \
        torch.randn(N, K, device=cuda, generator=g).to(torch.bfloat16)
    c0 = torch.randn(M, N, device=cuda, generator=g) if accumulate else \
        torch.full((M, N), float("nan"), device=cuda)     # without accumulate C is not read
    out = gemm_acc_f32(a, b, c0.clone(), alpha=0.5, accumulate=accumulate)
    again = gemm_acc_f32(a, b, c0.clone(), alpha=0.5, accumulate=accumulate)
    device_error()
    ref = 0.5 * (a.float() @ b.float().t())
    if accumulate:
        ref = c0 + ref
    torch.testing.assert_close(out, ref, rtol=1e-3, atol=2e-3 * (K ** 0.5) / 8)
    assert torch.equal(out, again)
    if shape == (3584, 64, 16384):     # 28 tiles of a 256-k-block K: the split path ran
        assert _lib.load().qb_gemm_bf16_acc_f32_workspace(M, N, K) > 0


@pytest.mark.parametrize("shape", [(16384, 64, 3584), (16384, 64, 18944), (300, 64, 200),
                                   (1000, 100, 96), (16384, 128, 512)])
def test_gemm_narrow_tiles(cuda, shape):
    """Outputs of at most 64 / 128 columns run 64- / 128-wide tiles (V = g (s B), U = xd A^T):
    the same products as the 256-wide kernel, against fp32 torch."""
    from hackathon_b200.gemm import device_error, gemm
    M, N, K = shape
    g = torch.Generator(device=cuda).manual_seed(N + K)
    a = torch.randn(M, K, device=cuda, generator=g).to(torch.bfloat16)
    b = torch.randn(K, N, device=cuda, generator=g).to(torch.bfloat16)
    out = gemm(a, b.t())                      # b.t(): the MN-major view the step passes
    device_error()
    _check(out, _ref(a, b.t()), torch.bfloat16)


def test_lora_products_match_torch(cuda):
    """The LoRA branch's backward products of one projection (V, dA, dB) on the tcgen05 GEMMs
    against the fp32 torch products, at the 7B o-projection shape (T = 16384, r = 64)."""
    from hackathon_b200.gemm import device_error, lora_products
    T, out_f, in_f, r, s = 16384, 3584, 3584, 64, 2.0
    g = torch.Generator(device=cuda).manual_seed(7)
    gy = torch.randn(T, out_f, device=cuda, generator=g).to(torch.bfloat16)
    u = torch.randn(T, 2 * r, device=cuda, generator=g).to(torch.bfloat16)[:, r:]   # a slice
    xd = torch.randn(T, in_f, device=cuda, generator=g).to(torch.bfloat16)
    sb = (torch.randn(out_f, r, device=cuda, generator=g) * 0.05).to(torch.bfloat16)
    v, da, db = lora_products(gy, u, xd, sb, (r, in_f), s)
    device_error()
    v_ref = gy.float() @ sb.float()
    torch.testing.assert_close(v.float(), v_ref, rtol=1.6e-2, atol=5e-2)
    da_ref = v.float().t() @ xd.float()
    db_ref = s * (gy.float().t() @ u.float())
    for got, want in ((da, da_ref), (db, db_ref)):
        assert got.dtype == torch.float32 and got.is_contiguous()
        assert float((got - want).norm() / want.norm()) < 1e-3

"""Parity of the CUDA ops (called through the C-ABI) with the reference: against the fixtures the
reference's kernels produced, and against the pinned CPU oracle on seeded inputs, at the
reference's test shapes and at BASELINE shapes. Tolerances follow the reference's tests
(solution/_testing.py:12 TOL, test_*.py) and the stated bars: NF4 bit-exact; RMSNorm / RoPE /
SwiGLU within atol 1e-2 / rtol 1.6e-2 in bf16."""

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import nf4_ref, ops_ref

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-5, torch.float16: 2e-3, torch.bfloat16: 1.6e-2}
BF16_ATOL = 1e-2


def _t(a, dev, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return t if dtype is None else t.to(dtype)


# ----------------------------------------------------------------------------------- NF4

def _state_from_golden(g, i, dev):
    from hackathon_b200.nf4 import QuantState
    rows, cols, bs, nested, bs2 = (int(v) for v in g[f"nf4_{i}_meta"])
    if nested:
        s2 = QuantState(absmax=_t(g[f"nf4_{i}_absmax2"], dev), code=_t(g["nf4_code2"], dev),
                        blocksize=bs2, quant_type="dynamic")
        return QuantState(absmax=_t(g[f"nf4_{i}_absmax_q"], dev), shape=(rows, cols),
                          blocksize=bs, offset=float(g[f"nf4_{i}_offset"][0]), state2=s2)
    return QuantState(absmax=_t(g[f"nf4_{i}_absmax"], dev), shape=(rows, cols), blocksize=bs)


def test_nf4_dequant_bit_exact_vs_reference_fixtures(cuda):
    from hackathon_b200.nf4 import dequantize_nf4
    g = golden("nf4")
    for i in range(5):
        st = _state_from_golden(g, i, cuda)
        packed = _t(g[f"nf4_{i}_packed"], cuda).reshape(-1, 1)
        ref32 = g[f"nf4_{i}_f32"]
        out32 = dequantize_nf4(packed, st, torch.float32).cpu().numpy()
        out16 = dequantize_nf4(packed, st, torch.float16).cpu().numpy()
        outbf = dequantize_nf4(packed, st, torch.bfloat16).cpu().view(torch.int16).numpy()
        assert np.array_equal(out32.view(np.uint32), ref32.view(np.uint32)), i
        assert np.array_equal(out16.view(np.uint16), g[f"nf4_{i}_f16"].view(np.uint16)), i
        assert np.array_equal(outbf.view(np.uint16), nf4_ref.f32_to_bf16_bits(ref32)), i


def _oracle_rows(packed_u8, q, absmax2, code2, offset, cols, rows_idx, bs=64, bs2=256):
    """Oracle bf16 bits of whole rows of a nested-NF4 matrix."""
    return np.stack([nf4_ref.dequant_nf4(packed_u8, cols, q, True, code2, absmax2, offset, bs,
                                         bs2, out="bf16", start=r * cols) for r in rows_idx])


@pytest.mark.parametrize("shape", [(3584, 3584), (512, 3584), (18944, 3584), (3584, 18944)])
def test_nf4_quantize_dequant_baseline_shapes(cuda, shape):
    """Cfg2 shapes: GPU quantiser -> GPU dequant (bf16). The WHOLE matrix is checked bit for bit
    against the C restatement of the reference's dequant (oracle/nf4_ref.c, every weight), a few
    rows also against the numpy oracle (which pins the C one), and the matrix against the
    quantisation error bound."""
    from hackathon_b200.nf4 import dequantize_nf4, quantize_nf4
    from oracle import c_ref, cpu_step
    gen = torch.Generator(device=cuda).manual_seed(0)
    w = (torch.randn(shape, generator=gen, device=cuda) * 0.02).to(torch.bfloat16)
    packed, st = quantize_nf4(w)
    out = dequantize_nf4(packed, st, torch.bfloat16)
    packed_h = packed.cpu().numpy().reshape(-1)
    q_h, a2_h = st.absmax.cpu().numpy(), st.state2.absmax.cpu().numpy()
    code2_h = st.state2.code.cpu().numpy()
    got_all = out.cpu().view(torch.int16).numpy().view(np.uint16).reshape(-1)
    want_all = c_ref.dequant_nf4_bf16(packed_h, w.numel(), q_h, code2_h, a2_h, st.offset, 64,
                                      256, threads=cpu_step.usable_cores())
    bad = np.flatnonzero(got_all != want_all)
    assert bad.size == 0, f"{bad.size} of {w.numel()} weights differ, first at {bad[:4]}"
    rows = [0, 1, shape[0] // 2, shape[0] - 1]
    want = _oracle_rows(packed_h, q_h, a2_h, code2_h, st.offset, shape[1], rows)
    assert np.array_equal(want_all.reshape(shape)[rows], want)
    blocks = w.float().abs().reshape(-1, 64).amax(1).repeat_interleave(64).view(shape)
    assert torch.all((out.float() - w.float()).abs() <= 0.17 * blocks + 1e-6)


def test_nf4_quantiser_matches_oracle(cuda):
    from hackathon_b200.nf4 import quantize_nf4, signed_dynamic_code
    rng = np.random.default_rng(5)
    w = (rng.standard_normal((192, 640)) * 0.03).astype(np.float32)
    packed, st = quantize_nf4(_t(w, cuda), compress_statistics=False)
    ref_packed, ref_absmax = nf4_ref.quantize_nf4(w, 64)
    assert np.array_equal(packed.cpu().numpy().reshape(-1), ref_packed)
    assert np.array_equal(st.absmax.cpu().numpy(), ref_absmax)
    packed2, st2 = quantize_nf4(_t(w, cuda), compress_statistics=True)
    q, a2, off = nf4_ref.double_quant(ref_absmax, signed_dynamic_code().numpy(), 256)
    assert abs(st2.offset - float(off)) <= 1e-6 * abs(float(off))
    np.testing.assert_allclose(st2.state2.absmax.cpu().numpy(), a2, rtol=1e-5)
    assert (st2.absmax.cpu().numpy() != q).mean() < 0.01


@pytest.mark.parametrize("bs,n", [(2, 10), (6, 36), (64, 64 * 7 + 2), (32, 1024)])
def test_nf4_dequant_generic_blocksizes(cuda, bs, n):
    """Block sizes the word path does not take (any even size) and ragged lengths."""
    from hackathon_b200.nf4 import QuantState, dequantize_nf4
    rng = np.random.default_rng(bs)
    w = (rng.standard_normal(n) * 0.05).astype(np.float32)
    packed, absmax = nf4_ref.quantize_nf4(w, bs)
    st = QuantState(absmax=_t(absmax, cuda), shape=(1, n), blocksize=bs)
    out = dequantize_nf4(_t(packed, cuda), st, torch.float32).cpu().numpy().reshape(-1)
    ref = nf4_ref.dequant_nf4(packed, n, absmax, False, None, None, 0.0, bs, 2, out="f32")
    assert np.array_equal(out.view(np.uint32), ref.view(np.uint32))


def test_nf4_rejects_bad_blocksize(cuda):
    from hackathon_b200.nf4 import QuantState, dequantize_nf4
    st = QuantState(absmax=torch.ones(4, device=cuda), shape=(2, 8), blocksize=3)
    with pytest.raises(RuntimeError, match="blocksize"):
        dequantize_nf4(torch.zeros(8, dtype=torch.uint8, device=cuda), st, torch.float16)


def test_nf4_linear_forward_backward(cuda):
    from hackathon_b200.nf4 import NF4Linear, dequantize_nf4, quantize_nf4
    torch.manual_seed(0)
    w = (torch.randn(256, 512, device=cuda) * 0.02).to(torch.bfloat16)
    packed, st = quantize_nf4(w)
    bias = torch.randn(256, device=cuda, dtype=torch.bfloat16)
    x = torch.randn(4, 33, 512, device=cuda, dtype=torch.bfloat16, requires_grad=True)
    y = NF4Linear.apply(x, packed, st, bias)
    wd = dequantize_nf4(packed, st, torch.bfloat16)
    xr = x.detach().float().requires_grad_()
    yr = torch.nn.functional.linear(xr, wd.float(), bias.float())
    torch.testing.assert_close(y.float(), yr, rtol=1.6e-2, atol=2e-2)
    g = torch.randn_like(y)
    y.backward(g)
    yr.backward(g.float())
    torch.testing.assert_close(x.grad.float(), xr.grad, rtol=1.6e-2, atol=2e-2)


# ----------------------------------------------------------------------------------- RMSNorm

@pytest.mark.parametrize("i", range(6))
def test_rmsnorm_vs_reference_fixtures(cuda, i):
    from hackathon_b200.rmsnorm import rmsnorm
    g = golden("rmsnorm")
    x = _t(g[f"rms_{i}_x"], cuda).requires_grad_()
    w = _t(g[f"rms_{i}_w"], cuda)
    y = rmsnorm(x, w, 1e-6)
    ref = _t(g[f"rms_{i}_y"], cuda)
    assert y.dtype == ref.dtype
    tol = TOL[x.dtype]
    torch.testing.assert_close(y, ref, rtol=tol, atol=tol)
    y.backward(_t(g[f"rms_{i}_g"], cuda))
    assert x.grad.dtype == x.dtype
    torch.testing.assert_close(x.grad, _t(g[f"rms_{i}_dx"], cuda), rtol=tol, atol=tol)


@pytest.mark.parametrize("x_dtype,w_dtype", [(torch.float32, torch.float32),
                                             (torch.float16, torch.float32),
                                             (torch.float16, torch.float16),
                                             (torch.bfloat16, torch.bfloat16),
                                             (torch.bfloat16, torch.float32)])
@pytest.mark.parametrize("hidden", [1536, 1000, 3584, 896, 1001])
def test_rmsnorm_vs_oracle(cuda, x_dtype, w_dtype, hidden):
    from hackathon_b200.rmsnorm import rmsnorm
    torch.manual_seed(0)
    weight = (1 + 0.1 * torch.randn(hidden)).to(w_dtype)
    x = torch.randn(4, 512, hidden, dtype=x_dtype)
    dy = torch.randn(4, 512, hidden)
    xr = x.clone().requires_grad_()
    yr = ops_ref.rmsnorm_ref(xr, weight, 1e-6)
    yr.backward(dy.to(yr.dtype))
    xg = x.to(cuda).requires_grad_()
    y = rmsnorm(xg, weight.to(cuda), 1e-6)
    assert y.dtype == yr.dtype and y.shape == yr.shape
    tol = TOL[x_dtype]
    atol = BF16_ATOL if x_dtype == torch.bfloat16 else tol
    torch.testing.assert_close(y.cpu(), yr.detach(), rtol=tol, atol=atol)
    y.backward(dy.to(cuda).to(y.dtype))
    torch.testing.assert_close(xg.grad.cpu(), xr.grad, rtol=tol, atol=atol)


def test_rmsnorm_strided_rows(cuda):
    """A row stride larger than the row (a column slice of a wider buffer)."""
    from hackathon_b200.rmsnorm import rmsnorm
    torch.manual_seed(1)
    buf = torch.randn(64, 2048, device=cuda, dtype=torch.bfloat16)
    x = buf[:, :1536]
    w = torch.randn(1536, device=cuda, dtype=torch.bfloat16)
    y = rmsnorm(x, w, 1e-6)
    yr = ops_ref.rmsnorm_ref(x.cpu(), w.cpu(), 1e-6)
    torch.testing.assert_close(y.cpu(), yr, rtol=1.6e-2, atol=BF16_ATOL)


@pytest.mark.parametrize("rows,hidden", [(3, 3584), (2375, 3584), (1000, 8192), (300, 5120),
                                         (64, 8), (777, 4096)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_rmsnorm_row_shapes(cuda, rows, hidden, dtype):
    """Row counts and lengths around the kernels' dispatch limits: a few rows, rows that do not
    fill the last CTA, rows of 4096 (the warp-per-row forward's longest) and beyond, a row of one
    16-byte chunk; forward and backward against the oracle."""
    from hackathon_b200.rmsnorm import rmsnorm
    torch.manual_seed(rows + hidden)
    weight = (1 + 0.1 * torch.randn(hidden)).to(dtype)
    x = torch.randn(rows, hidden, dtype=dtype)
    dy = torch.randn(rows, hidden).to(dtype)
    xr = x.clone().requires_grad_()
    yr = ops_ref.rmsnorm_ref(xr, weight, 1e-6)
    yr.backward(dy)
    xg = x.to(cuda).requires_grad_()
    y = rmsnorm(xg, weight.to(cuda), 1e-6)
    y.backward(dy.to(cuda))
    tol = TOL[dtype]
    atol = BF16_ATOL if dtype == torch.bfloat16 else tol
    torch.testing.assert_close(y.cpu(), yr.detach(), rtol=tol, atol=atol)
    torch.testing.assert_close(xg.grad.cpu(), xr.grad, rtol=tol, atol=atol)


# ----------------------------------------------------------------------------------- RoPE

@pytest.mark.parametrize("i", range(8))
def test_rope_vs_reference_fixtures(cuda, i):
    from hackathon_b200.rope import TritonRoPE
    g = golden("rope")
    half, equal, _ = (int(v) for v in g[f"rope_{i}_meta"])
    t = {k: _t(g[f"rope_{i}_{k}"], cuda) for k in
         ("q", "k", "cos", "sin", "qo", "ko", "gq", "gk", "dq", "dk")}
    # rebuild the (B,S,H,D) buffers seen as (B,H,S,D), as the attention does
    q = t["q"].transpose(1, 2).contiguous().transpose(1, 2).requires_grad_()
    k = t["k"].transpose(1, 2).contiguous().transpose(1, 2).requires_grad_()
    qo, ko = TritonRoPE.apply(q, k, t["cos"], t["sin"])
    tol = (2e-3 if half else 1e-5) * (1 if equal else 4)
    torch.testing.assert_close(qo, t["qo"], rtol=tol, atol=tol)
    torch.testing.assert_close(ko, t["ko"], rtol=tol, atol=tol)
    assert qo.stride() == q.stride()
    torch.autograd.backward((qo, ko), (t["gq"], t["gk"]))
    torch.testing.assert_close(q.grad, t["dq"], rtol=tol, atol=tol)
    torch.testing.assert_close(k.grad, t["dk"], rtol=tol, atol=tol)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("shape", [(4, 512, 12, 2, 128), (2, 256, 14, 2, 64),
                                   (1, 4096, 28, 4, 128), (2, 33, 3, 1, 10)])
def test_rope_vs_oracle(cuda, dtype, shape):
    from hackathon_b200.rope import TritonRoPE
    B, S, HQ, HK, D = shape
    torch.manual_seed(0)
    q = torch.randn(B, S, HQ, D, dtype=dtype).transpose(1, 2)
    k = torch.randn(B, S, HK, D, dtype=dtype).transpose(1, 2)
    cos, sin = ops_ref.qwen_cos_sin(1, S, D, dtype=dtype)
    qr, kr = q.clone().requires_grad_(), k.clone().requires_grad_()
    oq_r, ok_r = ops_ref.rope_ref(qr, kr, cos, sin)
    gq, gk = torch.randn_like(oq_r), torch.randn_like(ok_r)
    torch.autograd.backward((oq_r, ok_r), (gq, gk))
    qg = q.to(cuda).requires_grad_()
    kg = k.to(cuda).requires_grad_()
    oq, ok = TritonRoPE.apply(qg, kg, cos.to(cuda), sin.to(cuda))
    torch.autograd.backward((oq, ok), (gq.to(cuda), gk.to(cuda)))
    tol = TOL[dtype]
    atol = BF16_ATOL if dtype == torch.bfloat16 else tol
    for a, b in ((oq, oq_r), (ok, ok_r), (qg.grad, qr.grad), (kg.grad, kr.grad)):
        torch.testing.assert_close(a.cpu(), b.detach(), rtol=tol, atol=atol)


@pytest.mark.parametrize("heads", [4, 1, 28])
@pytest.mark.parametrize("backward", [False, True])
def test_rope_rows_few_heads(cuda, heads, backward):
    """rope_rows (the step's RoPE on projection outputs laid out as token rows) with few heads
    per position - several positions per CTA, the last CTA's positions running past the row
    count - against the rotation and its transpose computed in fp32 on the host."""
    from hackathon_b200.rope import rope_rows
    B, S, D = 3, 37, 128
    torch.manual_seed(heads)
    x2 = torch.randn(B * S, heads * D, device=cuda).to(torch.bfloat16)
    cos, sin = ops_ref.qwen_cos_sin(1, S, D, dtype=torch.bfloat16)
    cos, sin = cos[0].to(cuda), sin[0].to(cuda)
    out = rope_rows(x2, cos, sin, backward=backward)
    q = x2.view(B, S, heads, D).transpose(1, 2).float().cpu()
    c, s_ = cos.float().cpu()[None, None], sin.float().cpu()[None, None]
    x1, xh = q[..., :D // 2], q[..., D // 2:]
    c1, c2, s1, s2 = c[..., :D // 2], c[..., D // 2:], s_[..., :D // 2], s_[..., D // 2:]
    if backward:
        ref = torch.cat([x1 * c1 + xh * s2, xh * c2 - x1 * s1], -1)
    else:
        ref = torch.cat([x1 * c1 - xh * s1, xh * c2 + x1 * s2], -1)
    ref = ref.transpose(1, 2).reshape(B * S, heads * D)
    torch.testing.assert_close(out.float().cpu(), ref, rtol=1.6e-2, atol=BF16_ATOL)


# ----------------------------------------------------------------------------------- SwiGLU

@pytest.mark.parametrize("i", range(2))
def test_swiglu_vs_reference_fixtures(cuda, i):
    from hackathon_b200.swiglu import swiglu
    g = golden("swiglu")
    gate = _t(g[f"swiglu_{i}_gate"], cuda).requires_grad_()
    up = _t(g[f"swiglu_{i}_up"], cuda).requires_grad_()
    y = swiglu(gate, up)
    tol = TOL[gate.dtype]
    torch.testing.assert_close(y, _t(g[f"swiglu_{i}_y"], cuda), rtol=tol, atol=tol)
    y.backward(_t(g[f"swiglu_{i}_grad"], cuda))
    torch.testing.assert_close(gate.grad, _t(g[f"swiglu_{i}_dgate"], cuda), rtol=tol, atol=tol)
    torch.testing.assert_close(up.grad, _t(g[f"swiglu_{i}_dup"], cuda), rtol=tol, atol=tol)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("shape", [(4, 512, 8960), (3, 77, 1001), (1, 2048, 18944)])
def test_swiglu_vs_oracle(cuda, dtype, shape):
    from hackathon_b200.swiglu import swiglu
    torch.manual_seed(0)
    gate = torch.randn(shape, device=cuda, dtype=dtype, requires_grad=True)
    up = torch.randn(shape, device=cuda, dtype=dtype, requires_grad=True)
    grad = torch.randn(shape, device=cuda, dtype=dtype)
    gr = gate.detach().float().requires_grad_()
    ur = up.detach().float().requires_grad_()
    ref = ops_ref.swiglu_ref(gr, ur)
    ref.backward(grad.float())
    out = swiglu(gate, up)
    out.backward(grad)
    tol = TOL[dtype]
    atol = BF16_ATOL if dtype == torch.bfloat16 else tol
    torch.testing.assert_close(out.float(), ref, rtol=tol, atol=atol)
    torch.testing.assert_close(gate.grad.float(), gr.grad, rtol=tol, atol=atol)
    torch.testing.assert_close(up.grad.float(), ur.grad, rtol=tol, atol=atol)


# ----------------------------------------------------------------------------------- LoRA

def test_dropout_masks_equal_reference_bits(cuda):
    from hackathon_b200.lora import DropoutCast
    g = golden("lora")
    x = _t(g["drop_x"], cuda)
    for i in range(4):
        seed, p_micro = (int(v) for v in g[f"drop_{i}_meta"])
        p = p_micro / 1e6
        keep = np.unpackbits(g[f"drop_{i}_keep"])[: x.numel()].reshape(x.shape).astype(bool)
        xg = x.clone().requires_grad_()
        y = DropoutCast.apply(xg, p, seed, torch.float32)
        assert np.array_equal((y != 0).cpu().numpy(), keep), i
        if f"drop_{i}_y" in g:
            assert np.array_equal(y.detach().cpu().numpy().view(np.uint32),
                                  g[f"drop_{i}_y"].view(np.uint32))
        y.backward(torch.ones_like(y))
        dk = np.unpackbits(g[f"drop_{i}_dx_keep"])[: x.numel()].reshape(x.shape).astype(bool)
        assert np.array_equal((xg.grad != 0).cpu().numpy(), dk), i


@pytest.mark.parametrize("out_dtype", [torch.float16, torch.float32, torch.bfloat16])
def test_dropout_cast_no_dropout_is_a_cast(cuda, out_dtype):
    from hackathon_b200.lora import DropoutCast
    x = torch.randn(3, 7, 1536, device=cuda, requires_grad=True)
    y = DropoutCast.apply(x, 0.0, 0, out_dtype)
    assert y.dtype == out_dtype
    torch.testing.assert_close(y, x.detach().to(out_dtype), atol=0, rtol=0)
    g = torch.randn_like(y)
    y.backward(g)
    assert x.grad.dtype == x.dtype
    torch.testing.assert_close(x.grad, g.float(), atol=0, rtol=0)


def test_dropout_rate_scale_and_backward(cuda):
    from hackathon_b200.lora import DropoutCast
    p = 0.05
    x = torch.randn(2048, 1536, device=cuda, requires_grad=True)
    y = DropoutCast.apply(x, p, 1234, torch.float32)
    kept = y != 0
    rate = 1 - kept.float().mean().item()
    assert abs(rate - p) < 0.01, rate
    torch.testing.assert_close(y[kept], x.detach()[kept] / (1 - p))
    y.backward(torch.ones_like(y))
    torch.testing.assert_close(x.grad, kept.float() / (1 - p))
    y3 = DropoutCast.apply(x.detach(), p, 4321, torch.float32)
    assert not torch.equal(y3 != 0, kept)


def test_dropout_mask_at_step_shape_matches_oracle(cuda):
    """[16384, 3584] bf16 (the 7B step's q/k/v input): rows spread over the tensor, bit-exact."""
    from hackathon_b200.lora import DropoutCast
    rows, cols, p, seed = 16384, 3584, 0.05, 987654321
    x = torch.ones(rows, cols, device=cuda, dtype=torch.bfloat16)
    y = DropoutCast.apply(x, p, seed, torch.bfloat16)
    for r in (0, 1, 8191, rows - 1):
        want = nf4_ref.philox_uniform(seed, r * cols + np.arange(cols)) > np.float32(p)
        assert np.array_equal((y[r] != 0).cpu().numpy(), want), r


def test_dropout_flat_index_wraps_like_int32(cuda):
    """rows*cols > 2^31: the reference's int32 flat index wraps; so must ours."""
    from hackathon_b200 import _lib
    rows, cols, p, seed = 270_000, 8192, 0.5, 99
    src = torch.ones(1, cols, device=cuda, dtype=torch.bfloat16)
    out = torch.empty(rows, cols, device=cuda, dtype=torch.bfloat16)
    _lib.call("qb_dropout_scale", src.data_ptr(), _lib.BF16, 0, out.data_ptr(), _lib.BF16, cols,
              rows, cols, seed, p, 2.0, _lib.stream(cuda))
    for r in (262_143, 262_144, rows - 1):   # 262144 * 8192 = 2^31
        want = nf4_ref.philox_uniform(seed, r * cols + np.arange(cols)) > np.float32(p)
        assert np.array_equal((out[r] != 0).cpu().numpy(), want), r


@pytest.mark.parametrize("rows,cols", [(64, 1536), (300, 3584), (7, 40)])
def test_recorded_mask_is_the_reference_stream(cuda, rows, cols):
    """qb_dropout_mask records exactly the reference's Philox mask as bits and produces the same
    output as the regenerating kernel; qb_dropout_apply replays it (and accumulates)."""
    from hackathon_b200.lora import DropoutCast, dropout_apply, dropout_mask
    p, seed = 0.1, 424242
    scale = 1.0 / (1.0 - p)
    x = torch.randn(rows, cols, device=cuda).to(torch.bfloat16)
    y, bits = dropout_mask(x, p, seed, scale)
    want = nf4_ref.dropout_keep(seed, rows, cols, p)
    unpacked = ((bits.cpu().numpy().view(np.uint32)[:, :, None] >> np.arange(32)) & 1).reshape(
        rows, -1)[:, :cols].astype(bool)
    assert np.array_equal(unpacked, want)
    assert torch.equal(y, DropoutCast.apply(x, p, seed, torch.bfloat16))
    if cols % 8 == 0:
        assert torch.equal(dropout_apply(x, bits, scale), y)
        acc = torch.ones_like(x)
        dropout_apply(x, bits, scale, out=acc, accumulate=True)
        keep = torch.from_numpy(want).to(cuda)
        expect = (1.0 + torch.where(keep, x.float() * scale, torch.zeros_like(x.float())))
        assert torch.equal(acc, expect.to(torch.bfloat16))   # one rounding, as the kernel


@pytest.mark.parametrize("rows,cols,ctas", [(64, 1536, 0), (300, 3584, 2), (7, 40, 1),
                                             (5, 33, 8), (16384, 3584, 2)])
def test_bits_drawn_ahead_equal_recorded_mask(cuda, rows, cols, ctas):
    """qb_dropout_bits (no data, any grid cap) writes the very words qb_dropout_mask records,
    padding bits of a ragged last word included, and they are the reference's Philox mask."""
    from hackathon_b200.lora import dropout_bits, dropout_mask
    p, seed = 0.05, 20240607
    x = torch.ones(rows, cols, device=cuda, dtype=torch.bfloat16)
    _, want_bits = dropout_mask(x, p, seed, 1.0 / (1.0 - p))
    bits = dropout_bits(rows, cols, p, seed, cuda, ctas_per_sm=ctas)
    assert torch.equal(bits, want_bits)
    for r in sorted({0, rows // 2, rows - 1}):
        got = ((bits[r].cpu().numpy().view(np.uint32)[:, None] >> np.arange(32)) & 1).reshape(
            -1)[:cols].astype(bool)
        want = nf4_ref.philox_uniform(seed, r * cols + np.arange(cols)) > np.float32(p)
        assert np.array_equal(got, want), r


def test_gate_up_gemm_side_warps_draw_the_recorded_masks(cuda):
    """qb_gemm_gateup_swiglu_masks: the masks its side warps draw are the very words
    qb_dropout_bits writes (ragged last words, a seed with a high word, tiny and large jobs in
    one launch), and the GEMM's output equals the launch without side work bit for bit."""
    from hackathon_b200.gemm import gemm_gateup_swiglu
    from hackathon_b200.lora import dropout_bits
    torch.manual_seed(0)
    M, K0, I, r = 2000, 896, 1536, 16
    x = (torch.randn(M, K0, device=cuda) * 0.5).to(torch.bfloat16)
    wg = (torch.randn(I, K0, device=cuda) * 0.05).to(torch.bfloat16)
    wu = (torch.randn(I, K0, device=cuda) * 0.05).to(torch.bfloat16)
    lu = (torch.randn(M, 2 * r, device=cuda) * 0.5).to(torch.bfloat16)
    bg = (torch.randn(I, 2 * r, device=cuda) * 0.05).to(torch.bfloat16)
    bu = (torch.randn(I, 2 * r, device=cuda) * 0.05).to(torch.bfloat16)
    specs = [(M, K0, 0.1, 1234567890123), (M, 4864, 0.05, 7), (7, 40, 0.5, 3), (5, 33, 0.0, 11),
             (16384, 3584, 0.05, 20240607), (1, 1, 0.3, 5)]
    jobs = [(torch.full((rows, (cols + 31) // 32), -1, dtype=torch.int32, device=cuda), rows,
             cols, seed, p) for rows, cols, p, seed in specs]
    h0, g0, u0 = gemm_gateup_swiglu(x, wg, wu, lu, bg, bu, save_gu=True)
    h1, g1, u1 = gemm_gateup_swiglu(x, wg, wu, lu, bg, bu, save_gu=True, mask_jobs=jobs)
    assert torch.equal(h1, h0) and torch.equal(g1, g0) and torch.equal(u1, u0)
    for bits, rows, cols, seed, p in jobs:
        assert torch.equal(bits, dropout_bits(rows, cols, p, seed, cuda)), (rows, cols)
    r0 = jobs[0][0][M - 1].cpu().numpy().view(np.uint32)
    got = ((r0[:, None] >> np.arange(32)) & 1).reshape(-1)[:K0].astype(bool)
    want = nf4_ref.philox_uniform(specs[0][3], (M - 1) * K0 + np.arange(K0)) > np.float32(0.1)
    assert np.array_equal(got, want)
    # without the LoRA segment and without saving g / u
    h2 = gemm_gateup_swiglu(x, wg, wu, mask_jobs=jobs[2:4])
    assert torch.equal(h2, gemm_gateup_swiglu(x, wg, wu))
    with pytest.raises(ValueError):
        gemm_gateup_swiglu(x, wg, wu, mask_jobs=jobs + jobs[:3])


@pytest.mark.parametrize("rows,cols,n,in_dtype", [(16384, 3584, 3, torch.bfloat16),
                                                  (300, 1000, 2, torch.bfloat16),
                                                  (7, 40, 4, torch.float32),
                                                  (129, 264, 1, torch.bfloat16)])
def test_dropout_apply_multi_equals_single_applies(cuda, rows, cols, n, in_dtype):
    """qb_dropout_apply_multi (one input read once, 1..4 masks) writes, for every mask, the very
    bits dropout_apply writes for it alone: ragged last mask words, fp32 input into bf16."""
    from hackathon_b200.lora import dropout_apply, dropout_apply_multi, dropout_bits
    torch.manual_seed(3)
    x = torch.randn(rows, cols, device=cuda).to(in_dtype)
    masks = [(dropout_bits(rows, cols, p, 50 + j, cuda), 1.0 / (1.0 - p))
             for j, p in enumerate([0.1, 0.05, 0.3, 0.0][:n])]
    outs = dropout_apply_multi(x, masks, out_dtype=torch.bfloat16)
    for (bits, scale), got in zip(masks, outs):
        want = dropout_apply(x, bits, scale, out=torch.empty(rows, cols, dtype=torch.bfloat16,
                                                             device=cuda))
        assert torch.equal(got, want)
    with pytest.raises(ValueError):
        dropout_apply_multi(x, masks * 5)


def test_bits_drawn_on_a_side_stream_beside_a_gemm(cuda):
    """The prefetch pattern of the model: bits drawn on another stream while a tcgen05 GEMM
    runs, the consumer stream waiting on an event; the result equals the inline mask."""
    from hackathon_b200.gemm import gemm
    from hackathon_b200.lora import dropout_bits, dropout_mask
    rows, cols, p, seed = 16384, 3584, 0.05, 77
    a = torch.randn(16384, 3584, device=cuda).to(torch.bfloat16)
    b = torch.randn(3584, 3584, device=cuda).to(torch.bfloat16)
    main = torch.cuda.current_stream(cuda)
    side = torch.cuda.Stream(device=cuda)
    bits = torch.empty((rows, cols // 32), dtype=torch.int32, device=cuda)
    side.wait_stream(main)
    c = gemm(a, b.t())
    with torch.cuda.stream(side):
        dropout_bits(rows, cols, p, seed, cuda, ctas_per_sm=2, out=bits)
        ev = torch.cuda.Event()
        ev.record(side)
    c2 = gemm(a, b.t())
    main.wait_event(ev)
    _, want = dropout_mask(torch.ones(rows, cols, device=cuda, dtype=torch.bfloat16), p, seed,
                           1.0 / (1.0 - p))
    assert torch.equal(bits, want)
    assert torch.equal(c, c2)


@pytest.mark.parametrize("T,K,R", [(300, 256, 64), (16384, 3584, 64), (129, 18944, 64),
                                   (257, 40, 32), (64, 200, 128), (200, 136, 256),
                                   (1000, 3584, 96)])
def test_lora_xa_matches_dropout_then_product(cuda, T, K, R):
    """qb_lora_xa: the stored xd equals qb_dropout_apply's bit for bit, and U equals the fp32
    product of that xd with A rounded to bf16 (accumulation order aside); ragged row blocks,
    ragged k-blocks, ranks 32..256."""
    from hackathon_b200.lora import dropout_apply, dropout_bits, lora_xa
    g = torch.Generator(device=cuda).manual_seed(T + K + R)
    x = torch.randn(T, K, device=cuda, generator=g).to(torch.bfloat16)
    a = (torch.randn(R, K, device=cuda, generator=g) / K ** 0.5).to(torch.bfloat16)
    p, seed = 0.1, 31337
    scale = 1.0 / (1.0 - p)
    bits = dropout_bits(T, K, p, seed, cuda)
    xd = torch.empty_like(x)
    u = lora_xa(x, a, bits, scale, xd_out=xd)
    want_xd = dropout_apply(x, bits, scale)
    assert torch.equal(xd, want_xd)
    ref = want_xd.float() @ a.float().t()
    torch.testing.assert_close(u.float(), ref, rtol=1.6e-2, atol=1e-2)
    assert torch.equal(lora_xa(x, a, bits, scale), u)        # without the xd store: same U


def test_lora_xa_without_mask_and_into_a_column_slice(cuda):
    """bits None: U = x A^T; U written into half of a [T, 2R] buffer (the gate / up pair's
    layout), the other half untouched."""
    from hackathon_b200.lora import lora_xa
    T, K, R = 777, 512, 64
    x = torch.randn(T, K, device=cuda).to(torch.bfloat16)
    a = (torch.randn(R, K, device=cuda) / K ** 0.5).to(torch.bfloat16)
    buf = torch.full((T, 2 * R), 7.0, device=cuda, dtype=torch.bfloat16)
    lora_xa(x, a, out=buf[:, R:])
    torch.testing.assert_close(buf[:, R:].float(), x.float() @ a.float().t(), rtol=1.6e-2,
                               atol=1e-2)
    assert torch.all(buf[:, :R] == 7.0)


@pytest.mark.parametrize("out_features", [1536, 256])
def test_scaled_add_matches_peft(cuda, out_features):
    from hackathon_b200.lora import ScaledAdd
    torch.manual_seed(0)
    base = torch.randn(2, 5, out_features, device=cuda, requires_grad=True)
    lo = torch.randn(2, 5, out_features, device=cuda, dtype=torch.float16, requires_grad=True)
    base_ref = base.detach().clone().requires_grad_()
    lo_ref = lo.detach().clone().requires_grad_()
    out_ref = ops_ref.scaled_add_ref(base_ref, lo_ref, 2.0)
    out = ScaledAdd.apply(base, lo, 2.0)
    assert out.dtype == out_ref.dtype
    torch.testing.assert_close(out, out_ref, atol=1e-6, rtol=1e-6)
    g = torch.randn_like(out_ref)
    out_ref.backward(g)
    out.backward(g)
    torch.testing.assert_close(base.grad, base_ref.grad)
    assert lo.grad.dtype == lo_ref.grad.dtype
    torch.testing.assert_close(lo.grad, lo_ref.grad, atol=2e-3, rtol=2e-3)


def test_scaled_add_vs_reference_fixture(cuda):
    from hackathon_b200.lora import ScaledAdd
    g = golden("lora")
    base = _t(g["sadd_base"], cuda).requires_grad_()
    lo = _t(g["sadd_lo"], cuda, torch.float16).requires_grad_()
    y = ScaledAdd.apply(base, lo, 2.0)
    torch.testing.assert_close(y, _t(g["sadd_y"], cuda), rtol=1e-6, atol=1e-6)
    y.backward(_t(g["sadd_g"], cuda))
    torch.testing.assert_close(base.grad, _t(g["sadd_dbase"], cuda))
    torch.testing.assert_close(lo.grad.float(), _t(g["sadd_dlo"], cuda), rtol=2e-3, atol=2e-3)

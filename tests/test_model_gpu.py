"""The QLoRA step on the GPU: a tiny Qwen2.5-shaped model runs forward + backward + AdamW, the
dropout masks replay under activation checkpointing, and one decoder layer matches the eager CPU
oracle (NF4 rebuilt by the oracle, LoRA, RoPE, SwiGLU, attention) in forward and backward."""

import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_tiny_step_runs_and_loss_is_sane(cuda):
    from hackathon_b200.qlora import QwenQLoRA, make_optimizer, preset, synthetic_batch, train_step
    shape = preset("0.5b", layers=2)
    model = QwenQLoRA(shape, cuda, seed=0)
    opt = make_optimizer(model)
    ids, labels = synthetic_batch(shape, 2, 128, cuda, seed=1)
    losses = [float(train_step(model, opt, ids, labels)) for _ in range(3)]
    assert all(np.isfinite(losses))
    assert abs(losses[0] - math.log(shape.vocab)) < 1.0


@pytest.mark.parametrize("p", [0.0, 0.1])
@pytest.mark.parametrize("shape", [(3584, 512, 300), (896, 4864, 128)])
def test_fused_projection_matches_reference_composition(cuda, p, shape):
    """LoRANF4Proj (fused NF4 GEMM, LoRA as extra K) against the reference's composition of the
    same op: NF4Linear + DropoutCast + lora_B(lora_A(.)) + ScaledAdd, forward and all grads."""
    from hackathon_b200.qlora import LoRANF4Linear, preset
    in_f, out_f, T = shape
    s = preset("0.5b", lora_r=64, lora_alpha=128, lora_dropout=p)
    gen = torch.Generator(device=cuda).manual_seed(5)
    mod = LoRANF4Linear(in_f, out_f, True, s, cuda, gen)
    with torch.no_grad():
        mod.lora_B.normal_(0, 0.05, generator=gen)
    x = torch.randn(T, in_f, device=cuda, generator=gen).to(torch.bfloat16)
    gy = torch.randn(T, out_f, device=cuda, generator=gen).to(torch.bfloat16)
    outs = []
    for fused in (True, False):
        mod.fused = fused
        mod.lora_A.grad = mod.lora_B.grad = None
        xi = x.clone().requires_grad_()
        y = mod(xi, seed=1234)
        y.backward(gy)
        outs.append((y.detach().float(), xi.grad.float(), mod.lora_A.grad.clone(),
                     mod.lora_B.grad.clone()))
    (y1, dx1, da1, db1), (y0, dx0, da0, db0) = outs
    torch.testing.assert_close(y1, y0, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(dx1, dx0, rtol=2e-2, atol=2e-2)
    for a, b in ((da1, da0), (db1, db0)):
        rel = (a - b).norm() / b.norm()
        assert rel < 2e-2, float(rel)


@pytest.mark.parametrize("p", [0.0, 0.1])
def test_long_token_projection_with_residual_matches_composition(cuda, p):
    """At the long-token path (transient bf16 weight kept from forward to backward, residual in
    the GEMM epilogue, masked-accumulate GEMM for the dropped-out LoRA input gradient): forward
    and all grads, residual grad included, against the reference's composition + a residual add."""
    from hackathon_b200.nf4 import DEQUANT_GEMM_MIN_TOKENS
    from hackathon_b200.qlora import LoRANF4Linear, preset
    in_f, out_f, T = 896, 640, DEQUANT_GEMM_MIN_TOKENS
    s = preset("0.5b", lora_r=64, lora_alpha=128, lora_dropout=p)
    gen = torch.Generator(device=cuda).manual_seed(6)
    mod = LoRANF4Linear(in_f, out_f, False, s, cuda, gen)
    with torch.no_grad():
        mod.lora_B.normal_(0, 0.05, generator=gen)
    x = torch.randn(T, in_f, device=cuda, generator=gen).to(torch.bfloat16)
    h = torch.randn(T, out_f, device=cuda, generator=gen).to(torch.bfloat16)
    gy = torch.randn(T, out_f, device=cuda, generator=gen).to(torch.bfloat16)
    outs = []
    for fused in (True, False):
        mod.fused = fused
        mod.lora_A.grad = mod.lora_B.grad = None
        xi, hi = x.clone().requires_grad_(), h.clone().requires_grad_()
        y = mod(xi, seed=99, residual=hi)
        y.backward(gy)
        outs.append((y.detach().float(), xi.grad.float(), hi.grad.float(),
                     mod.lora_A.grad.clone(), mod.lora_B.grad.clone()))
    (y1, dx1, dh1, da1, db1), (y0, dx0, dh0, da0, db0) = outs
    torch.testing.assert_close(y1, y0, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(dx1, dx0, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(dh1, dh0, rtol=0, atol=0)
    for a, b in ((da1, da0), (db1, db0)):
        rel = (a - b).norm() / b.norm()
        assert rel < 2e-2, float(rel)


def test_checkpoint_replays_dropout_masks(cuda):
    """With dropout on, the gradients with and without activation checkpointing agree (the
    recompute must draw the same Philox masks)."""
    from hackathon_b200.qlora import QwenQLoRA, preset, synthetic_batch
    shape = preset("0.5b", layers=2, lora_dropout=0.1)
    ids, labels = synthetic_batch(shape, 1, 64, cuda, seed=2)
    grads = []
    for ckpt in (True, False):
        model = QwenQLoRA(shape, cuda, seed=0, checkpoint=ckpt)
        model.train()
        loss, _ = model(ids, labels)
        loss.backward()
        grads.append(torch.cat([p.grad.flatten() for p in model.adapter_parameters()]))
    torch.testing.assert_close(grads[0], grads[1], rtol=1e-3, atol=1e-5)


def test_masks_drawn_ahead_give_the_same_step(cuda):
    """Dropout masks drawn ahead on the side stream (layer i+1's beside layer i's GEMMs) give
    the same loss and adapter gradients as masks drawn inline, bit for bit."""
    from hackathon_b200.qlora import QwenQLoRA, preset, synthetic_batch
    shape = preset("0.5b", layers=3, lora_dropout=0.1)
    ids, labels = synthetic_batch(shape, 1, 256, cuda, seed=5)
    out = []
    for ahead in (True, False):
        model = QwenQLoRA(shape, cuda, seed=0)
        model.mask_prefetch = ahead
        model.train()
        loss, _ = model(ids, labels)
        loss.backward()
        out.append((loss.detach(), torch.cat([p.grad.flatten()
                                              for p in model.adapter_parameters()])))
    assert torch.equal(out[0][0], out[1][0])
    assert torch.equal(out[0][1], out[1][1])


def test_masks_drawn_in_the_gate_up_gemm_give_the_same_step(cuda):
    """Dropout masks drawn by the gate/up GEMM's side warps (each layer's down mask and the next
    layer's six) are the words drawn at their use, bit for bit, and the forward is unchanged
    bit for bit; only layer 0's six projections draw their own. (The gradients are compared
    within a tolerance: the attention backward accumulates dQ in a run-dependent order.)"""
    from hackathon_b200 import _lib
    from hackathon_b200.qlora import MASKS, QwenQLoRA, preset, synthetic_batch
    shape = preset("0.5b", layers=3, lora_dropout=0.1)
    ids, labels = synthetic_batch(shape, 1, 2048, cuda, seed=5)
    model = QwenQLoRA(shape, cuda, seed=0)
    model.train()
    out = []
    for in_gemm in (True, False):
        model.gemm_masks = in_gemm
        model.zero_grad(set_to_none=True)
        with _lib.KernelTimer() as timer:
            loss, _ = model(ids, labels)
        calls = timer.summary()
        masks = {k: v.clone() for k, v in MASKS.items()}
        loss.backward()
        out.append((loss.detach(), torch.cat([p.grad.flatten()
                                              for p in model.adapter_parameters()]), calls,
                    masks))
    assert torch.equal(out[0][0], out[1][0])
    assert out[0][3].keys() == out[1][3].keys() and len(out[0][3]) == 7 * shape.layers
    for key, bits in out[0][3].items():
        assert torch.equal(bits, out[1][3][key]), key
    rel = (out[0][1] - out[1][1]).norm() / out[1][1].norm()
    assert rel < 1e-2, float(rel)
    with_jobs, without = out[0][2], out[1][2]
    assert with_jobs["qb_gemm_gateup_swiglu_masks"]["launches"] == shape.layers
    assert with_jobs["qb_dropout_mask"]["launches"] == 6
    assert without["qb_dropout_mask"]["launches"] == 7 * shape.layers
    # from layer 1 on the masks are recorded before use: q / k / v take one pass over their
    # common input, gate / up one over theirs; o and down apply their own (layer 0's down too)
    assert with_jobs["qb_dropout_apply_multi"]["launches"] == 2 * (shape.layers - 1)
    assert with_jobs["qb_dropout_apply"]["launches"] == 2 * (shape.layers - 1) + 1
    assert "qb_dropout_apply_multi" not in without


@pytest.mark.parametrize("S", [256, 2048])
def test_recompute_reuses_first_pass_lora_products(cuda, S):
    """The checkpoint recompute takes U = xd Aᵀ of every projection from the first pass instead
    of running the rank-r GEMM again: the same loss and adapter gradients (bit for bit where the
    attention backward is deterministic, S = 256; within a tolerance at S = 2048, where it
    accumulates dQ in a run-dependent order), and one rank-r GEMM call fewer in the backward
    for every product kept (two for the gate / up pair's)."""
    from hackathon_b200 import _lib
    from hackathon_b200 import qlora
    from hackathon_b200.qlora import QwenQLoRA, preset, synthetic_batch
    shape = preset("0.5b", layers=3, lora_dropout=0.1)
    ids, labels = synthetic_batch(shape, 1, S, cuda, seed=7)
    model = QwenQLoRA(shape, cuda, seed=0)
    model.train()
    out = []
    try:
        for keep in (True, False):
            qlora.KEEP_UPRODS = keep
            model.zero_grad(set_to_none=True)
            loss, _ = model(ids, labels)
            kept = len(qlora.UPRODS)
            with _lib.KernelTimer() as timer:
                loss.backward()
            calls = timer.summary()
            out.append((loss.detach(), torch.cat([p.grad.flatten()
                                                  for p in model.adapter_parameters()]),
                        calls["qb_gemm_bf16"]["launches"], kept, len(qlora.UPRODS)))
    finally:
        qlora.KEEP_UPRODS = True
    (l1, g1, n1, k1, left1), (l0, g0, n0, k0, _) = out
    assert torch.equal(l1, l0)
    pairs = 0 if S == 256 else shape.layers     # the gate / up pair from 2048 tokens on
    if S == 256:
        assert torch.equal(g1, g0)
    else:
        rel = (g1 - g0).norm() / g0.norm()
        assert rel < 1e-2, float(rel)
    # every kept product saves one GEMM call in the recompute, a kept pair two; at least the q,
    # o and down projections (and gate / up) of every layer take the fused path here
    assert k1 >= 3 * shape.layers + pairs
    assert n0 - n1 == k1 + pairs
    assert k0 == 0 and left1 == 0


@pytest.mark.parametrize("name,S", [("0.5b", 64), ("1.5b", 2048)])
def test_decoder_layer_matches_eager_oracle(cuda, name, S):
    """One decoder layer (dropout off): GPU ops vs the eager CPU oracle with the same NF4
    bytes, bf16 activations; forward and the LoRA-A gradient within bf16 tolerance. 0.5B shapes
    at 64 tokens (the fused NF4 kernel, RoPE as its own kernel for 64-dim heads); 1.5B shapes
    (the 1.5B configuration: 12 / 2 heads of 128) at 2048 tokens (transient weights, RoPE in the q / k
    GEMM epilogue)."""
    from hackathon_b200.qlora import DecoderLayer, preset
    from oracle import ops_ref
    shape = preset(name, layers=1, lora_dropout=0.0)
    gen = torch.Generator(device=cuda).manual_seed(0)
    layer = DecoderLayer(shape, cuda, gen)
    B = 1
    torch.manual_seed(0)
    h = (torch.randn(B, S, shape.hidden) * 0.5).to(torch.bfloat16)
    cos, sin = ops_ref.qwen_cos_sin(1, S, shape.head_dim, shape.theta, torch.bfloat16)
    hg = h.to(cuda).requires_grad_()
    out = layer(hg, cos.to(cuda), sin.to(cuda), 0)
    gout = torch.randn_like(out)
    out.backward(gout)

    # eager CPU twin with the same dequantised weights and adapters
    def twin(m):
        qs = m.quant_state
        return ops_ref.NF4LoRALinearRef(
            m.packed.cpu().numpy().reshape(-1), qs.absmax.cpu().numpy(),
            qs.state2.code.cpu().numpy(), qs.state2.absmax.cpu().numpy(), qs.offset,
            (m.out_features, m.in_features), None if m.bias is None else m.bias.cpu(),
            m.lora_A.detach().cpu(), m.lora_B.detach().cpu(), m.scaling)

    t = {n: twin(getattr(layer, n)) for n in ("q", "k", "v", "o", "gate", "up", "down")}
    hr = h.clone().requires_grad_()
    x = ops_ref.rmsnorm_ref(hr, layer.ln1.cpu(), shape.eps)
    q = t["q"](x).view(B, S, shape.heads, shape.head_dim).transpose(1, 2)
    k = t["k"](x).view(B, S, shape.kv_heads, shape.head_dim).transpose(1, 2)
    v = t["v"](x).view(B, S, shape.kv_heads, shape.head_dim).transpose(1, 2)
    q, k = ops_ref.rope_ref(q, k, cos, sin)
    rep = shape.heads // shape.kv_heads
    a = torch.nn.functional.scaled_dot_product_attention(
        q.float(), k.float().repeat_interleave(rep, 1), v.float().repeat_interleave(rep, 1),
        is_causal=True).to(torch.bfloat16)
    hh = hr + t["o"](a.transpose(1, 2).reshape(B, S, -1))
    x2 = ops_ref.rmsnorm_ref(hh, layer.ln2.cpu(), shape.eps)
    m = ops_ref.swiglu_ref(t["gate"](x2), t["up"](x2)).to(torch.bfloat16)
    ref = hh + t["down"](m)
    ref.backward(gout.cpu())
    torch.testing.assert_close(out.detach().float().cpu(), ref.detach().float(), rtol=5e-2,
                               atol=5e-2)
    # the input gradient runs through every projection's backward, attention and two norms, each
    # side rounding to bf16 in its own order: elementwise at the same tolerance except for a
    # 1e-4 fraction of outliers, and within 2 % in norm
    got, want = hg.grad.float().cpu(), hr.grad.float()
    outside = ((got - want).abs() > 5e-2 + 5e-2 * want.abs()).float().mean()
    assert float(outside) < 1e-4, float(outside)
    assert float((got - want).norm() / want.norm()) < 2e-2
    ga = layer.down.lora_B.grad.cpu()
    gr = t["down"].lora_b.grad
    rel = (ga - gr).norm() / gr.norm()
    assert rel < 5e-2, float(rel)


@pytest.mark.parametrize("p", [0.0, 0.1])
def test_fused_gate_up_swiglu_matches_separate_projections(cuda, p):
    """The MLP's gate/up pair as one GEMM with the SwiGLU in its epilogue (long-token path)
    against the separate LoRANF4Proj projections + the SwiGLU kernel: forward bit for bit (same
    bf16 g and u, same SwiGLU arithmetic), all gradients within bf16 tolerance, with and without
    activation checkpointing of the layer."""
    from hackathon_b200.nf4 import DEQUANT_GEMM_MIN_TOKENS
    from hackathon_b200.qlora import DecoderLayer, preset
    shape = preset("0.5b", layers=1, lora_dropout=p, lora_r=16, lora_alpha=32)
    gen = torch.Generator(device=cuda).manual_seed(3)
    layer = DecoderLayer(shape, cuda, gen)
    layer.train()
    with torch.no_grad():
        for mod in (layer.gate, layer.up):
            mod.lora_B.normal_(0, 0.05, generator=gen)
    T = DEQUANT_GEMM_MIN_TOKENS
    x = torch.randn(1, T, shape.hidden, device=cuda, generator=gen).to(torch.bfloat16)
    gy = torch.randn(1, T, shape.intermediate, device=cuda, generator=gen).to(torch.bfloat16)
    from hackathon_b200.qlora import GateUpSwiGLU, MASKS
    from hackathon_b200.swiglu import swiglu
    assert layer.mlp_fused_ok(x)
    outs = []
    for fused in (True, False):
        MASKS.clear()
        for mod in (layer.gate, layer.up):
            mod.lora_A.grad = mod.lora_B.grad = None
        xi = x.clone().requires_grad_()
        if fused:
            m = GateUpSwiGLU.apply(xi, layer.gate.lora_A, layer.gate.lora_B, layer.up.lora_A,
                                   layer.up.lora_B, layer.gate, layer.up, p, 40, 41, True)
        else:
            m = swiglu(layer.gate(xi, 40), layer.up(xi, 41))
        m.backward(gy)
        outs.append([m.detach(), xi.grad] + [t.grad.clone() for mod in (layer.gate, layer.up)
                                            for t in (mod.lora_A, mod.lora_B)])
    (m1, dx1, *g1), (m0, dx0, *g0) = outs
    assert torch.equal(m1.view(torch.int16), m0.view(torch.int16))
    torch.testing.assert_close(dx1.float(), dx0.float(), rtol=2e-2, atol=2e-2)
    for a, b in zip(g1, g0):
        rel = (a - b).norm() / b.norm()
        assert rel < 2e-2, float(rel)


def test_checkpointed_layer_with_fused_mlp_matches_uncheckpointed(cuda):
    """A decoder layer at the long-token path (fused gate/up SwiGLU, placeholders saved in the
    checkpoint's first pass) gives the same adapter gradients with and without checkpointing.
    At this length the attention backward (cuDNN) accumulates dQ with atomics, so the two runs
    agree to rounding, not bit for bit: compared by relative norm."""
    from hackathon_b200.nf4 import DEQUANT_GEMM_MIN_TOKENS
    from hackathon_b200.qlora import QwenQLoRA, preset, synthetic_batch
    shape = preset("0.5b", layers=2, lora_dropout=0.1)
    ids, labels = synthetic_batch(shape, 1, DEQUANT_GEMM_MIN_TOKENS, cuda, seed=4)
    grads = []
    for ckpt in (True, False):
        model = QwenQLoRA(shape, cuda, seed=0, checkpoint=ckpt)
        model.train()
        loss, _ = model(ids, labels)
        loss.backward()
        grads.append(torch.cat([p.grad.flatten() for p in model.adapter_parameters()]))
    rel = (grads[0] - grads[1]).norm() / grads[1].norm()
    assert rel < 1e-3, float(rel)


@pytest.mark.parametrize("T", [256, 8192])
def test_projection_with_rope_epilogue_matches_rope_kernel(cuda, T):
    """q projection with the RoPE in its GEMM epilogue (long-token path) or right after the
    fused kernel (short) against the projection followed by the RoPE kernel: forward bit for bit
    (same rounding points, same rotation arithmetic), input and adapter gradients within bf16
    tolerance (the backward applies the RoPE transpose before the projection's)."""
    from hackathon_b200.qlora import MASKS, LoRANF4Linear, preset
    from hackathon_b200.rope import CudaRoPE
    from oracle import ops_ref
    s = preset("0.5b", lora_r=16, lora_alpha=32, lora_dropout=0.1, heads=8, head_dim=128)
    gen = torch.Generator(device=cuda).manual_seed(12)
    in_f, heads = 896, 8
    mod = LoRANF4Linear(in_f, heads * 128, True, s, cuda, gen)
    with torch.no_grad():
        mod.lora_B.normal_(0, 0.05, generator=gen)
    S = 128 if T == 256 else 1024
    cos, sin = ops_ref.qwen_cos_sin(1, S, 128, 1e6, torch.bfloat16)
    cos, sin = cos.to(cuda), sin.to(cuda)
    x = torch.randn(T // S, S, in_f, device=cuda, generator=gen).to(torch.bfloat16)
    gy = torch.randn(T // S, heads, S, 128, device=cuda, generator=gen).to(torch.bfloat16)
    outs = []
    for fused_rope in (True, False):
        MASKS.clear()
        mod.lora_A.grad = mod.lora_B.grad = None
        xi = x.clone().requires_grad_()
        if fused_rope:
            q = mod(xi, 5, rope=(cos[0], sin[0])).view(T // S, S, heads, 128).transpose(1, 2)
        else:
            q = mod(xi, 5).view(T // S, S, heads, 128).transpose(1, 2)
            q, _ = CudaRoPE.apply(q, q[:, :0], cos, sin)
        q.backward(gy)
        outs.append((q.detach().contiguous(), xi.grad.float(), mod.lora_A.grad.clone(),
                     mod.lora_B.grad.clone()))
    (q1, dx1, da1, db1), (q0, dx0, da0, db0) = outs
    assert torch.equal(q1.view(torch.int16), q0.view(torch.int16))
    torch.testing.assert_close(dx1, dx0, rtol=2e-2, atol=2e-2)
    for a, b in ((da1, da0), (db1, db0)):
        rel = (a - b).norm() / b.norm()
        assert rel < 2e-2, float(rel)


def _mask_of_bits(bits, cols):
    """bool [rows, cols] from the step's mask words (bit j of word w = element 32 w + j)."""
    sh = torch.arange(32, device=bits.device, dtype=torch.int32)
    return ((bits.unsqueeze(-1) >> sh) & 1).bool().reshape(bits.shape[0], -1)[:, :cols]


def test_long_token_checkpointed_layer_with_dropout_matches_eager_oracle(cuda):
    """The decoder layer on the path the 7B step runs - T >= DEQUANT_GEMM_MIN_TOKENS (transient
    bf16 weights), dropout p = 0.1, activation checkpointing, the q/k projections with the RoPE
    in their GEMM epilogue, the gate/up pair as one GEMM with the SwiGLU in its epilogue, the
    masked LoRA input gradient - against the eager oracle: the reference's composition
    (NF4 rebuilt by the numpy oracle, F.linear, peft's dropout -> lora_A -> lora_B -> scaled add,
    eager RMSNorm / RoPE / SwiGLU, fp32 attention), run with torch ops on the device. Both apply
    the masks the step drew; those masks are first checked, on sampled rows of every
    projection, against the oracle's Philox-4x32-10 stream (the reference's tl.rand). Forward,
    input gradient and all fourteen adapter gradients within bf16 tolerance."""
    from hackathon_b200 import qlora
    from hackathon_b200.gemm import device_error
    from hackathon_b200.nf4 import DEQUANT_GEMM_MIN_TOKENS
    from oracle import nf4_ref, ops_ref
    p = 0.1
    shape = qlora.preset("0.5b", hidden=512, intermediate=1408, heads=4, kv_heads=2,
                         head_dim=128, layers=1, lora_r=64, lora_alpha=128, lora_dropout=p)
    gen = torch.Generator(device=cuda).manual_seed(21)
    layer = qlora.DecoderLayer(shape, cuda, gen)
    layer.train()
    with torch.no_grad():
        for name in qlora._PROJ:
            getattr(layer, name).lora_B.normal_(0, 0.05, generator=gen)
    B, S, H = 2, 4096, shape.hidden
    assert B * S >= DEQUANT_GEMM_MIN_TOKENS
    h = (torch.randn(B, S, H, device=cuda, generator=gen) * 0.5).to(torch.bfloat16)
    cos, sin = ops_ref.qwen_cos_sin(1, S, 128, shape.theta, torch.bfloat16, device=cuda)
    cos, sin = cos.contiguous(), sin.contiguous()
    assert layer.rope_fused_ok(h, cos) and layer.mlp_fused_ok(h)
    seed = 777
    qlora.MASKS.clear()
    hg = h.clone().requires_grad_()
    out = torch.utils.checkpoint.checkpoint(layer, hg, cos, sin, seed, [0], None,
                                            use_reentrant=False, determinism_check="none")
    bits = {name: qlora.MASKS[(id(getattr(layer, name)), seed + k)].clone()
            for k, name in enumerate(qlora._PROJ)}
    gout = torch.randn(out.shape, device=cuda, generator=gen).to(torch.bfloat16)
    out.backward(gout)
    device_error()

    # the masks are the reference's Philox stream (sampled rows of every projection)
    rows = [0, 1, 4097, B * S - 1]
    for k, name in enumerate(qlora._PROJ):
        mod = getattr(layer, name)
        got = _mask_of_bits(bits[name][rows], mod.in_features).cpu().numpy()
        for i, r in enumerate(rows):
            want = nf4_ref.dropout_keep(seed + k, B * S, mod.in_features, p, row_range=(r, r + 1))
            assert np.array_equal(got[i], want[0]), (name, r)

    # eager twin: same NF4 bytes, same adapters, the same masks
    scale = 1.0 / (1.0 - p)

    class Twin(torch.nn.Module):
        def __init__(self, m, mask):
            super().__init__()
            qs = m.quant_state
            n = m.out_features * m.in_features
            wb = nf4_ref.dequant_nf4(m.packed.cpu().numpy().reshape(-1), n,
                                     qs.absmax.cpu().numpy(), True, qs.state2.code.cpu().numpy(),
                                     qs.state2.absmax.cpu().numpy(), qs.offset, 64, 256,
                                     out="bf16")
            self.w = torch.from_numpy(wb.view(np.int16).copy()).view(torch.bfloat16).view(
                m.out_features, m.in_features).to(cuda)
            self.b = m.bias
            self.a = torch.nn.Parameter(m.lora_A.detach().clone())
            self.bb = torch.nn.Parameter(m.lora_B.detach().clone())
            self.s = m.scaling
            self.mask = mask

        def forward(self, x):
            x2 = x.reshape(-1, x.shape[-1])
            base = torch.nn.functional.linear(x2, self.w, self.b)
            xd = (x2.float() * self.mask * scale).to(x.dtype)          # DropoutCast
            lo = torch.nn.functional.linear(torch.nn.functional.linear(xd, self.a.to(x.dtype)),
                                            self.bb.to(x.dtype))
            return ops_ref.scaled_add_ref(base, lo, self.s).view(*x.shape[:-1], -1)

    t = {name: Twin(getattr(layer, name),
                    _mask_of_bits(bits[name], getattr(layer, name).in_features))
         for name in qlora._PROJ}
    hr = h.clone().requires_grad_()
    x = ops_ref.rmsnorm_ref(hr, layer.ln1, shape.eps)
    q = t["q"](x).view(B, S, shape.heads, 128).transpose(1, 2)
    kk = t["k"](x).view(B, S, shape.kv_heads, 128).transpose(1, 2)
    v = t["v"](x).view(B, S, shape.kv_heads, 128).transpose(1, 2)
    q, kk = ops_ref.rope_ref(q, kk, cos, sin)
    rep = shape.heads // shape.kv_heads
    a = torch.nn.functional.scaled_dot_product_attention(
        q.float(), kk.float().repeat_interleave(rep, 1), v.float().repeat_interleave(rep, 1),
        is_causal=True).to(torch.bfloat16)
    hh = hr + t["o"](a.transpose(1, 2).reshape(B, S, -1))
    x2 = ops_ref.rmsnorm_ref(hh, layer.ln2, shape.eps)
    m = ops_ref.swiglu_ref(t["gate"](x2), t["up"](x2)).to(torch.bfloat16)
    ref = hh + t["down"](m)
    ref.backward(gout)

    torch.testing.assert_close(out.detach().float(), ref.detach().float(), rtol=5e-2, atol=5e-2)
    torch.testing.assert_close(hg.grad.float(), hr.grad.float(), rtol=5e-2, atol=5e-2)
    for name in qlora._PROJ:
        mod, tw = getattr(layer, name), t[name]
        for mine, theirs in ((mod.lora_A.grad, tw.a.grad), (mod.lora_B.grad, tw.bb.grad)):
            rel = (mine.float() - theirs.float()).norm() / theirs.float().norm()
            assert rel < 5e-2, (name, float(rel))


def test_many_long_token_steps_in_a_row(cuda):
    """Twenty consecutive training steps of 7B-shaped layers at the step's token count (4 x
    4096), each followed by a read of the tensor-core error flag, and the launch monitor after
    each: every step's loss is finite, no bounded wait gives up, and no traced launch is left
    with CTAs that started and never finished."""
    import ctypes
    from hackathon_b200 import _lib
    from hackathon_b200.gemm import device_error
    from hackathon_b200.qlora import QwenQLoRA, make_optimizer, preset, synthetic_batch, \
        train_step
    shape = preset("7b", layers=2)
    model = QwenQLoRA(shape, cuda, seed=0)
    opt = make_optimizer(model)
    data = [synthetic_batch(shape, 4, 4096, cuda, seed=i) for i in range(2)]
    lib = _lib.load()
    buf = ctypes.create_string_buffer(1024)
    for i in range(20):
        ids, labels = data[i % 2]
        loss = float(train_step(model, opt, ids, labels))
        device_error()
        assert np.isfinite(loss), (i, loss)
        assert lib.qb_monitor_report(cuda.index or 0, buf, len(buf)) == 0
        assert "no CTA of these launches is running" in buf.value.decode(), (i, buf.value)


def test_adapter_shadow_matches_per_use_conversion(cuda):
    """The shadow's bf16 operands (one qb_adapter_pack launch) equal the per-projection
    conversions bit for bit, follow an optimizer step, and a step with the shadow attached gives
    the same loss and adapter gradients as one that converts at every use."""
    from hackathon_b200.qlora import QwenQLoRA, make_optimizer, preset, synthetic_batch
    bf16 = torch.bfloat16
    shape = preset("0.5b", layers=2, lora_dropout=0.1)
    model = QwenQLoRA(shape, cuda, seed=0)
    ids, labels = synthetic_batch(shape, 1, 128, cuda, seed=3)

    def check_shadow():
        sh = model.adapter_shadow
        for m in sh.modules:
            a16, sb16 = m._shadow16
            assert torch.equal(a16, m.lora_A.detach().to(bf16))
            assert torch.equal(sb16, (m.lora_B.detach() * m.scaling).to(bf16))
        for g, u in sh.pairs:
            r = g.lora_B.shape[1]
            b1g, b1u = g._shadow_b1
            assert torch.equal(b1g[:, :r], (g.lora_B.detach() * g.scaling).to(bf16))
            assert torch.equal(b1u[:, r:], (u.lora_B.detach() * u.scaling).to(bf16))
            assert not b1g[:, r:].any() and not b1u[:, :r].any()

    opt = make_optimizer(model, lr=1e-2)
    model.train()
    loss, _ = model(ids, labels)
    check_shadow()
    loss.backward()
    opt.step()                      # fused AdamW: in place, no version bump
    opt.zero_grad(set_to_none=True)
    out = []
    for attached in (True, False):
        if not attached:
            model.adapter_shadow.detach()
            model.adapter_shadow = None
        loss, _ = model(ids, labels)
        if attached:
            check_shadow()          # refreshed by this forward: the stepped adapters
        loss.backward()
        out.append((loss.detach(), torch.cat([p.grad.flatten()
                                              for p in model.adapter_parameters()])))
        opt.zero_grad(set_to_none=True)
    assert torch.equal(out[0][0], out[1][0])
    assert torch.equal(out[0][1], out[1][1])


def test_step_launches_no_library_gemm(cuda):
    """One 7B-shaped training step (2 layers, the step's 4 x 4096 tokens) launches no cuBLAS /
    cuBLASLt / CUTLASS GEMM: every matrix product - projections, their input gradients, the LoRA
    products and weight gradients, the head - is one of this library's tcgen05 kernels. Kernel
    names come from the CUDA activity of torch.profiler; attention stays on cuDNN's SDPA."""
    from torch.profiler import ProfilerActivity, profile
    from hackathon_b200.qlora import QwenQLoRA, make_optimizer, preset, synthetic_batch, \
        train_step
    shape = preset("7b", layers=2)
    model = QwenQLoRA(shape, cuda, seed=0)
    opt = make_optimizer(model)
    ids, labels = synthetic_batch(shape, 4, 4096, cuda, seed=0)
    train_step(model, opt, ids, labels)          # warm-up: workspaces, library handles
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        train_step(model, opt, ids, labels)
        torch.cuda.synchronize()
    names = {e.key for e in prof.key_averages() if e.device_time_total > 0}
    ours = [n for n in names if "tc_gemm_kernel" in n]
    assert ours, sorted(names)
    library_gemms = [n for n in names if any(k in n.lower() for k in
                                             ("cublas", "nvjet", "cutlass", "xmma", "gemv",
                                              "splitkreduce", "sm100_gemm", "sm90_gemm"))]
    assert not library_gemms, library_gemms

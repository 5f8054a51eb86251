"""Pins the CPU oracle to the reference: every restatement in oracle/ against the fixtures the
reference's own kernels produced (tests/golden/make_golden.py). No GPU needed."""

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import nf4_ref, ops_ref


# ----------------------------------------------------------------------------------- NF4

def _nf4_cases(g):
    return sorted({int(k.split("_")[1]) for k in g if k.startswith("nf4_") and k[4].isdigit()})


def _nf4_args(g, i):
    rows, cols, bs, nested, bs2 = (int(v) for v in g[f"nf4_{i}_meta"])
    n = rows * cols
    if nested:
        return (g[f"nf4_{i}_packed"], n, g[f"nf4_{i}_absmax_q"], True, g["nf4_code2"],
                g[f"nf4_{i}_absmax2"], float(g[f"nf4_{i}_offset"][0]), bs, bs2)
    return (g[f"nf4_{i}_packed"], n, g[f"nf4_{i}_absmax"], False, None, None, 0.0, bs, bs2)


def test_nf4_dequant_matches_reference_bit_for_bit():
    g = golden("nf4")
    cases = _nf4_cases(g)
    assert len(cases) == 5
    for i in cases:
        args = _nf4_args(g, i)
        f32 = nf4_ref.dequant_nf4(*args, out="f32")
        f16 = nf4_ref.dequant_nf4(*args, out="f16")
        ref32 = g[f"nf4_{i}_f32"].reshape(-1)
        ref16 = g[f"nf4_{i}_f16"].reshape(-1)
        assert np.array_equal(f32.view(np.uint32), ref32.view(np.uint32)), i
        assert np.array_equal(f16.view(np.uint16), ref16.view(np.uint16)), i


def test_nf4_bf16_is_rne_of_the_reference_fp32():
    """bf16 parity goes through the fp32 fixture: the interpreter truncates where the compiled
    kernel rounds to nearest even; the fixture shows the truncation."""
    g = golden("nf4")
    args = _nf4_args(g, 0)
    bf16 = nf4_ref.dequant_nf4(*args, out="bf16")
    ref32 = g["nf4_0_f32"].reshape(-1)
    assert np.array_equal(bf16, nf4_ref.f32_to_bf16_bits(ref32))
    truncated = (ref32.view(np.uint32) >> 16).astype(np.uint16)
    assert np.array_equal(g["nf4_0_bf16_interp"].reshape(-1), truncated)


def test_bf16_rounding_is_nearest_even():
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5e-8, 3.0e38, np.inf], dtype=np.float32)
    # 1 + 2^-8 is a tie between 1 and 1 + 2^-7: even mantissa (1.0) wins; 1 + 3*2^-8 rounds up
    bits = nf4_ref.f32_to_bf16_bits(x)
    back = nf4_ref.bf16_bits_to_f32(bits)
    assert back[0] == 1.0 and back[1] == 1.0 and back[2] == np.float32(1.015625)
    ref = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(bits, ref)


def test_nf4_quantiser_round_trip():
    rng = np.random.default_rng(3)
    w = (rng.standard_normal(64 * 40) * 0.02).astype(np.float32)
    packed, absmax = nf4_ref.quantize_nf4(w, 64)
    code2 = ops_code2()
    q, absmax2, offset = nf4_ref.double_quant(absmax, code2, 256)
    back = nf4_ref.dequant_nf4(packed, w.size, q, True, code2, absmax2, offset, 64, 256,
                               out="f32")
    # NF4 spacing is at most ~0.3 of the block absmax; double quant adds < 1% of the scale
    blocks = np.abs(w).reshape(-1, 64).max(1).repeat(64)
    assert np.all(np.abs(back - w) <= 0.17 * blocks + 1e-6)


def ops_code2():
    from hackathon_b200.nf4 import signed_dynamic_code
    return signed_dynamic_code().numpy()


def test_code2_table_shape():
    c = ops_code2()
    assert c.shape == (256,) and np.all(np.diff(c) >= 0) and c[-1] == 1.0 and c.min() < 0
    assert 0.0 in c


# ----------------------------------------------------------------------------------- LoRA

def test_dropout_mask_matches_reference_bits():
    g = golden("lora")
    x = g["drop_x"]
    for i in range(4):
        seed, p_micro = (int(v) for v in g[f"drop_{i}_meta"])
        p = p_micro / 1e6
        keep = np.unpackbits(g[f"drop_{i}_keep"])[: x.size].reshape(x.shape).astype(bool)
        dx_keep = np.unpackbits(g[f"drop_{i}_dx_keep"])[: x.size].reshape(x.shape).astype(bool)
        if p > 0:
            mine = nf4_ref.dropout_keep(seed, x.shape[0], x.shape[1], p)
            assert np.array_equal(mine, keep), i
            assert np.array_equal(mine, dx_keep), i      # the backward regenerates the mask
        scale = 1.0 / (1.0 - p) if p > 0 else 1.0
        y = nf4_ref.dropout_scale(x, p, seed, scale)
        assert np.array_equal(y != 0, keep & (x != 0)), i
        if f"drop_{i}_y" in g:
            assert np.array_equal(y.view(np.uint32), g[f"drop_{i}_y"].view(np.uint32))


def test_scaled_add_matches_reference():
    g = golden("lora")
    out = ops_ref.scaled_add_ref(torch.from_numpy(g["sadd_base"]),
                                 torch.from_numpy(g["sadd_lo"]).half(), 2.0)
    torch.testing.assert_close(out, torch.from_numpy(g["sadd_y"]), rtol=1e-6, atol=1e-6)


# ----------------------------------------------------------------------------------- RMSNorm

@pytest.mark.parametrize("i", range(6))
def test_rmsnorm_oracle_matches_reference(i):
    g = golden("rmsnorm")
    x = torch.from_numpy(g[f"rms_{i}_x"]).requires_grad_()
    w = torch.from_numpy(g[f"rms_{i}_w"])
    y = ops_ref.rmsnorm_ref(x, w, 1e-6)
    ref_y = torch.from_numpy(g[f"rms_{i}_y"])
    assert y.dtype == ref_y.dtype
    tol = 2e-3 if x.dtype == torch.float16 else 1e-5
    torch.testing.assert_close(y, ref_y, rtol=tol, atol=tol)
    y.backward(torch.from_numpy(g[f"rms_{i}_g"]))
    torch.testing.assert_close(x.grad, torch.from_numpy(g[f"rms_{i}_dx"]), rtol=tol, atol=tol)


# ----------------------------------------------------------------------------------- RoPE

@pytest.mark.parametrize("i", range(8))
def test_rope_oracle_matches_reference(i):
    g = golden("rope")
    half, equal, _ = (int(v) for v in g[f"rope_{i}_meta"])
    t = {k: torch.from_numpy(g[f"rope_{i}_{k}"]) for k in
         ("q", "k", "cos", "sin", "qo", "ko", "gq", "gk", "dq", "dk")}
    q = t["q"].clone().requires_grad_()
    k = t["k"].clone().requires_grad_()
    qo, ko = ops_ref.rope_ref(q, k, t["cos"], t["sin"])
    tol = (2e-3 if half else 1e-5) * (1 if equal else 4)
    torch.testing.assert_close(qo, t["qo"], rtol=tol, atol=tol)
    torch.testing.assert_close(ko, t["ko"], rtol=tol, atol=tol)
    torch.autograd.backward((qo, ko), (t["gq"], t["gk"]))
    torch.testing.assert_close(q.grad, t["dq"], rtol=tol, atol=tol)
    torch.testing.assert_close(k.grad, t["dk"], rtol=tol, atol=tol)


# ----------------------------------------------------------------------------------- SwiGLU

@pytest.mark.parametrize("i", range(2))
def test_swiglu_oracle_matches_reference(i):
    g = golden("swiglu")
    gate = torch.from_numpy(g[f"swiglu_{i}_gate"]).float().requires_grad_()
    up = torch.from_numpy(g[f"swiglu_{i}_up"]).float().requires_grad_()
    y = ops_ref.swiglu_ref(gate, up)
    tol = 2e-3 if g[f"swiglu_{i}_y"].dtype == np.float16 else 1e-5
    torch.testing.assert_close(y, torch.from_numpy(g[f"swiglu_{i}_y"]).float(), rtol=tol, atol=tol)
    y.backward(torch.from_numpy(g[f"swiglu_{i}_grad"]).float())
    torch.testing.assert_close(gate.grad, torch.from_numpy(g[f"swiglu_{i}_dgate"]).float(),
                               rtol=tol, atol=tol)
    torch.testing.assert_close(up.grad, torch.from_numpy(g[f"swiglu_{i}_dup"]).float(),
                               rtol=tol, atol=tol)


# ----------------------------------------------------------------------------------- CE

@pytest.mark.parametrize("i", range(6))
def test_ce_oracle_matches_reference(i):
    g = golden("ce")
    vocab = int(g[f"ce_{i}_vocab"][0])
    hidden = torch.from_numpy(g[f"ce_v{vocab}_hidden"]).requires_grad_()
    weight = torch.from_numpy(g[f"ce_v{vocab}_weight"])
    labels = torch.from_numpy(g[f"ce_v{vocab}_labels"])
    items = int(g[f"ce_{i}_num_items"][0])
    num_items = None if items < 0 else torch.tensor(items)
    loss, entropy, token_loss, correct, labelled, _ = ops_ref.ce_ref(hidden, weight, labels,
                                                                     num_items)
    torch.testing.assert_close(loss, torch.tensor(g[f"ce_{i}_loss"][0]), rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(entropy, torch.from_numpy(g[f"ce_{i}_entropy"]), rtol=1e-5,
                               atol=1e-5)
    torch.testing.assert_close(token_loss, torch.from_numpy(g[f"ce_{i}_token_loss"]), rtol=1e-5,
                               atol=1e-5)
    assert int(correct) == int(g[f"ce_{i}_correct"][0])
    assert int(labelled) == int(g[f"ce_{i}_labelled"][0])
    (loss * 1024.0).backward()
    torch.testing.assert_close(hidden.grad, torch.from_numpy(g[f"ce_{i}_grad"]), rtol=1e-4,
                               atol=1e-4)


def test_fused_head_loss_oracle_matches_reference():
    """fused_ce.fused_head_loss: fp16 head, padding dropped, metrics over real tokens."""
    g = golden("ce")
    hidden = torch.from_numpy(g["fce_hidden"]).requires_grad_()
    weight = torch.from_numpy(g["fce_weight"])
    labels = torch.from_numpy(g["fce_labels"])
    mask = torch.from_numpy(g["fce_mask"])
    items = (labels[:, 1:] != -100).sum()
    logits = (hidden.half() @ weight.half().t()).float()
    loss, entropy, token_loss, correct, labelled, _ = ops_ref.ce_ref(hidden, weight, labels,
                                                                     items, logits=logits)
    torch.testing.assert_close(loss, torch.tensor(g["fce_loss"][0]), rtol=2e-3, atol=2e-3)
    ent_sum = (entropy * mask).sum()
    torch.testing.assert_close(ent_sum, torch.tensor(g["fce_entropy_sum"][0]), rtol=2e-3,
                               atol=2e-3)
    assert int(correct) == int(g["fce_correct"][0])
    assert int(labelled) == int(g["fce_labelled"][0])
    torch.testing.assert_close(token_loss, torch.from_numpy(g["fce_token_loss"]), rtol=2e-3,
                               atol=2e-3)


def test_c_restatement_matches_reference():
    """oracle/nf4_ref.c (the CPU baseline of the dequant sweep) against the fixtures."""
    from oracle import c_ref
    g = golden("nf4")
    for i in (0, 2, 4):
        rows, cols, bs, _, bs2 = (int(v) for v in g[f"nf4_{i}_meta"])
        got = c_ref.dequant_nf4_bf16(g[f"nf4_{i}_packed"], rows * cols, g[f"nf4_{i}_absmax_q"],
                                     g["nf4_code2"], g[f"nf4_{i}_absmax2"],
                                     float(g[f"nf4_{i}_offset"][0]), bs, bs2, threads=3)
        assert np.array_equal(got, nf4_ref.f32_to_bf16_bits(g[f"nf4_{i}_f32"].reshape(-1))), i

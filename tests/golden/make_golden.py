"""Generates tests/golden/*.npz by running the REFERENCE's own kernels on the CPU.

    TRITON_INTERPRET=1 python tests/golden/make_golden.py --ref <checkout of the reference>

The reference (imoshka2009-lab/hackathon, `solution/`) is Python + Triton; Triton's interpreter
runs its kernels on CPU tensors. This script runs only where the reference is checked out; the
fixtures it writes are what the tests read (nothing at test time touches the reference).

bitsandbytes is not installed, and the reference reads only one thing from it on this path: the
NF4 code book (`bnbf.get_4bit_type("nf4")`, solution/nf4.py:55-62). A stand-in module supplies
the QLoRA paper's table. Quantised inputs are produced by the oracle's own quantiser.

Caveat recorded in the fixtures: the interpreter converts fp32 -> bf16 by truncation, not
round-to-nearest-even, so bf16 outputs are stored as the interpreter produced them and the tests
compare bf16 through the fp32 fixture instead.
"""

import argparse
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


def _install_bnb_stub(torch, code):
    bnb = types.ModuleType("bitsandbytes")
    fn = types.ModuleType("bitsandbytes.functional")
    fn.get_4bit_type = lambda name, device=None: torch.tensor(code, dtype=torch.float32,
                                                              device=device)
    bnb.functional = fn
    sys.modules["bitsandbytes"] = bnb
    sys.modules["bitsandbytes.functional"] = fn


class _State:
    pass


def _bits16(t):
    import torch
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def gen_nf4(torch, sol, nf4_ref, code2):
    out = {}
    rng = np.random.default_rng(0)
    cases = [((96, 320), 64, True), ((96, 320), 64, False), ((128, 512), 64, True),
             ((64, 384), 128, False), ((40, 130), 64, True)]
    for i, (shape, bs, nested) in enumerate(cases):
        w = (rng.standard_normal(shape) * 0.05).astype(np.float32)
        packed, absmax = nf4_ref.quantize_nf4(w, blocksize=bs)
        st = _State()
        st.shape, st.blocksize, st.nested, st.quant_type = shape, bs, nested, "nf4"
        if nested:
            q, absmax2, offset = nf4_ref.double_quant(absmax, code2, 256)
            st.absmax = torch.from_numpy(q)
            st.offset = float(offset)
            st.state2 = _State()
            st.state2.code = torch.from_numpy(code2)
            st.state2.absmax = torch.from_numpy(absmax2)
            st.state2.blocksize = 256
            out[f"nf4_{i}_absmax_q"] = q
            out[f"nf4_{i}_absmax2"] = absmax2
            out[f"nf4_{i}_offset"] = np.array([offset], dtype=np.float32)
        else:
            st.absmax = torch.from_numpy(absmax)
            st.state2 = None
        out[f"nf4_{i}_absmax"] = absmax
        out[f"nf4_{i}_packed"] = packed
        out[f"nf4_{i}_meta"] = np.array([shape[0], shape[1], bs, int(nested), 256], np.int64)
        pk = torch.from_numpy(packed).reshape(-1, 1)
        out[f"nf4_{i}_f32"] = sol.nf4.dequantize_nf4(pk, st, torch.float32).numpy()
        out[f"nf4_{i}_f16"] = sol.nf4.dequantize_nf4(pk, st, torch.float16).numpy()
        if i == 0:  # documents the interpreter's truncating bf16 cast
            out[f"nf4_{i}_bf16_interp"] = _bits16(sol.nf4.dequantize_nf4(pk, st, torch.bfloat16))
    out["nf4_code2"] = code2
    return out


def gen_rmsnorm(torch, sol):
    out = {}
    i = 0
    for hidden in (1536, 1000):
        for xd, wd in ((torch.float32, torch.float32), (torch.float16, torch.float32),
                       (torch.float16, torch.float16)):
            torch.manual_seed(0)
            weight = (1 + 0.1 * torch.randn(hidden)).to(wd)
            x = torch.randn(2, 3, hidden, dtype=xd, requires_grad=True)
            y = sol.rmsnorm.rmsnorm(x, weight, 1e-6)
            g = torch.randn(y.shape, dtype=torch.float32).to(y.dtype)
            y.backward(g)
            out[f"rms_{i}_x"] = x.detach().numpy()
            out[f"rms_{i}_w"] = weight.numpy()
            out[f"rms_{i}_g"] = g.numpy()
            out[f"rms_{i}_y"] = y.detach().numpy()
            out[f"rms_{i}_dx"] = x.grad.numpy()
            i += 1
    return out


def gen_rope(torch, sol, ops_ref):
    out = {}
    i = 0
    B, S, HQ, HK, D = 2, 3, 6, 2, 128
    for dtype in (torch.float32, torch.float16):
        for equal in (True, False):
            for batch_cos in (1, None):
                torch.manual_seed(0)
                q = torch.randn(B, S, HQ, D, dtype=dtype).transpose(1, 2).requires_grad_()
                k = torch.randn(B, S, HK, D, dtype=dtype).transpose(1, 2).requires_grad_()
                if equal:
                    cos, sin = ops_ref.qwen_cos_sin(batch_cos or B, S, D, dtype=dtype)
                else:
                    cos = torch.randn(batch_cos or B, S, D, dtype=dtype)
                    sin = torch.randn(batch_cos or B, S, D, dtype=dtype)
                qo, ko = sol.rope.TritonRoPE.apply(q, k, cos, sin)
                gq, gk = torch.randn(qo.shape, dtype=dtype), torch.randn(ko.shape, dtype=dtype)
                torch.autograd.backward((qo, ko), (gq, gk))
                for name, t in (("q", q.detach()), ("k", k.detach()), ("cos", cos), ("sin", sin),
                                ("qo", qo.detach()), ("ko", ko.detach()), ("gq", gq), ("gk", gk),
                                ("dq", q.grad), ("dk", k.grad)):
                    out[f"rope_{i}_{name}"] = t.contiguous().numpy()
                out[f"rope_{i}_meta"] = np.array([int(dtype == torch.float16), int(equal),
                                                  batch_cos or B], np.int64)
                i += 1
    return out


def gen_swiglu(torch, sol):
    out = {}
    for i, dtype in enumerate((torch.float32, torch.float16)):
        torch.manual_seed(0)
        gate = torch.randn(3, 7, 201, dtype=dtype, requires_grad=True)   # 201: a ragged tail
        up = torch.randn(3, 7, 201, dtype=dtype, requires_grad=True)
        grad = torch.randn(3, 7, 201, dtype=dtype)
        y = sol.swiglu.swiglu(gate, up)
        y.backward(grad)
        for name, t in (("gate", gate.detach()), ("up", up.detach()), ("grad", grad), ("y", y),
                        ("dgate", gate.grad), ("dup", up.grad)):
            out[f"swiglu_{i}_{name}"] = t.detach().numpy()
    return out


def gen_lora(torch, sol):
    out = {}
    for i, (seed, p) in enumerate(((1234, 0.05), (4321, 0.05), (2**33 + 5, 0.3), (7, 0.0))):
        torch.manual_seed(0)
        x = torch.randn(32, 1536, requires_grad=True)
        y = sol.lora.DropoutCast.apply(x, p, seed, torch.float32)
        y.backward(torch.ones_like(y))
        if i == 0:
            out["drop_x"] = x.detach().numpy()
        # y is x * keep * scale: store the mask (bits) and, for one case, the exact result
        out[f"drop_{i}_keep"] = np.packbits(y.detach().numpy() != 0)
        out[f"drop_{i}_dx_keep"] = np.packbits(x.grad.numpy() != 0)
        if i == 0:
            out[f"drop_{i}_y"] = y.detach().numpy()
        out[f"drop_{i}_meta"] = np.array([seed, int(round(p * 1e6))], np.int64)
    torch.manual_seed(0)
    base = torch.randn(2, 3, 256, requires_grad=True)
    lo = torch.randn(2, 3, 256, dtype=torch.float16, requires_grad=True)
    y = sol.lora.ScaledAdd.apply(base, lo, 2.0)
    g = torch.randn(y.shape)
    y.backward(g)
    out.update({"sadd_base": base.detach().numpy(), "sadd_lo": lo.detach().float().numpy(),
                "sadd_y": y.detach().numpy(), "sadd_g": g.numpy(),
                "sadd_dbase": base.grad.numpy(), "sadd_dlo": lo.grad.float().numpy()})
    return out


def gen_ce(torch, sol):
    out = {}
    i = 0
    B, T, H = 2, 9, 16
    for vocab in (1000, 4096, 9001):
        for with_items in (True, False):
            torch.manual_seed(0)
            hidden = torch.randn(B, T, H, requires_grad=True)
            weight = 0.05 * torch.randn(vocab, H)
            labels = torch.randint(0, vocab, (B, T))
            labels[:, : T // 3] = -100
            labels[1, -2:] = -100
            num_items = (labels[:, 1:] != -100).sum() if with_items else None
            loss, step = sol.cross_entropy.fused_causal_lm_loss(
                hidden, weight, labels, num_items_in_batch=num_items, chunk_rows=7)
            (loss * 1024.0).backward()
            if with_items:  # both cases of a vocab share the seeded inputs: store them once
                out.update({f"ce_v{vocab}_hidden": hidden.detach().numpy(),
                            f"ce_v{vocab}_weight": weight.numpy(),
                            f"ce_v{vocab}_labels": labels.numpy()})
            out.update({
                f"ce_{i}_vocab": np.array([vocab]),
                f"ce_{i}_num_items": np.array([-1 if num_items is None else int(num_items)]),
                f"ce_{i}_loss": np.array([float(loss)], np.float32),
                f"ce_{i}_token_loss": step.token_loss.detach().numpy(),
                f"ce_{i}_entropy": step.token_entropy.detach().numpy(),
                f"ce_{i}_correct": np.array([int(step.correct)]),
                f"ce_{i}_labelled": np.array([int(step.labelled)]),
                f"ce_{i}_grad": hidden.grad.numpy(),
            })
            i += 1
    # the earlier API (fused_ce.py): fp16 head, padding dropped, labelled rows first
    torch.manual_seed(0)
    b, t, h, v = 2, 12, 32, 500
    hidden = torch.randn(b, t, h, requires_grad=True)
    weight = (torch.randn(v, h) * 0.05).half().float()
    labels = torch.randint(0, v, (b, t))
    labels[:, :3] = -100
    mask = torch.ones(b, t, dtype=torch.long)
    mask[1, 9:] = 0
    labels[1, 9:] = -100
    items = (labels[:, 1:] != -100).sum()
    loss, stats = sol.fused_ce.fused_head_loss(hidden, weight, labels, mask, items)
    (loss * 1024).backward()
    out.update({"fce_hidden": hidden.detach().numpy(), "fce_weight": weight.numpy(),
                "fce_labels": labels.numpy(), "fce_mask": mask.numpy(),
                "fce_loss": np.array([float(loss)], np.float32),
                "fce_token_loss": stats.token_loss.detach().numpy(),
                "fce_entropy_sum": np.array([float(stats.entropy_sum)], np.float32),
                "fce_correct": np.array([int(stats.correct)]),
                "fce_labelled": np.array([int(stats.labelled)]),
                "fce_grad": hidden.grad.numpy()})
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="checkout of the reference (its solution/ package)")
    args = ap.parse_args()
    if os.environ.get("TRITON_INTERPRET") != "1":
        sys.exit("run with TRITON_INTERPRET=1 (the reference's kernels run in Triton's CPU interpreter)")
    import torch

    sys.path.insert(0, ROOT)
    sys.path.insert(0, args.ref)
    from oracle import nf4_ref, ops_ref
    from hackathon_b200.nf4 import signed_dynamic_code

    _install_bnb_stub(torch, nf4_ref.NF4_CODE.tolist())
    import solution.cross_entropy
    import solution.fused_ce
    import solution.lora
    import solution.nf4
    import solution.rmsnorm
    import solution.rope
    import solution.swiglu
    sol = sys.modules["solution"]

    code2 = signed_dynamic_code().numpy()
    parts = {
        "nf4": gen_nf4(torch, sol, nf4_ref, code2),
        "rmsnorm": gen_rmsnorm(torch, sol),
        "rope": gen_rope(torch, sol, ops_ref),
        "swiglu": gen_swiglu(torch, sol),
        "lora": gen_lora(torch, sol),
        "ce": gen_ce(torch, sol),
    }
    for name, arrays in parts.items():
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(path, **arrays)
        print(f"{path}: {len(arrays)} arrays, {os.path.getsize(path) / 1024:.0f} KiB")


if __name__ == "__main__":
    main()

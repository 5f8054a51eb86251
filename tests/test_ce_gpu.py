"""Parity of the fused linear cross-entropy paths (C-ABI kernels) with the reference fixtures and
the CPU oracle: loss, per-token loss, entropy, accuracy counts and the hidden-state gradient."""

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import ops_ref

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("i", range(6))
def test_fused_causal_lm_loss_vs_reference_fixtures(cuda, i):
    from hackathon_b200.cross_entropy import fused_causal_lm_loss
    g = golden("ce")
    vocab = int(g[f"ce_{i}_vocab"][0])
    hidden = torch.from_numpy(g[f"ce_v{vocab}_hidden"]).to(cuda).requires_grad_()
    weight = torch.from_numpy(g[f"ce_v{vocab}_weight"]).to(cuda)
    labels = torch.from_numpy(g[f"ce_v{vocab}_labels"]).to(cuda)
    items = int(g[f"ce_{i}_num_items"][0])
    num_items = None if items < 0 else torch.tensor(items, device=cuda)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False   # fp32 logits, as the fixture's CPU matmul
    try:
        loss, step = fused_causal_lm_loss(hidden, weight, labels, num_items_in_batch=num_items,
                                          chunk_rows=7)
        (loss * 1024.0).backward()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    torch.testing.assert_close(loss.cpu(), torch.tensor(g[f"ce_{i}_loss"][0]), rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(step.token_loss.cpu(), torch.from_numpy(g[f"ce_{i}_token_loss"]),
                               rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(step.token_entropy.cpu(), torch.from_numpy(g[f"ce_{i}_entropy"]),
                               rtol=1e-4, atol=1e-4)
    assert int(step.correct) == int(g[f"ce_{i}_correct"][0])
    assert int(step.labelled) == int(g[f"ce_{i}_labelled"][0])
    torch.testing.assert_close(hidden.grad.cpu(), torch.from_numpy(g[f"ce_{i}_grad"]),
                               rtol=1e-3, atol=1e-4)


def test_fused_head_loss_vs_reference_fixture(cuda):
    from hackathon_b200.fused_ce import fused_head_loss
    g = golden("ce")
    hidden = torch.from_numpy(g["fce_hidden"]).to(cuda).requires_grad_()
    weight = torch.from_numpy(g["fce_weight"]).to(cuda)
    labels = torch.from_numpy(g["fce_labels"]).to(cuda)
    mask = torch.from_numpy(g["fce_mask"]).to(cuda)
    items = (labels[:, 1:] != -100).sum()
    loss, stats = fused_head_loss(hidden, weight, labels, mask, items)
    (loss * 1024).backward()
    torch.testing.assert_close(loss.cpu(), torch.tensor(g["fce_loss"][0]), rtol=2e-3, atol=2e-3)
    torch.testing.assert_close(stats.entropy_sum.cpu(), torch.tensor(g["fce_entropy_sum"][0]),
                               rtol=2e-3, atol=2e-3)
    assert int(stats.correct) == int(g["fce_correct"][0])
    assert int(stats.labelled) == int(g["fce_labelled"][0])
    torch.testing.assert_close(stats.token_loss.cpu(), torch.from_numpy(g["fce_token_loss"]),
                               rtol=2e-3, atol=2e-3)
    torch.testing.assert_close(hidden.grad.cpu(), torch.from_numpy(g["fce_grad"]), rtol=2e-2,
                               atol=2e-3)


@pytest.mark.parametrize("vocab", [1000, 4096, 9001])
@pytest.mark.parametrize("with_num_items", [True, False])
def test_fused_ce_matches_base_fp16_autocast(cuda, vocab, with_num_items):
    """The reference's own GPU test (test_cross_entropy.py:32-66) at its GPU shapes."""
    from hackathon_b200.cross_entropy import fused_causal_lm_loss
    torch.manual_seed(0)
    B, T, H = 4, 512, 1536
    hidden = torch.randn(B, T, H, device=cuda, requires_grad=True)
    weight = 0.05 * torch.randn(vocab, H, device=cuda)
    labels = torch.randint(0, vocab, (B, T), device=cuda)
    labels[:, : T // 3] = -100
    labels[1, -2:] = -100
    num_items = (labels[:, 1:] != -100).sum() if with_num_items else None
    hidden_ref = hidden.detach().cpu().clone().requires_grad_()
    with torch.autocast("cuda", dtype=torch.float16):
        loss, step = fused_causal_lm_loss(hidden, weight, labels, num_items_in_batch=num_items,
                                          chunk_rows=512)
    loss_ref, ent_ref, tok_ref, correct_ref, total_ref, _ = ops_ref.ce_ref(
        hidden_ref, weight.cpu(), labels.cpu(), None if num_items is None else num_items.cpu(),
        matmul_dtype=torch.float16)
    tol = 2e-3
    torch.testing.assert_close(loss.cpu(), loss_ref, atol=tol, rtol=tol)
    torch.testing.assert_close(step.token_entropy.cpu(), ent_ref, atol=tol, rtol=tol)
    torch.testing.assert_close(step.token_loss.cpu(), tok_ref, atol=tol, rtol=tol)
    assert int(step.labelled) == int(total_ref)
    assert abs(int(step.correct) - int(correct_ref)) <= 2     # argmax ties in fp16
    (loss * 1024.0).backward()
    (loss_ref * 1024.0).backward()
    torch.testing.assert_close(hidden.grad.cpu(), hidden_ref.grad, atol=5e-3, rtol=2e-2)


def _fp32_logits(hidden2d, weight):
    """Oracle logits: exact products of the bf16 operands, fp32 sums (no TF32)."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        return (hidden2d.float() @ weight.float().t()).cpu()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def test_fused_ce_baseline_shape_rows(cuda):
    """H=3584, V=152064 (Cfg3 shapes), bf16 activations and head on the tcgen05 path (logits only
    in TMEM): 256 rows against the oracle's fp32-accumulated logits; loss within 1e-4 relative."""
    from hackathon_b200.cross_entropy import fused_causal_lm_loss
    from hackathon_b200.gemm import device_error
    gen = torch.Generator(device=cuda).manual_seed(0)
    H, V, T = 3584, 152064, 256
    hidden = torch.randn(1, T, H, device=cuda, generator=gen).to(torch.bfloat16)
    weight = (torch.randn(V, H, device=cuda, generator=gen) * 0.02).to(torch.bfloat16)
    labels = torch.randint(0, V, (1, T), device=cuda, generator=gen)
    labels[torch.rand(1, T, device=cuda, generator=gen) < 0.1] = -100
    h = hidden.detach().requires_grad_()
    loss, step = fused_causal_lm_loss(h, weight, labels)
    loss.backward()
    device_error()
    logits = _fp32_logits(hidden[0], weight)
    hr = hidden.float().cpu().requires_grad_()
    loss_ref, ent_ref, tok_ref, correct_ref, total_ref, _ = ops_ref.ce_ref(
        hr, weight.float().cpu(), labels.cpu(), logits=logits[None])
    assert abs(float(loss) - float(loss_ref)) <= 1e-4 * abs(float(loss_ref))
    torch.testing.assert_close(step.token_loss.cpu(), tok_ref, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(step.token_entropy.cpu(), ent_ref, rtol=1e-4, atol=1e-3)
    assert int(step.labelled) == int(total_ref)
    assert abs(int(step.correct) - int(correct_ref)) <= 1
    # dH = dZ @ W with dZ = (softmax - onehot)/n: check against the oracle's autograd on the
    # same logits
    lg = logits.clone().requires_grad_()
    lref = ops_ref.ce_ref(None, None, labels.cpu(), logits=lg[None])[0]
    lref.backward()
    dh_ref = (lg.grad @ weight.float().cpu())
    torch.testing.assert_close(h.grad[0].float().cpu(), dh_ref, rtol=2e-2, atol=2e-3)


def _fp32_ce_reference(hidden2d, weight, target, chunk=1024):
    """The reference's loss (test_cross_entropy.py:9-30: fp32 logits, logsumexp, mean over the
    labelled rows) and dH = dZ W with dZ = (softmax - onehot) / n, chunked over rows so no more
    than `chunk` rows of fp32 logits exist at a time. Exact products of the bf16 operands with
    fp32 sums (TF32 off), on the GPU: a plain PyTorch fp32 reference of this floating-point op."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        w = weight.float()
        n = int((target != -100).sum())
        tok = torch.empty(target.shape[0], dtype=torch.float32, device=hidden2d.device)
        dh = torch.empty(hidden2d.shape, dtype=torch.float32, device=hidden2d.device)
        for a in range(0, target.shape[0], chunk):
            z = hidden2d[a:a + chunk].float() @ w.t()
            t = target[a:a + chunk]
            lab = t != -100
            lse = torch.logsumexp(z, dim=1)
            zl = z.gather(1, t.clamp(min=0)[:, None])[:, 0]
            tok[a:a + chunk] = torch.where(lab, lse - zl, torch.zeros_like(lse))
            p = torch.softmax(z, dim=1)
            p[torch.arange(t.shape[0], device=t.device)[lab], t[lab]] -= 1.0
            p[~lab] = 0.0
            dh[a:a + chunk] = (p / n) @ w
            del z, p
        return tok.sum() / n, tok, dh
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


@pytest.mark.parametrize("store_logits", [False, True])
def test_fused_ce_cfg3_full_size(cuda, store_logits):
    """Cfg3 at its full size: 16384 tokens (8 x 2048), hidden 3584, vocab 152064, hidden N(0,1),
    head N(0, 0.02), 10 % of labels -100, on the tcgen05 path (with the logits recomputed for
    the gradient, and with them stored). Every row's loss and every dH element against the
    chunked fp32 reference: loss within 1e-4 relative, dH within bf16 tolerance."""
    from hackathon_b200 import cross_entropy as ce
    from hackathon_b200.gemm import device_error
    gen = torch.Generator(device=cuda).manual_seed(3)
    B, S, H, V = 8, 2048, 3584, 152064
    hidden = torch.randn(B, S, H, device=cuda, generator=gen).to(torch.bfloat16)
    weight = (torch.randn(V, H, device=cuda, generator=gen) * 0.02).to(torch.bfloat16)
    labels = torch.randint(0, V, (B, S), device=cuda, generator=gen)
    labels[torch.rand(B, S, device=cuda, generator=gen) < 0.1] = -100
    prev = ce.STORE_LOGITS
    ce.STORE_LOGITS = store_logits
    try:
        h = hidden.detach().requires_grad_()
        loss, step = ce.fused_causal_lm_loss(h, weight, labels)
        loss.backward()
        device_error()
    finally:
        ce.STORE_LOGITS = prev
    target = ce.shift_labels_of(labels).reshape(-1)
    loss_ref, tok_ref, dh_ref = _fp32_ce_reference(hidden.reshape(-1, H), weight, target)
    assert abs(float(loss) - float(loss_ref)) <= 1e-4 * abs(float(loss_ref))
    torch.testing.assert_close(step.token_loss.reshape(-1), tok_ref, rtol=1e-4, atol=1e-4)
    assert int(step.labelled) == int((target != -100).sum())
    # per-row gradients (x n: the 1/n scale would make any absolute bound vacuous)
    n = int(step.labelled)
    got = h.grad.reshape(-1, H).float() * n
    want = dh_ref * n
    torch.testing.assert_close(got, want, rtol=2e-2, atol=1e-3)
    assert float((got - want).norm() / want.norm()) < 1e-2


def test_ce_rows_kernel_edge_cases(cuda):
    """Unlabelled rows (0 loss, 0 gradient), ties (first index wins), a ragged vocab and an
    unaligned row stride (scalar path)."""
    from hackathon_b200.fused_ce import ce_rows
    logits = torch.zeros(4, 1001, device=cuda)
    logits[0, 5] = 3.0
    logits[0, 9] = 3.0          # tie: argmax is 5
    logits[1, 1000] = 7.0
    logits[2] = torch.linspace(-3, 3, 1001, device=cuda)
    target = torch.tensor([5, 1000, -100, 0], device=cuda)
    want_lse = torch.logsumexp(logits.cpu(), -1)
    loss, ent, correct = ce_rows(logits.clone(), target, write_grad=False)
    assert correct.tolist() == [1, 1, 0, 1]   # row 3 is all zeros: argmax 0 == label 0
    assert loss[2].item() == 0.0
    torch.testing.assert_close(loss[0].cpu(), want_lse[0] - 3.0, rtol=1e-5, atol=1e-5)
    g = logits.clone()
    ce_rows(g, target, write_grad=True)
    assert torch.all(g[2] == 0)
    p = torch.softmax(logits.cpu(), -1)
    p[0, 5] -= 1
    torch.testing.assert_close(g[0].cpu(), p[0], rtol=1e-4, atol=1e-6)
    # unaligned stride
    wide = torch.randn(3, 1003, device=cuda)
    view = wide[:, :1001]
    l1, e1, _ = ce_rows(view, torch.tensor([1, 2, 3], device=cuda), write_grad=False)
    l2, e2, _ = ce_rows(view.contiguous(), torch.tensor([1, 2, 3], device=cuda), write_grad=False)
    torch.testing.assert_close(l1, l2)
    torch.testing.assert_close(e1, e2)


@pytest.mark.parametrize("vocab", [1000, 4096, 9001, 32768])
@pytest.mark.parametrize("rows,chunk", [(300, 4096), (600, 256)])
def test_tc_linear_ce_vs_oracle(cuda, vocab, rows, chunk):
    """The tcgen05 path at ragged vocab sizes and across row chunks: statistics against the
    fp32-logit oracle (loss 1e-4 relative), gradient within bf16 tolerance."""
    from hackathon_b200.cross_entropy import fused_causal_lm_loss
    from hackathon_b200.gemm import device_error
    gen = torch.Generator(device=cuda).manual_seed(vocab + rows)
    H = 512
    hidden = torch.randn(1, rows, H, device=cuda, generator=gen).to(torch.bfloat16)
    weight = (torch.randn(vocab, H, device=cuda, generator=gen) * 0.05).to(torch.bfloat16)
    labels = torch.randint(0, vocab, (1, rows), device=cuda, generator=gen)
    labels[:, :7] = -100
    h = hidden.detach().requires_grad_()
    items = (labels[:, 1:] != -100).sum()
    loss, step = fused_causal_lm_loss(h, weight, labels, num_items_in_batch=items,
                                      chunk_rows=chunk)
    (loss * 1024.0).backward()
    device_error()
    logits = _fp32_logits(hidden[0], weight)
    lg = logits.clone().requires_grad_()
    loss_ref, ent_ref, tok_ref, correct_ref, total_ref, _ = ops_ref.ce_ref(
        None, None, labels.cpu(), items.cpu(), logits=lg[None])
    (loss_ref * 1024.0).backward()
    assert abs(float(loss) - float(loss_ref)) <= 1e-4 * abs(float(loss_ref))
    torch.testing.assert_close(step.token_loss.cpu(), tok_ref, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(step.token_entropy.cpu(), ent_ref, rtol=1e-4, atol=1e-3)
    assert int(step.labelled) == int(total_ref)
    assert abs(int(step.correct) - int(correct_ref)) <= 1
    dh_ref = lg.grad @ weight.float().cpu()
    torch.testing.assert_close(h.grad[0].float().cpu(), dh_ref, rtol=2e-2, atol=2e-3)


def test_tc_linear_ce_unlabelled_rows_have_zero_gradient(cuda):
    from hackathon_b200.cross_entropy import fused_causal_lm_loss
    gen = torch.Generator(device=cuda).manual_seed(7)
    hidden = torch.randn(1, 130, 256, device=cuda, generator=gen).to(torch.bfloat16)
    weight = torch.randn(777, 256, device=cuda, generator=gen).to(torch.bfloat16)
    labels = torch.randint(0, 777, (1, 130), device=cuda, generator=gen)
    labels[0, 60:] = -100     # shifted targets 59.. are unlabelled
    h = hidden.detach().requires_grad_()
    loss, step = fused_causal_lm_loss(h, weight, labels)
    loss.backward()
    assert torch.all(h.grad[0, 59:] == 0)
    assert torch.all(step.token_loss[0, 59:] == 0)
    assert torch.isfinite(loss)


@pytest.mark.parametrize("vocab", [1000, 9001, 32771])
def test_tc_linear_ce_stored_logits_equal_recompute(cuda, vocab):
    """The dZ pass from stored fp32 logits (qb_linear_ce_stats_logits + qb_ce_grad_from_logits)
    gives the same dH, bit for bit, as the pass that recomputes the logits GEMM
    (qb_linear_ce_grad): same z, same arithmetic. Statistics are the same launch either way."""
    from hackathon_b200 import cross_entropy as ce
    from hackathon_b200.gemm import device_error
    gen = torch.Generator(device=cuda).manual_seed(vocab)
    rows, H = 700, 384
    h2 = torch.randn(rows, H, device=cuda, generator=gen).to(torch.bfloat16)
    w = (torch.randn(vocab, H, device=cuda, generator=gen) * 0.05).to(torch.bfloat16)
    tgt = torch.randint(0, vocab, (rows,), device=cuda, generator=gen)
    tgt[::5] = -100
    scale = torch.tensor([1.0 / 512], device=cuda)
    outs = []
    for keep in (True, False):
        tl = torch.empty(rows, device=cuda)
        en = torch.empty(rows, device=cuda)
        pr = torch.empty(rows, dtype=torch.int64, device=cuda)
        gh = torch.empty(rows, H, device=cuda)
        ce.linear_ce_tc(h2, w, tgt, tl, en, pr, gh, scale, 256, store_logits=keep)
        device_error()
        outs.append((tl, en, pr, gh))
    for a, b in zip(*outs):
        assert torch.equal(a, b)

"""Host logic of the data-parallel step on CPU: gloo ranks (world size 2) check that the global
label count and the flat adapter-gradient all-reduce give the gradient of the global mean loss."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _model():
    return torch.nn.Sequential(torch.nn.Linear(8, 5), torch.nn.Linear(5, 3))


def _worker(rank, world, port, out, overlap=True, bucket_bytes=64):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from hackathon_b200.dp import AdapterGradSync, global_label_count, shard_rows
        torch.manual_seed(0)
        model = _model()
        xs = torch.randn(10, 6, 8)
        labels = torch.randint(0, 3, (10, 6))
        labels[labels == 2] = -100
        lo, hi = shard_rows(10, rank, world)
        x, lb = xs[lo:hi], labels[lo:hi]
        sync = AdapterGradSync(model.parameters(), bucket_bytes=bucket_bytes, overlap=overlap)
        out[f"buckets{rank}"] = len(sync.buckets)
        n = global_label_count(lb)
        logits = model(x)[:, :-1]
        tgt = lb[:, 1:]
        loss = torch.nn.functional.cross_entropy(logits.reshape(-1, 3), tgt.reshape(-1),
                                                 ignore_index=-100, reduction="sum") / n
        loss.backward()
        sync()
        out[rank] = ([p.grad.clone() for p in model.parameters()], float(n))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(180)
@pytest.mark.parametrize("overlap", [True, False])
def test_dp_gradient_equals_global_mean_gradient(overlap):
    """Two gloo ranks, four parameters (40, 5, 15 and 3 values) in three buckets under a 64-byte
    limit: reduced from the backward's gradient hooks as each bucket completes (overlap) or all
    after the backward - either way every rank ends with the gradient of the global mean
    loss."""
    world = 2
    mgr = mp.get_context("spawn").Manager()   # no fork of this (possibly threaded) process
    out = mgr.dict()
    mp.spawn(_worker, args=(world, _free_port(), out, overlap), nprocs=world, join=True)
    torch.manual_seed(0)
    model = _model()
    xs = torch.randn(10, 6, 8)
    labels = torch.randint(0, 3, (10, 6))
    labels[labels == 2] = -100
    logits = model(xs)[:, :-1]
    loss = torch.nn.functional.cross_entropy(logits.reshape(-1, 3), labels[:, 1:].reshape(-1),
                                             ignore_index=-100)
    loss.backward()
    for r in range(world):
        assert out[f"buckets{r}"] == 3
        g, n = out[r]
        assert n == float((labels[:, 1:] != -100).sum())
        for a, b in zip(g, model.parameters()):
            torch.testing.assert_close(a, b.grad, rtol=1e-5, atol=1e-6)


def test_shard_rows_cover_everything():
    from hackathon_b200.dp import shard_rows
    for n in (0, 1, 7, 16):
        for w in (1, 2, 3, 8):
            spans = [shard_rows(n, r, w) for r in range(w)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))

"""Data-parallel training plumbing on CPU: gradient buckets, the overlapped
all-reduce over two gloo ranks, Muon's Newton-Schulz step, and a few training
steps of a tiny encoder. The encoder's token preparation and attention here
are the plain-torch reference ops (tests/encoder_ref.py); the GPU tests run the same model on the
library's kernels."""
import os
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from encoder_ref import RefOps, dense_masks, make_cells, tiny_config, to_torch
from tributary_b200.encoder import RTEncoder
from tributary_b200.train import GradBuckets, TrainStep, newton_schulz

KINDS = (0, 1, 2, 3)


def _model(seed):
    torch.manual_seed(seed)
    return RTEncoder(tiny_config(), ops=RefOps())


def _loss(model, cells):
    c, col, cat = to_torch(cells, "cpu")
    out = model(c, dense_masks(cells, KINDS, "cpu"), col, cat)
    return model.loss(out, c, cat)


def test_buckets_hold_the_autograd_gradients():
    cells = make_cells(3)
    ref = _model(0)
    _loss(ref, cells).backward()
    model = _model(0)
    buckets = GradBuckets(model.parameters(), bucket_bytes=64 << 10)
    assert len(buckets.buffers) > 1
    for _ in range(2):  # the second pass checks zero() restarts cleanly
        buckets.zero()
        _loss(model, cells).backward()
        buckets.finish()
        for (n, p), (_, q) in zip(model.named_parameters(), ref.named_parameters()):
            want = q.grad if q.grad is not None else torch.zeros_like(q)  # heads the target type leaves unused
            torch.testing.assert_close(p.grad, want, rtol=1e-5, atol=1e-7, msg=n)


def _rank(rank, world, init_file, result_file):
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
    try:
        model = _model(0)
        buckets = GradBuckets(model.parameters(), bucket_bytes=64 << 10)
        buckets.zero()
        _loss(model, make_cells(10 + rank)).backward()
        buckets.finish()
        if rank == 0:
            torch.save({n: p.grad.clone() for n, p in model.named_parameters()}, result_file)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_rank_allreduce_is_the_mean_gradient():
    world = 2
    with tempfile.TemporaryDirectory() as d:
        init_file, result_file = os.path.join(d, "init"), os.path.join(d, "grads.pt")
        mp.start_processes(_rank, args=(world, init_file, result_file), nprocs=world, start_method="spawn")
        got = torch.load(result_file)
    want = {n: torch.zeros_like(p) for n, p in _model(0).named_parameters()}
    for r in range(world):
        m = _model(0)
        _loss(m, make_cells(10 + r)).backward()
        for n, p in m.named_parameters():
            if p.grad is not None:
                want[n] += p.grad / world
    for n in want:
        torch.testing.assert_close(got[n], want[n], rtol=1e-5, atol=1e-7, msg=n)


def test_newton_schulz_orthogonalises():
    g = torch.randn(3, 48, 96)
    o = newton_schulz(g).float()
    s = torch.linalg.svdvals(o)
    assert s.min() > 0.5 and s.max() < 1.3  # the quintic's band around 1
    tall = newton_schulz(torch.randn(2, 96, 32)).float()
    assert tall.shape == (2, 96, 32)


def test_train_steps_reduce_the_loss():
    cells = make_cells(5)
    model = _model(1)
    step = TrainStep(model, muon_lr=0.01, adamw_lr=1e-3)
    c, col, cat = to_torch(cells, "cpu")
    masks = dense_masks(cells, KINDS, "cpu")
    losses = [float(step(c, masks, col, cat)) for _ in range(6)]
    assert all(np.isfinite(losses))
    assert losses[-1] < losses[0]

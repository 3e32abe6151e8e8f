"""The RT encoder on the library's kernels: one forward + backward of a small
encoder on the kernels (token preparation, tile-plan attention, unpermute)
against the same model (same weights, same bf16 autocast) on the plain-torch
reference ops with dense fp32 attention, and training steps with the tile plans
built by the prepass kernel."""
import numpy as np
import pytest
import torch

from encoder_ref import RefOps, dense_masks, make_cells, tiny_config, to_torch

pytestmark = pytest.mark.gpu

KINDS = (0, 1, 2, 3)
TOL_LOSS = 1e-2        # relative
TOL_GRAD_ALL = 2e-2    # relative L2 over all gradients together
TOL_GRAD_PARAM = 5e-2  # relative L2 per parameter tensor; looser because some gradients are
                       # near-cancelling sums (the categorical encoder bias: each token's softmax
                       # cross-entropy gradient sums to zero over the categories), where bf16
                       # rounding upstream is large relative to the small result


def _models(cfg):
    from tributary_b200.encoder import RTEncoder
    torch.manual_seed(7)
    kern = RTEncoder(cfg).cuda()
    ref = RTEncoder(cfg, ops=RefOps()).cuda()
    ref.load_state_dict(kern.state_dict())
    return kern, ref


def _run(model, cells, masks):
    c, col, cat = to_torch(cells, "cuda")
    with torch.autocast("cuda", dtype=torch.bfloat16):
        out = model(c, masks, col, cat)
        loss = model.loss(out, c, cat)
    loss.backward()
    return float(loss.detach())


def test_encoder_kernel_matches_dense_attention(cuda_lib):
    from tributary_b200.attention import device_status
    from tributary_b200.train import build_masks
    cfg = tiny_config(d_model=128, n_heads=2, d_head=64, d_ff=256, n_layers=2)
    cells = make_cells(21, B=2, S=384)
    kern, ref = _models(cfg)
    meta = {k: torch.from_numpy(cells[k].astype(np.int32) if cells[k].dtype == np.uint16 else cells[k]).cuda()
            for k in ("seq_row_ids", "column_ids", "is_padding", "fk_adj", "col_perm", "out_perm", "in_perm")}
    lk = _run(kern, cells, build_masks(meta, KINDS))
    lr = _run(ref, cells, dense_masks(cells, KINDS, "cuda"))
    torch.cuda.synchronize()
    assert device_status() == 0
    assert abs(lk - lr) <= TOL_LOSS * abs(lr)
    errs, num, den = {}, 0.0, 0.0
    for (n, p), (_, q) in zip(kern.named_parameters(), ref.named_parameters()):
        if q.grad is None or q.grad.norm() == 0:
            continue
        d2, r2 = float((p.grad - q.grad).norm() ** 2), float(q.grad.norm() ** 2)
        errs[n] = (d2 / r2) ** 0.5
        num, den = num + d2, den + r2
    assert len(errs) > 20
    assert (num / den) ** 0.5 < TOL_GRAD_ALL
    worst = sorted(errs.items(), key=lambda kv: -kv[1])[:8]
    assert worst[0][1] < TOL_GRAD_PARAM, worst


def test_train_steps_on_kernels(cuda_lib):
    from tributary_b200.attention import device_status
    from tributary_b200.encoder import RTEncoder
    from tributary_b200.train import TrainStep, build_masks
    cfg = tiny_config(d_model=128, n_heads=2, d_head=64, d_ff=256, n_layers=2)
    cells = make_cells(22, B=2, S=512)
    torch.manual_seed(3)
    model = RTEncoder(cfg).cuda()
    step = TrainStep(model, muon_lr=0.01, adamw_lr=1e-3)
    c, col, cat = to_torch(cells, "cuda")
    meta = {k: c[k] for k in ("seq_row_ids", "column_ids", "is_padding", "fk_adj", "col_perm", "out_perm", "in_perm")}
    losses = []
    for _ in range(5):
        losses.append(float(step(c, build_masks(meta, KINDS), col, cat)))
    torch.cuda.synchronize()
    assert device_status() == 0
    assert all(np.isfinite(losses)) and losses[-1] < losses[0]

"""Data-parallel training step of the RT encoder.

One process per GPU; every rank holds a full model replica and its own shard
of the batch (attention never crosses samples, confluence/confluence/model.py:
201-264), so the only exchange is the gradient mean over ranks
(confluence/confluence/train.py:212-214, jax.lax.pmean).

GradBuckets lays the gradients out in flat fp32 buckets (parameters in
reverse registration order, roughly the order backward produces them) and
points every parameter's .grad at its slice, so autograd accumulates straight
into the buckets. A post-accumulate hook counts each bucket's parameters; the
moment a bucket is complete its all-reduce is launched asynchronously (NCCL
over NVLink / NVSwitch on GPUs, gloo on CPU) and overlaps the rest of the
backward pass. finish() waits for all of them.

The optimizer follows confluence/confluence/optimizer.py (optax.contrib.muon):
Muon -- momentum, Nesterov, then the quintic Newton-Schulz orthogonalisation of
Jordan et al. (2024) -- for 2-D weights and AdamW for everything else, after
clipping the global gradient norm (config.py:64).
"""
from __future__ import annotations

import datetime
import math

import torch
import torch.distributed as dist


class RankFailure(RuntimeError):
    """A rank did not reach a training step within the heartbeat deadline (it
    left, crashed or stalled), or a gradient all-reduce failed or ran past its
    deadline. The process group has been aborted when this is raised, so no
    rank is left waiting in a collective."""


class Heartbeat:
    """Per-step liveness of the data-parallel ranks through the process
    group's key-value store (documentation/system_architecture.md:747 asks
    for failure detection around the gradient exchange).

    step(n) records that this rank reached step n, then waits until every rank
    has, before any collective of step n is launched. A rank that left between
    steps therefore surfaces on the host as RankFailure (naming the missing
    ranks) within `timeout_s`, instead of as a collective that never
    completes."""

    def __init__(self, group=None, store=None, timeout_s: float = 60.0, prefix: str = "rt_train_hb"):
        self.group = group
        self.store = store if store is not None else dist.distributed_c10d._get_default_store()
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.timeout = datetime.timedelta(seconds=timeout_s)
        self.prefix = prefix

    def _key(self, step, rank):
        return f"{self.prefix}/{step}/{rank}"

    def step(self, n: int):
        self.store.set(self._key(n, self.rank), "1")
        keys = [self._key(n, r) for r in range(self.world)]
        try:
            self.store.wait(keys, self.timeout)
        except Exception as e:  # the store raises on its deadline
            missing = [r for r, k in enumerate(keys) if not self.store.check([k])]
            abort(self.group)
            raise RankFailure(f"step {n}: rank(s) {missing} did not arrive within "
                              f"{self.timeout.total_seconds():g} s") from e
        if n >= 2:  # every rank has passed step n - 1, so nobody reads step n - 2 any more
            self.store.delete_key(self._key(n - 2, self.rank))


def abort(group=None):
    """Abort the process group (pending collectives end with an error on every
    rank instead of waiting for the missing one)."""
    try:
        dist.distributed_c10d._abort_process_group(group)
    except Exception:  # already aborted or destroyed
        pass


class GradBuckets:
    """Flat fp32 gradient buckets with overlapped all-reduce. ``reduce=False``
    keeps the buckets but launches no collective (each rank steps on its own
    gradients): the single-GPU step on the same device, for comparison."""

    def __init__(self, params, group=None, bucket_bytes: int = 32 << 20, reduce: bool = True):
        self.group = group
        joined = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if joined and reduce else 1
        self.avg = self.world > 1 and dist.get_backend(group) == "nccl"  # NCCL averages in the reduction
        params = [p for p in params if p.requires_grad]
        groups, cur, size = [], [], 0
        for p in reversed(params):
            if cur and size + 4 * p.numel() > bucket_bytes:
                groups.append(cur)
                cur, size = [], 0
            cur.append(p)
            size += 4 * p.numel()
        if cur:
            groups.append(cur)
        self.params = groups
        self.buffers, self.views = [], []
        for i, grp in enumerate(groups):
            buf = torch.zeros(sum(p.numel() for p in grp), dtype=torch.float32, device=grp[0].device)
            off = 0
            views = []
            for p in grp:
                v = buf[off:off + p.numel()].view_as(p)
                off += p.numel()
                p.grad = v
                views.append(v)
                p.register_post_accumulate_grad_hook(self._hook(i, len(views) - 1))
            self.buffers.append(buf)
            self.views.append(views)
        self.pending = [len(g) for g in groups]
        self.works = []
        self.launch_error = None
        self.launched = [False] * len(groups)
        # defer: the hooks only count (a backward recorded into a CUDA graph
        # launches no collective; reduce_all() exchanges the buckets after it)
        self.defer = False

    @property
    def bucket_sizes(self):
        return [b.numel() * 4 for b in self.buffers]

    def _hook(self, i, j):
        def hook(p):
            v = self.views[i][j]
            if p.grad is not v:  # autograd replaced the buffer view: fold it back in
                if p.grad.data_ptr() != v.data_ptr():
                    v.copy_(p.grad)
                p.grad = v
            self.pending[i] -= 1
            if self.pending[i] == 0:
                self._launch(i)
        return hook

    def _launch(self, i):
        if self.launched[i]:
            return
        self.launched[i] = True
        if self.world > 1 and not self.defer:
            op = dist.ReduceOp.AVG if self.avg else dist.ReduceOp.SUM
            try:
                self.works.append(dist.all_reduce(self.buffers[i], op=op, group=self.group, async_op=True))
            except Exception as e:  # raised from a backward hook: report it from finish()
                self.launch_error = e

    def zero(self):
        """Clear the buckets before a backward pass."""
        for buf in self.buffers:
            buf.zero_()
        for grp, views in zip(self.params, self.views):
            for p, v in zip(grp, views):
                p.grad = v
        self.pending = [len(g) for g in self.params]
        self.launched = [False] * len(self.params)
        self.works = []
        self.launch_error = None

    def finish(self, timeout_s: float | None = None):
        """Reduce the buckets no hook completed (parameters without a
        gradient this step), wait for every all-reduce, and turn sums into
        means where the backend cannot average. With `timeout_s`, an
        all-reduce that fails or does not complete in time aborts the process
        group and raises RankFailure. (NCCL's wait only orders the current
        stream behind the collective; its deadline is the process group's
        timeout, and the heartbeat catches ranks that left between steps.)"""
        for i in range(len(self.buffers)):
            self._launch(i)
        try:
            if self.launch_error is not None:
                raise self.launch_error
            for w in self.works:
                if timeout_s is None:
                    w.wait()
                else:
                    w.wait(timeout=datetime.timedelta(seconds=timeout_s))
        except Exception as e:
            self.works = []
            self.launch_error = None
            abort(self.group)
            raise RankFailure(f"gradient all-reduce failed: {e}") from e
        self.works = []
        if self.world > 1 and not self.avg:
            for buf in self.buffers:
                buf.div_(self.world)

    def reduce_all(self, timeout_s: float | None = None):
        """All-reduce every bucket now and wait, as finish() does: the
        exchange between the two graphs of a step recorded with deferred
        hooks."""
        self.launched = [False] * len(self.buffers)
        self.works = []
        self.launch_error = None
        self.finish(timeout_s)

    def global_norm(self) -> torch.Tensor:
        return torch.linalg.vector_norm(torch.stack([torch.linalg.vector_norm(b) for b in self.buffers]))


def newton_schulz(g: torch.Tensor, steps: int = 5, eps: float = 1e-7) -> torch.Tensor:
    """Approximate U V^T of each matrix of a [n, rows, cols] stack by the
    quintic iteration X <- a X + (b A + c A^2) X, A = X X^T, with
    (a, b, c) = (3.4445, -4.7750, 2.0315), in bf16 (Jordan et al., 2024)."""
    a, b, c = 3.4445, -4.7750, 2.0315
    x = g.to(torch.bfloat16)
    tall = x.shape[-2] > x.shape[-1]
    if tall:
        x = x.transpose(-2, -1)
    x = x / (torch.linalg.vector_norm(x.float(), dim=(-2, -1), keepdim=True) + eps).to(x.dtype)
    for _ in range(steps):
        m = x @ x.transpose(-2, -1)
        x = a * x + (b * m + c * (m @ m)) @ x
    if tall:
        x = x.transpose(-2, -1)
    return x


class Muon:
    """Momentum + Nesterov + Newton-Schulz orthogonalised updates for 2-D
    weights, scaled by sqrt(max(1, rows / cols)); matrices of one shape are
    orthogonalised together as a batch."""

    def __init__(self, params, lr: float = 0.02, beta: float = 0.95, ns_steps: int = 5):
        self.params = [p for p in params if p.requires_grad]
        self.lr, self.beta, self.ns_steps = lr, beta, ns_steps
        self.momentum = [torch.zeros_like(p) for p in self.params]
        self.by_shape = {}
        for i, p in enumerate(self.params):
            self.by_shape.setdefault(tuple(p.shape), []).append(i)

    @torch.no_grad()
    def step(self):
        for shape, idx in self.by_shape.items():
            ms = [self.momentum[i] for i in idx]
            gs = [self.params[i].grad for i in idx]
            torch._foreach_mul_(ms, self.beta)
            torch._foreach_add_(ms, gs)
            upd = torch.stack(torch._foreach_add(gs, ms, alpha=self.beta))  # Nesterov
            o = newton_schulz(upd, self.ns_steps)
            scale = -self.lr * math.sqrt(max(1.0, shape[0] / shape[1]))
            for k, i in enumerate(idx):
                self.params[i].add_(o[k].to(self.params[i].dtype), alpha=scale)


class TrainStep:
    """Forward, loss, backward with overlapped gradient all-reduce, clipping
    and the Muon / AdamW update, for one rank's shard of the batch."""

    def __init__(self, model, group=None, muon_lr: float = 0.02, adamw_lr: float = 3e-4,
                 weight_decay: float = 0.1, max_grad_norm: float = 1.0, bucket_bytes: int = 32 << 20,
                 autocast: bool = True, reduce: bool = True, heartbeat: Heartbeat | None = None,
                 allreduce_timeout_s: float | None = None, capturable: bool = False):
        self.model = model
        self.heartbeat = heartbeat
        self.allreduce_timeout_s = allreduce_timeout_s
        self.steps = 0
        self.buckets = GradBuckets(model.parameters(), group, bucket_bytes, reduce=reduce)
        # (start, end) CUDA events around finish() of each step while set: the
        # all-reduce time the backward did not hide
        self.finish_events = None
        mats = [p for p in model.parameters() if p.requires_grad and p.ndim == 2]
        rest = [p for p in model.parameters() if p.requires_grad and p.ndim != 2]
        dev = next(model.parameters()).device
        self.muon = Muon(mats, lr=muon_lr)
        # capturable: the optimizer's step counters stay on the device, so the
        # whole step can be replayed from a CUDA graph (capture())
        self.adamw = torch.optim.AdamW(rest, lr=adamw_lr, betas=(0.9, 0.95), eps=1e-8,
                                       weight_decay=weight_decay, fused=dev.type == "cuda",
                                       capturable=capturable and dev.type == "cuda")
        self.capturable = capturable
        self.max_grad_norm = max_grad_norm
        self.autocast = autocast and dev.type == "cuda"
        self.graph = None
        self.graph_update = None
        self.graph_loss = None

    def __call__(self, cells, masks, col_table, cat_table) -> torch.Tensor:
        if self.heartbeat is not None:  # every rank is here before any collective of this step
            self.heartbeat.step(self.steps)
        self.steps += 1
        return self._step(cells, masks, col_table, cat_table)

    def capture(self, cells, col_table, cat_table, kinds, warmup: int = 3, split: bool | None = None) -> None:
        """Record the step as CUDA graphs, after ``warmup`` eager steps on a
        side stream (which also create the optimizer state). Every replay()
        then reads ``cells`` in place: copy each new batch into those tensors
        first. Needs capturable=True.

        One GPU: one graph holds the whole step -- the tile plans of ``kinds``
        built from ``cells``, forward, loss, backward, clipping and both
        optimizer updates. Several GPUs (or ``split``): the gradient
        all-reduce stays outside, so the step is two graphs -- plans, forward,
        loss and backward into the buckets, then clipping and the updates --
        with reduce_all() between them on the host (the exchange no longer
        overlaps the backward, in exchange for no per-kernel launch cost)."""
        if not self.capturable:
            raise ValueError("TrainStep(capturable=True) is needed for capture()")
        if split is None:
            split = self.buckets.world > 1
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self._step(cells, build_masks(cells, kinds), col_table, cat_table)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        if not split:
            with torch.cuda.graph(graph):
                loss = self._step(cells, build_masks(cells, kinds), col_table, cat_table)
            self.graph, self.graph_update, self.graph_loss = graph, None, loss
            return
        self.buckets.defer = True
        try:
            with torch.cuda.graph(graph):
                loss = self._forward_backward(cells, build_masks(cells, kinds), col_table, cat_table)
        finally:
            self.buckets.defer = False
        update = torch.cuda.CUDAGraph()
        with torch.cuda.graph(update, pool=graph.pool()):
            self._update()
        self.graph, self.graph_update, self.graph_loss = graph, update, loss

    def replay(self) -> torch.Tensor:
        """One captured step on the current contents of the captured cells;
        returns the (static) loss tensor, valid until the next replay."""
        if self.graph is None:
            raise RuntimeError("capture() first")
        if self.heartbeat is not None:
            self.heartbeat.step(self.steps)
        self.steps += 1
        self.graph.replay()
        if self.graph_update is not None:
            if self.finish_events is not None:
                ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                ev[0].record()
                self.buckets.reduce_all(self.allreduce_timeout_s)
                ev[1].record()
                self.finish_events.append(ev)
            else:
                self.buckets.reduce_all(self.allreduce_timeout_s)
            self.graph_update.replay()
        return self.graph_loss

    def _forward_backward(self, cells, masks, col_table, cat_table) -> torch.Tensor:
        self.buckets.zero()
        with torch.autocast("cuda", dtype=torch.bfloat16, enabled=self.autocast):
            out = self.model(cells, masks, col_table, cat_table)
            loss = self.model.loss(out, cells, cat_table)
        loss.backward()
        return loss.detach()

    def _update(self) -> None:
        norm = self.buckets.global_norm()
        clip = torch.clamp(self.max_grad_norm / (norm + 1e-6), max=1.0)
        torch._foreach_mul_(self.buckets.buffers, clip)
        self.muon.step()
        self.adamw.step()

    def _step(self, cells, masks, col_table, cat_table) -> torch.Tensor:
        loss = self._forward_backward(cells, masks, col_table, cat_table)
        if self.finish_events is not None:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record()
            self.buckets.finish(self.allreduce_timeout_s)
            ev[1].record()
            self.finish_events.append(ev)
        else:
            self.buckets.finish(self.allreduce_timeout_s)
        self._update()
        return loss


def build_masks(meta: dict, kinds, max_rows: int | None = None):
    """Per sublayer kind: (int16 cell order, tile plan), on the device of
    ``meta`` (batch.make_cells arrays moved to the GPU). The plans are rebuilt
    for every batch, as build_attention_masks is inside the reference's jitted
    step (model.py:299-313). The column kind's order is sorted on the GPU; the
    feature / neighbor orders (reverse Cuthill-McKee, sequential per sample)
    come with the batch."""
    from . import attention as rt
    from .batch import MASK_COLUMN, MASK_FEATURE, MASK_NEIGHBOR
    from .tokens import _order16
    key = {MASK_FEATURE: "out_perm", MASK_NEIGHBOR: "in_perm"}
    out = []
    for kind in kinds:
        if kind == MASK_COLUMN:  # sorted on the GPU from the batch's own tensors
            order = rt.column_order(meta["column_ids"], meta["is_padding"])
        elif kind in key:
            order = _order16(meta[key[kind]])
        else:
            b, s = meta["seq_row_ids"].shape
            order = torch.arange(s, device=meta["seq_row_ids"].device, dtype=torch.int32).to(torch.int16)
            order = order.expand(b, s).contiguous()
        plan = rt.build_tile_plan(order, meta["seq_row_ids"], meta["column_ids"], meta["is_padding"],
                                  meta["fk_adj"], kind, max_rows=max_rows)
        out.append((order, plan))
    return out

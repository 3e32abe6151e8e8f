"""Benchmark: RT masked attention fwd+bwd on B200 (cells/s, live-tile TFLOP/s).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c|b] [--impl ours|reference]

One step = for each mask kind (column, feature, neighbor, full): the
tile-plan prepass from the batch's token metadata, the forward and the
backward attention kernels, all through the library's C ABI. Inputs (token
metadata and q/k/v/dO for every kind, > 1 GB for the default workload) are
resident in HBM, larger than L2, and distinct per kind. Under torchrun each
rank runs the same workload on its own batch (weak scaling, no collective in
the data path); the time is the max over ranks.

``--impl reference`` times the CPU restatement of the reference math
(numpy fp32 dense masked attention + analytic backward, multithreaded BLAS)
on a bounded sample of the same workload on rank 0.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

KIND_NAMES = ("column", "feature", "neighbor", "full")

# Workloads (benchmark configurations of the RT attention path)
CONFIGS = {
    # B=8, S=4096, 16 heads x 64; generator tuned for a spread of tile densities
    "c": dict(name="rt_attn_fwd_bwd_b8_s4096_h16_d64", B=8, S=4096, H=16, Dh=64,
              tables=24, cells_lo=4, cells_hi=16, p_fk=0.9, max_parents=2, pad=0.05),
    # B=32, S=1024, 8 heads x 32; 6 tables, 4-16 cells, p_fk 0.7, 10% padding
    "b": dict(name="rt_attn_fwd_bwd_b32_s1024_h8_d32", B=32, S=1024, H=8, Dh=32,
              tables=6, cells_lo=4, cells_hi=16, p_fk=0.7, max_parents=1, pad=0.10),
    # full encoder training step, data-parallel: 12 layers, d_model 512, 8 heads x 64,
    # each layer column -> feature -> neighbor -> full attention + SwiGLU FFN; per-GPU B=32, S=1024
    "d": dict(name="rt_encoder_train_b32_s1024_l12_d512_h8x64", train=True, B=32, S=1024, H=8, Dh=64,
              d_model=512, d_ff=1536, layers=12, d_text=384, d_time=8, n_categories=4096,
              tables=6, cells_lo=4, cells_hi=16, p_fk=0.7, max_parents=1, pad=0.10),
}

FLOPS_PER_LIVE_TILE = {"fwd": 4, "bwd": 10}  # x 128^2 x Dh per live (b, h, tile pair)

# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one dkdvq_kernel
# launch -- the fused dK/dV/dQ backward, the dominant kernel -- from an ncu
# capture of the full-mask launch at B = 4 (301.9 MB, summarised under
# profiles/) scaled by 2 to this workload's B = 8 launch: q, k, v, dO and the
# row statistics read once, dK and dV written once, plus the fp32 dQ
# accumulator's L2 misses under the reduce-adds.
NCU_DKDVQ_TRAFFIC = {"rt_attn_fwd_bwd_b8_s4096_h16_d64": 603.8e6}


def measured_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 1590.0, 6650.0, "fallback"


def make_metadata(cfg, seed):
    """Seeded synthetic token metadata and the sampler's cell orderings."""
    from tributary_b200 import batch as rb
    return rb.make_batch(seed, cfg["B"], cfg["S"], cfg["tables"], cfg["cells_lo"], cfg["cells_hi"],
                         cfg["p_fk"], cfg["pad"], max_parents=cfg["max_parents"])


def perm_for(bt, kind):
    from tributary_b200 import batch as rb
    return rb.order_for_kind(bt, kind)


# ----------------------------------------------------------------------------
# clocks sampling (nvidia-smi during the timed region)
# ----------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.device_index = device_index
        self.proc = None
        self.path = os.path.join("/tmp", f"rt_bench_clocks_{os.getpid()}.csv")

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device_index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    smax = float(parts[2])
                except ValueError:
                    continue
                for name, val in zip(names, parts[5:9]):
                    if val.lower().startswith("active"):
                        reasons.add(name)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------
# our arm
# ----------------------------------------------------------------------------
class Workload:
    """Device-resident inputs, plans and outputs for one rank."""

    def __init__(self, cfg, seed, device):
        import torch
        from tributary_b200 import attention as rt
        self.cfg = cfg
        self.rt = rt
        self.torch = torch
        B, S, H, Dh = cfg["B"], cfg["S"], cfg["H"], cfg["Dh"]
        bt = make_metadata(cfg, seed)
        self.meta_host = bt
        g = torch.Generator(device="cpu").manual_seed(seed)
        self.kinds = []
        for kind in range(4):
            perm = torch.from_numpy(np.ascontiguousarray(perm_for(bt, kind)).view(np.int16))
            host = {
                "perm": perm,
                "seq_row_ids": torch.from_numpy(bt["seq_row_ids"].view(np.int16)),
                "column_ids": torch.from_numpy(bt["column_ids"]),
                "is_padding": torch.from_numpy(bt["is_padding"]),
                "fk_adj": torch.from_numpy(bt["fk_adj"]),
            }
            # q_hat, k_hat unit vectors (tau = sqrt(Dh) folded into q), v, dO ~ N(0,1)
            q = torch.randn(B, H, S, Dh, generator=g)
            k = torch.randn(B, H, S, Dh, generator=g)
            q = q / q.norm(dim=-1, keepdim=True) * math.sqrt(Dh)
            k = k / k.norm(dim=-1, keepdim=True)
            v = torch.randn(B, H, S, Dh, generator=g)
            do = torch.randn(B, H, S, Dh, generator=g)
            for name, t in (("q", q), ("k", k), ("v", v), ("do", do)):
                host[name] = t.to(torch.bfloat16)
            dev = {n: t.to(device) for n, t in host.items()}
            plan = rt.build_tile_plan(dev["perm"], dev["seq_row_ids"], dev["column_ids"],
                                      dev["is_padding"], dev["fk_adj"], kind)
            o = torch.empty_like(dev["q"])
            lse = torch.empty(B, H, S, dtype=torch.float32, device=device)
            grads = [torch.empty_like(dev["q"]) for _ in range(3)]
            ws = torch.empty(rt._lib.load().rt_attention_bwd_workspace_bytes(B, H, S),
                             dtype=torch.uint8, device=device)
            pinned = {n: t.pin_memory() for n, t in host.items()}
            out_pinned = [torch.empty_like(host["q"]).pin_memory() for _ in range(4)]
            self.kinds.append(dict(kind=kind, dev=dev, plan=plan, o=o, lse=lse, grads=grads, ws=ws,
                                   pinned=pinned, out_pinned=out_pinned))
        torch.cuda.synchronize()
        self.nnz = [k["plan"].nnz() for k in self.kinds]
        self.tiles = self.kinds[0]["plan"].tiles

    def launches_per_step(self):
        # prepass: set-up (perm check, fk packing), tile mask, tile list;
        # forward: one kernel; backward: row stats, dK/dV/dQ, dQ conversion
        return sum(3 + 1 + 3 for _ in range(4))

    def rebuild_plan(self, k):
        lib = self.rt._lib
        d = k["dev"]
        B, S = self.cfg["B"], self.cfg["S"]
        R = d["fk_adj"].shape[1]
        lib.check(lib.load().rt_build_tile_plan(
            d["perm"].data_ptr(), d["seq_row_ids"].data_ptr(), d["column_ids"].data_ptr(),
            d["is_padding"].data_ptr(), d["fk_adj"].data_ptr(), B, S, R, k["kind"],
            self.rt.ctypes.byref(k["plan"].c), self.torch.cuda.current_stream().cuda_stream),
            "rt_build_tile_plan")

    def step(self, events=None):
        rt = self.rt
        scale = 1.0 / math.sqrt(self.cfg["Dh"])
        for k in self.kinds:
            d = k["dev"]
            if events is not None:
                events["plan"][0].record()
            self.rebuild_plan(k)
            if events is not None:
                events["plan"][1].record()
                events["fwd"][0].record()
            rt.attention_fwd(d["q"], d["k"], d["v"], k["plan"], scale, out=k["o"], lse=k["lse"])
            if events is not None:
                events["fwd"][1].record()
                events["bwd"][0].record()
            rt.attention_bwd(d["q"], d["k"], d["v"], k["o"], k["lse"], d["do"], k["plan"], scale,
                             dq=k["grads"][0], dk=k["grads"][1], dv=k["grads"][2], workspace=k["ws"])
            if events is not None:
                events["bwd"][1].record()
                for name in ("plan", "fwd", "bwd"):
                    events["acc"][name].append((events[name][0], events[name][1]))
                    events["by_kind"].setdefault((k["kind"], name), []).append(
                        (events[name][0], events[name][1]))
                    events[name] = (self.torch.cuda.Event(enable_timing=True),
                                    self.torch.cuda.Event(enable_timing=True))

    def step_e2e(self):
        """Same pass through the public API with host buffers: pinned host ->
        device copies of every input, then o, dq, dk, dv back to the host."""
        rt = self.rt
        scale = 1.0 / math.sqrt(self.cfg["Dh"])
        h2d = d2h = 0
        for k in self.kinds:
            d, p = k["dev"], k["pinned"]
            for n in ("perm", "seq_row_ids", "column_ids", "is_padding", "fk_adj", "q", "k", "v", "do"):
                d[n].copy_(p[n], non_blocking=True)
                h2d += p[n].numel() * p[n].element_size()
            self.rebuild_plan(k)
            rt.attention_fwd(d["q"], d["k"], d["v"], k["plan"], scale, out=k["o"], lse=k["lse"])
            rt.attention_bwd(d["q"], d["k"], d["v"], k["o"], k["lse"], d["do"], k["plan"], scale,
                             dq=k["grads"][0], dk=k["grads"][1], dv=k["grads"][2], workspace=k["ws"])
            for dst, src in zip(k["out_pinned"], [k["o"]] + k["grads"]):
                dst.copy_(src, non_blocking=True)
                d2h += src.numel() * src.element_size()
        return h2d, d2h

    def step_e2e_pipelined(self, streams, events):
        """step_e2e with the copies overlapped: per kind, the inputs go up on
        streams[0], the plan + forward + backward run on streams[1] and the
        outputs come down on streams[2] (PCIe is full duplex), ordered by
        events; a kind's inputs are not overwritten before the previous step's
        compute on them is done, nor its outputs before they were read back."""
        torch = self.torch
        rt = self.rt
        s_in, s_comp, s_out = streams
        scale = 1.0 / math.sqrt(self.cfg["Dh"])
        h2d = d2h = 0
        for i, k in enumerate(self.kinds):
            d, p = k["dev"], k["pinned"]
            ev = events[i]
            with torch.cuda.stream(s_in):
                if ev["comp"] is not None:
                    s_in.wait_event(ev["comp"])  # previous step's compute read these inputs
                for n in ("perm", "seq_row_ids", "column_ids", "is_padding", "fk_adj", "q", "k", "v", "do"):
                    d[n].copy_(p[n], non_blocking=True)
                    h2d += p[n].numel() * p[n].element_size()
                ev["in"] = torch.cuda.Event()
                ev["in"].record(s_in)
            with torch.cuda.stream(s_comp):
                s_comp.wait_event(ev["in"])
                if ev["out"] is not None:
                    s_comp.wait_event(ev["out"])  # previous step's outputs have been read back
                self.rebuild_plan(k)
                rt.attention_fwd(d["q"], d["k"], d["v"], k["plan"], scale, out=k["o"], lse=k["lse"])
                rt.attention_bwd(d["q"], d["k"], d["v"], k["o"], k["lse"], d["do"], k["plan"], scale,
                                 dq=k["grads"][0], dk=k["grads"][1], dv=k["grads"][2], workspace=k["ws"])
                ev["comp"] = torch.cuda.Event()
                ev["comp"].record(s_comp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev["comp"])
                for dst, src in zip(k["out_pinned"], [k["o"]] + k["grads"]):
                    dst.copy_(src, non_blocking=True)
                    d2h += src.numel() * src.element_size()
                ev["out"] = torch.cuda.Event()
                ev["out"].record(s_out)
        return h2d, d2h

    def live_tile_flops(self):
        """Algorithmic FLOPs of one step (fwd 4, bwd 10 x 128^2 x Dh per live tile-head)."""
        h, dh = self.cfg["H"], self.cfg["Dh"]
        per = {"fwd": 0, "bwd": 0}
        for nnz in self.nnz:
            for p in per:
                per[p] += FLOPS_PER_LIVE_TILE[p] * 128 * 128 * dh * h * nnz
        return per

    def algorithmic_bytes(self):
        b, s, h, dh = (self.cfg[x] for x in ("B", "S", "H", "Dh"))
        fwd = 8 * b * h * s * dh + 4 * b * h * s
        bwd = 16 * b * h * s * dh + 8 * b * h * s
        return {"fwd": 4 * fwd, "bwd": 4 * bwd}


# ----------------------------------------------------------------------------
# sub-records of the default line: the B=32, S=1024, Dh=32 workload and the
# sequence-length x density sweep (8 heads x 64)
# ----------------------------------------------------------------------------
SWEEP_S = (512, 1024, 2048, 4096, 8192)
SWEEP_TARGETS = (0.01, 0.05, 0.20, 0.50, 1.00)
SWEEP_TOKENS = 1 << 18  # B * S per point: q, k, v, dO are 256 MB each, above L2
# generator settings the sweep picks from (tables, cells_lo, cells_hi, p_fk,
# max_parents, parent_window), from sparse to dense live tiles; with the four
# mask kinds they span about 5-50% at S = 4096 (and 100%: full kind, no padding)
SWEEP_SETTINGS = (
    (96, 16, 32, 0.3, 1, 8),
    (96, 8, 24, 0.3, 1, 32),
    (24, 2, 6, 0.5, 2, 128),
    (24, 4, 16, 0.9, 2, None),
    (48, 1, 3, 0.9, 6, None),
    (96, 2, 6, 1.0, 6, None),
)


def _sweep_batch(seed, b, s, setting, pad):
    from tributary_b200 import batch as rb
    t, lo, hi, p, mp, win = setting
    return rb.make_batch(seed, b, s, t, lo, hi, p, pad, parent_window=win, max_parents=mp)


def _plan_for(bt, kind, device):
    import torch
    from tributary_b200 import attention as rt
    from tributary_b200 import batch as rb
    dev = {k: torch.from_numpy(np.ascontiguousarray(v).view(np.int16) if v.dtype == np.uint16 else
                               np.ascontiguousarray(v)).to(device)
           for k, v in bt.items() if k in ("seq_row_ids", "column_ids", "is_padding", "fk_adj")}
    perm = torch.from_numpy(np.ascontiguousarray(rb.order_for_kind(bt, kind)).view(np.int16)).to(device)
    return rt.build_tile_plan(perm, dev["seq_row_ids"], dev["column_ids"], dev["is_padding"], dev["fk_adj"],
                              kind), (perm, dev)


def sweep_choices(s, device):
    """(target, setting, kind, calibration density) per density target at
    sequence length s: the generator setting and mask kind whose live-tile
    density on a 2-sample calibration batch is nearest the target (log
    scale). The seed does not depend on the rank, so every rank picks alike."""
    cands = [(1.0, None, 3)]
    for setting in SWEEP_SETTINGS:
        bt = _sweep_batch(77, 2, s, setting, 0.05)
        for kind in (0, 1, 2):
            plan, _ = _plan_for(bt, kind, device)
            t = plan.tiles
            cands.append((plan.nnz() / (2 * t * t), setting, kind))
    out = []
    for target in SWEEP_TARGETS:
        d, setting, kind = min(cands, key=lambda c: abs(math.log(c[0] / target)))
        out.append((target, setting, kind, d))
    return out


def sweep_point(s, setting, kind, seed, device, world, steps=5, warmup=2, h=8, dh=64):
    """fwd + bwd of one mask kind at sequence length s on SWEEP_TOKENS cells,
    device-resident inputs; times are CUDA events, max over ranks."""
    import torch
    from tributary_b200 import attention as rt
    b = SWEEP_TOKENS // s
    bt = _sweep_batch(seed, b, s, setting if setting is not None else SWEEP_SETTINGS[0],
                      0.0 if kind == 3 else 0.05)
    plan, (perm, dev) = _plan_for(bt, kind, device)
    g = torch.Generator(device=device).manual_seed(seed)
    q = torch.randn(b, h, s, dh, device=device, generator=g)
    k = torch.randn(b, h, s, dh, device=device, generator=g)
    q = (q / q.norm(dim=-1, keepdim=True) * math.sqrt(dh)).to(torch.bfloat16)
    k = (k / k.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
    v = torch.randn(b, h, s, dh, device=device, generator=g).to(torch.bfloat16)
    do = torch.randn(b, h, s, dh, device=device, generator=g).to(torch.bfloat16)
    o, lse = torch.empty_like(q), torch.empty(b, h, s, dtype=torch.float32, device=device)
    grads = [torch.empty_like(q) for _ in range(3)]
    ws = torch.empty(rt._lib.load().rt_attention_bwd_workspace_bytes(b, h, s), dtype=torch.uint8, device=device)
    scale = 1.0 / math.sqrt(dh)

    def call():
        rt.attention_fwd(q, k, v, plan, scale, out=o, lse=lse)
        rt.attention_bwd(q, k, v, o, lse, do, plan, scale, dq=grads[0], dk=grads[1], dv=grads[2], workspace=ws)

    for _ in range(warmup):
        call()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        call()
    e1.record()
    barrier(world)
    ms = max_over_ranks(e0.elapsed_time(e1) / steps, world)
    nnz, t = plan.nnz(), plan.tiles
    tflops = 14 * 128 * 128 * dh * h * nnz / (ms * 1e-3) / 1e12
    return {"S": s, "B": b, "kind": KIND_NAMES[kind], "live_tile_density": nnz / (b * t * t),
            "ms_fwd_bwd": ms, "cells_per_s": world * b * s / (ms * 1e-3), "tflops_live_tiles": tflops}


def run_sweep(world, rank, device, peak_tf):
    import torch
    points = []
    for s in SWEEP_S:
        for target, setting, kind, _ in sweep_choices(s, device):
            rec = sweep_point(s, setting, kind, 2000 + rank, device, world)
            rec["target_density"] = target
            rec["generator"] = None if setting is None else dict(zip(
                ("tables", "cells_lo", "cells_hi", "p_fk", "max_parents", "parent_window"), setting))
            rec["frac_of_bf16_peak"] = rec["tflops_live_tiles"] / peak_tf
            points.append(rec)
            torch.cuda.empty_cache()
    return {"what": "fwd+bwd of one mask kind, H=8, Dh=64, B*S = %d cells per point (inputs > L2), "
                    "generator setting and kind chosen per point for the live-tile density nearest the "
                    "target (the diagonal tiles alone are 1/T, so 1%% is out of reach below S = 12800)"
                    % SWEEP_TOKENS,
            "points": points}


def measure_workload(cfg, seed, device, world, steps=5, warmup=3):
    """Device time of the attention step (prepass, fwd, bwd of the four kinds)
    on cfg's workload, with the per-kind breakdown; max over ranks."""
    import torch
    wl = Workload(cfg, seed=seed, device=device)
    for _ in range(warmup):
        wl.step()
    barrier(world)
    ev = {n: (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for n in ("plan", "fwd", "bwd")}
    ev["acc"] = {"plan": [], "fwd": [], "bwd": []}
    ev["by_kind"] = {}
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        wl.step(events=ev)
    e1.record()
    barrier(world)
    step_ms = max_over_ranks(e0.elapsed_time(e1) / steps, world)
    kind_ms = {KIND_NAMES[kk]: {n: max_over_ranks(sum(a.elapsed_time(b) for a, b in ev["by_kind"][(kk, n)]) / steps,
                                                  world) for n in ("plan", "fwd", "bwd")} for kk in range(4)}
    flops = wl.live_tile_flops()
    attn_ms = sum(v["fwd"] + v["bwd"] for v in kind_ms.values())
    tf = (flops["fwd"] + flops["bwd"]) / (attn_ms * 1e-3) / 1e12
    densities = {KIND_NAMES[i]: wl.nnz[i] / (cfg["B"] * wl.tiles * wl.tiles) for i in range(4)}
    rec = {"workload": cfg["name"], "B": cfg["B"], "S": cfg["S"], "H": cfg["H"], "Dh": cfg["Dh"],
           "ms_per_step": step_ms, "cells_per_s": world * 4 * cfg["B"] * cfg["S"] / (step_ms * 1e-3),
           "breakdown_ms_by_kind": kind_ms, "live_tile_density": densities, "tflops_live_tiles": tf}
    del wl
    torch.cuda.empty_cache()
    return rec


def dist_setup(n_gpus):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    import torch
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()


def oracle_sample_batch(cfg, seed):
    """Sample 0 of the workload's batch and its four cell orders, built by the
    oracle's numpy restatement of the generator and of the sampler's orders
    (the same draws as the library's generator, pinned equal by the tests), so
    that the CPU legs load nothing of the library."""
    from oracle import rt_oracle as orc  # CPU baseline leg
    return orc.make_batch(seed, 1, cfg["S"], cfg["tables"], cfg["cells_lo"], cfg["cells_hi"], cfg["p_fk"],
                          cfg["pad"], max_parents=cfg["max_parents"])


class CpuSample:
    """The numpy restatement of the reference math (fp32 dense masked
    attention, confluence/confluence/layers.py:83-97, plus its analytic
    backward) on a bounded sample of the workload: batch element 0 of the
    same seeded batch, `hs` of the H heads, every mask kind under its own cell
    order. One call = forward + backward of every kind and sampled head, the
    (kind, head) problems spread over all host cores (one BLAS thread each)."""

    def __init__(self, cfg, seed):
        from concurrent.futures import ThreadPoolExecutor
        from oracle import rt_oracle as orc  # CPU baseline leg
        self.orc = orc
        bt = oracle_sample_batch(cfg, seed)
        S, H, Dh = cfg["S"], cfg["H"], cfg["Dh"]
        self.S, self.H, self.B = S, H, cfg["B"]
        self.cores = len(os.sched_getaffinity(0))
        # enough (kind, head) problems to occupy every core once
        self.hs = min(H, max(2, -(-self.cores // 4)))
        rng = np.random.default_rng(seed)
        self.q, self.k, self.v, self.do = (rng.standard_normal((1, self.hs, S, Dh)).astype(np.float32)
                                           for _ in range(4))
        self.scale = np.float32(1.0 / math.sqrt(Dh))
        self.masks = []
        for kind in range(4):
            m = orc.mask_for_kind(kind, bt["seq_row_ids"], bt["fk_adj"], bt["column_ids"], bt["is_padding"])
            self.masks.append(orc.permute_mask(m, orc.perm_for_kind(bt, kind)))
        self.pool = ThreadPoolExecutor(max_workers=self.cores)

    def cells_per_call(self):
        # one attention call over all H heads counts S cells, per kind
        return 4 * self.S * self.hs / self.H

    def _one(self, kind_head):
        kind, h = kind_head
        sel = (slice(0, 1), slice(h, h + 1))
        q, k, v, do = self.q[sel], self.k[sel], self.v[sel], self.do[sel]
        o, _ = self.orc.attention_fwd(q, k, v, self.masks[kind], self.scale)
        self.orc.attention_bwd(q, k, v, o, do, self.masks[kind], self.scale)

    def call(self):
        from threadpoolctl import threadpool_limits
        with threadpool_limits(limits=1):
            list(self.pool.map(self._one, [(kd, h) for kd in range(4) for h in range(self.hs)]))

    def describe(self, calls):
        return (f"b=1 of {self.B}, {self.hs} of {self.H} heads, {calls} fwd+bwd calls of each of the 4 kinds; "
                f"numpy fp32 restatement of the reference path, (kind, head) problems on {self.cores} threads "
                f"(jax/XLA-CPU not installable)")


def cpu_sample(cfg, seed, budget_s=15.0):
    """(cells/s, sample description) of CpuSample over about budget_s seconds."""
    smp = CpuSample(cfg, seed)
    t0 = time.perf_counter()
    calls = 0
    while calls == 0 or time.perf_counter() - t0 < budget_s:
        smp.call()
        calls += 1
    dt = time.perf_counter() - t0
    return calls * smp.cells_per_call() / dt, smp.describe(calls)


def config_record(cfg, world):
    """The `config` object both arms print for the attention workload."""
    return {"workload": cfg["name"], "B": cfg["B"], "S": cfg["S"], "H": cfg["H"], "Dh": cfg["Dh"],
            "masks": list(KIND_NAMES),
            "generator": {k: cfg[k] for k in ("tables", "cells_lo", "cells_hi", "p_fk", "max_parents", "pad")},
            "l2": "inputs > L2 (q/k/v/dO distinct per kind, %.2f GB resident)" % (
                16 * cfg["B"] * cfg["H"] * cfg["S"] * cfg["Dh"] * 2 / 1e9),
            "parallelism": f"batch-sharded x{world}: attention with no collective; training step dp{world} "
                           f"with NCCL gradient all-reduce (train_step)"}


def run_reference_arm(args, cfg):
    """The reference's CPU path: the oracle port (the reference's JAX path on
    XLA-CPU cannot be installed here) on the host cores, rank 0 only. A step
    is one bounded sample of the workload (CpuSample.call); ms_per_step is the
    time a step actually took and value the sample's cells per second."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cores = len(os.sched_getaffinity(0))
    smp = CpuSample(cfg, 1000)
    for _ in range(args.warmup):
        smp.call()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        smp.call()
    dt = time.perf_counter() - t0
    value = args.steps * smp.cells_per_call() / dt
    line = {
        "impl": "reference", "metric": "rt_attention_fwd_bwd_cells_per_s", "value": value,
        "unit": "cells/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * dt / args.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": config_record(cfg, world),
        "sample": smp.describe(1) + " per step",
        "cpu_baseline": {"value": value, "unit": "cells/s", "cores": cores, "kind": "port",
                         "sample": smp.describe(args.steps)},
        "e2e": {"value": value, "unit": "cells/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_our_arm(args, cfg):
    import torch
    world, rank, local = dist_setup(args.gpus)
    wl = Workload(cfg, seed=1000 + rank, device=torch.device("cuda", local))
    from tributary_b200.attention import device_status

    for _ in range(args.warmup):
        wl.step()
    barrier(world)
    if device_status(reset=True) != 0:
        raise RuntimeError("device status error during warm-up")

    # ---- timed region: K steps, device time by events, max over ranks ----
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    barrier(world)
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record()
    for _ in range(args.steps):
        wl.step()
    t_end.record()
    barrier(world)
    step_ms = t_start.elapsed_time(t_end) / args.steps
    # per-entry-point breakdown over the same number of steps
    ev = {n: (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for n in ("plan", "fwd", "bwd")}
    ev["acc"] = {"plan": [], "fwd": [], "bwd": []}
    ev["by_kind"] = {}
    for _ in range(args.steps):
        wl.step(events=ev)
    barrier(world)
    clocks = sampler.stop()
    part_ms = {n: sum(a.elapsed_time(b) for a, b in ev["acc"][n]) / args.steps for n in ("plan", "fwd", "bwd")}
    kind_ms = {KIND_NAMES[kk]: {n: sum(a.elapsed_time(b) for a, b in ev["by_kind"][(kk, n)]) / args.steps
                                for n in ("plan", "fwd", "bwd")} for kk in range(4)}
    step_ms = max_over_ranks(step_ms, world)
    part_ms = {n: max_over_ranks(v, world) for n, v in part_ms.items()}

    # ---- end to end through the public API with host buffers ----
    # copies in and out overlap the compute of the neighbouring mask kinds
    cur = torch.cuda.current_stream()
    streams = [torch.cuda.Stream() for _ in range(3)]
    pipe_events = [{"in": None, "comp": None, "out": None} for _ in wl.kinds]
    for st in streams:
        st.wait_stream(cur)
    for _ in range(2):
        wl.step_e2e_pipelined(streams, pipe_events)
    for st in streams:
        cur.wait_stream(st)
    torch.cuda.synchronize()
    barrier(world)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(cur)
    for st in streams:
        st.wait_event(e0)
    for _ in range(args.steps):
        h2d, d2h = wl.step_e2e_pipelined(streams, pipe_events)
    for st in streams:
        cur.wait_stream(st)
    e1.record(cur)
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world)
    status = device_status(reset=True)
    if status != 0:
        raise RuntimeError(f"device status error {status}")

    cfgd = wl.cfg
    launches = wl.launches_per_step() * args.steps
    cells_step = 4 * cfgd["B"] * cfgd["S"]  # 4 attention calls (one per mask kind) per step
    value = world * cells_step / (step_ms * 1e-3)
    flops = wl.live_tile_flops()
    peak_tf, peak_gbs, peak_src = measured_peaks()
    attn_ms = part_ms["fwd"] + part_ms["bwd"]
    achieved_tf = (flops["fwd"] + flops["bwd"]) / (attn_ms * 1e-3) / 1e12
    bwd_tf = flops["bwd"] / (part_ms["bwd"] * 1e-3) / 1e12
    fwd_tf = flops["fwd"] / (part_ms["fwd"] * 1e-3) / 1e12
    densities = {KIND_NAMES[i]: wl.nnz[i] / (cfgd["B"] * wl.tiles * wl.tiles) for i in range(4)}
    del wl
    torch.cuda.empty_cache()
    sweep = config_b = None
    if not args.no_sweep:
        dev = torch.device("cuda", local)
        config_b = measure_workload(dict(CONFIGS["b"]), 1000 + rank, dev, world)
        config_b["frac_of_bf16_peak"] = config_b["tflops_live_tiles"] / peak_tf
        sweep = run_sweep(world, rank, dev, peak_tf)
    train = None
    if not args.no_train:
        train = measure_train(dict(CONFIGS["d"]), args.train_steps, 3, world, rank, local)
    if rank == 0:
        line = {
            "metric": "rt_attention_fwd_bwd_cells_per_s", "value": value, "unit": "cells/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": config_record(cfgd, world),
            "live_tile_density": densities,
            "tflops_live_tiles": achieved_tf,
            "frac_of_bf16_peak": achieved_tf / peak_tf,
            "breakdown_ms_per_step": part_ms,
            "breakdown_ms_by_kind": kind_ms,
            # dominant kernel: dkdvq_kernel, timed with CUDA events around each
            # rt_attention_bwd call (its row_stats and dq_convert launches are 7%
            # of that time); per-launch flops over the average launch time
            "roofline": {"bound": "tensor",
                         "kernel": "dkdvq_kernel (fused dK/dV/dQ backward), timed as rt_attention_bwd",
                         "achieved": bwd_tf, "peak": peak_tf, "unit": "TFLOP/s",
                         "frac": bwd_tf / peak_tf, "peak_source": peak_src + " bf16 dense (burst)",
                         "traffic": NCU_DKDVQ_TRAFFIC.get(cfgd["name"]),
                         "traffic_unit": "bytes per launch (ncu dram__bytes_read.sum + dram__bytes_write.sum)",
                         "algorithmic_flops_per_launch": flops["bwd"] / 4,
                         "forward": {"kernel": "attn_fwd_kernel", "achieved": fwd_tf, "frac": fwd_tf / peak_tf},
                         "fwd_plus_bwd": {"achieved": achieved_tf, "frac": achieved_tf / peak_tf}},
            "e2e": {"value": world * cells_step / (e2e_ms * 1e-3), "unit": "cells/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": launches,
            "clocks": clocks,
        }
        if config_b is not None:
            line["config_b"] = config_b
            line["sweep"] = sweep
        if train is not None:
            line["train_step"] = train
        if not args.no_cpu_baseline:
            v, sample = cpu_sample(cfgd, 1000, budget_s=args.cpu_seconds)
            line["cpu_baseline"] = {"value": v, "unit": "cells/s", "cores": len(os.sched_getaffinity(0)),
                                    "kind": "port", "sample": sample}
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


# ----------------------------------------------------------------------------
# full encoder training step (config d): data-parallel, NCCL gradient all-reduce
# ----------------------------------------------------------------------------
TRAIN_KINDS = (0, 1, 2, 3)
CELL_ARRAYS = ("seq_row_ids", "column_ids", "is_padding", "fk_adj", "out_perm", "in_perm", "stypes",
               "numeric_values", "timestamp_values", "bool_values", "categorical_ids", "text_ids", "text_vectors",
               "is_null", "is_target")


def make_train_cells(cfg, seed):
    from tributary_b200 import batch as rb
    return rb.make_cells(seed, cfg["B"], cfg["S"], cfg["tables"], cfg["cells_lo"], cfg["cells_hi"], cfg["p_fk"],
                         cfg["pad"], max_parents=cfg["max_parents"], d_text=cfg["d_text"], d_time=cfg["d_time"],
                         n_categories=cfg["n_categories"])


def encoder_config(cfg, layers=None):
    from tributary_b200.encoder import EncoderConfig
    return EncoderConfig(d_model=cfg["d_model"], n_heads=cfg["H"], d_head=cfg["Dh"], d_ff=cfg["d_ff"],
                         n_layers=layers or cfg["layers"], d_text=cfg["d_text"], d_time=cfg["d_time"],
                         kinds=TRAIN_KINDS)


def cells_to_host_tensors(cells):
    import torch
    out = {}
    for k in CELL_ARRAYS:
        a = cells[k].astype(np.int32) if cells[k].dtype == np.uint16 else cells[k]
        out[k] = torch.from_numpy(np.ascontiguousarray(a))
    return out


def train_flops(model, cfg, masks, tokens):
    """Algorithmic FLOPs of one training step on one rank: 6 x (Linear
    weights) x tokens for every matmul of the model (forward 2, backward 4),
    the categorical loss logits, and 14 x 128^2 x Dh per live (b, h, tile pair)
    of every attention sublayer (forward 4, backward 10)."""
    import torch.nn as nn
    lin = sum(m.in_features * m.out_features for m in model.modules() if isinstance(m, nn.Linear))
    lin_flops = 6 * lin * tokens
    logits = 6 * tokens * model.cfg.max_categories * cfg["d_model"]
    attn = 0
    for _, plan in masks:
        attn += 14 * 128 * 128 * cfg["Dh"] * cfg["H"] * plan.nnz()
    return lin_flops + logits + attn * cfg["layers"], attn * cfg["layers"]


class TrainRun:
    """The config-d training step on this rank's GPU: its own B=32 shard of
    cells, a replica with the same initial weights on every rank, and a
    TrainStep whose gradient buckets are all-reduced over NCCL (reduce=True)
    or kept local (reduce=False, the single-GPU step on the same device).
    graph=True records the step as CUDA graphs and replays them (one graph on
    one GPU; with an all-reduce, two graphs with the exchange between them):
    the cells are static tensors that a new batch is copied into."""

    def __init__(self, cfg, rank, dev, reduce=True, graph=False):
        import torch
        from tributary_b200.encoder import RTEncoder
        from tributary_b200.train import TrainStep
        self.cfg = cfg
        cells = make_train_cells(cfg, 1000 + rank)
        self.host = {k: v.pin_memory() for k, v in cells_to_host_tensors(cells).items()}
        self.d = {k: v.to(dev) for k, v in self.host.items()}
        for k in ("target_stype", "cat_start"):
            self.d[k] = cells[k]
        self.col = torch.from_numpy(cells["col_table"]).to(dev)
        self.cat = torch.from_numpy(cells["cat_table"]).to(dev)
        torch.manual_seed(1234)  # identical initial weights on every rank
        self.model = RTEncoder(encoder_config(cfg)).to(dev)
        self.step = TrainStep(self.model, reduce=reduce, capturable=graph)
        if graph:
            self.step.capture(self.d, self.col, self.cat, TRAIN_KINDS)

    def __call__(self):
        from tributary_b200.train import build_masks
        if self.step.graph is not None:
            return self.step.replay()
        return self.step(self.d, build_masks(self.d, TRAIN_KINDS), self.col, self.cat)

    def timed(self, steps, world, finish_events=False):
        """Device ms per step over `steps` steps (max over ranks) and, with
        finish_events, the mean exposed all-reduce ms (max over ranks)."""
        import torch
        barrier(world)
        self.step.finish_events = [] if finish_events else None
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            loss = self()
        e1.record()
        barrier(world)
        ms = max_over_ranks(e0.elapsed_time(e1) / steps, world)
        exposed = None
        if finish_events:
            exposed = max_over_ranks(sum(a.elapsed_time(b) for a, b in self.step.finish_events) / steps, world)
            self.step.finish_events = None
        return ms, exposed, loss

    def checksum_spread(self, world):
        """Relative spread over ranks of the sum of all parameters: 0 when the
        replicas stayed identical (same weights, same averaged gradients)."""
        import torch
        with torch.no_grad():
            chk = torch.stack([p.double().sum() for p in self.model.parameters()]).sum().reshape(1)
        if world == 1:
            return 0.0
        import torch.distributed as dist
        allc = [torch.zeros_like(chk) for _ in range(world)]
        dist.all_gather(allc, chk)
        vals = torch.cat(allc)
        return float((vals.max() - vals.min()).abs() / vals.abs().max().clamp_min(1e-30))


def measure_train(cfg, steps, warmup, world, rank, local):
    """The data-parallel training step (config d) at this world size: ms per
    step with the overlapped NCCL gradient all-reduce, the all-reduce time the
    backward does not hide, and the same step without the collective on the
    same GPUs (its ratio to the data-parallel step is the weak-scaling
    efficiency against one GPU). Every rank calls it (collectives inside)."""
    import torch
    from tributary_b200.attention import device_status
    dev = torch.device("cuda", local)
    run = TrainRun(cfg, rank, dev, reduce=True)
    for _ in range(warmup):
        run()
    dp_ms, exposed_ms, loss = run.timed(steps, world, finish_events=True)
    spread = run.checksum_spread(world)
    loss_val = float(loss.item())
    grad_bytes = sum(run.step.buckets.bucket_sizes)
    n_buckets = len(run.step.buckets.buffers)
    del run
    torch.cuda.empty_cache()
    solo = TrainRun(cfg, rank, dev, reduce=False)
    for _ in range(warmup):
        solo()
    solo_ms, _, _ = solo.timed(steps, world)
    del solo
    torch.cuda.empty_cache()
    # the same data-parallel step replayed from CUDA graphs (one graph on one
    # GPU; two around the all-reduce on several)
    gr = TrainRun(cfg, rank, dev, reduce=True, graph=True)
    for _ in range(warmup):
        gr()
    graph_ms, graph_exposed_ms, _ = gr.timed(steps, world, finish_events=world > 1)
    del gr
    torch.cuda.empty_cache()
    status = device_status(reset=True)
    if status != 0 or not math.isfinite(loss_val):
        raise RuntimeError(f"training step: device status {status}, loss {loss_val}")
    tokens = cfg["B"] * cfg["S"]
    return {"workload": cfg["name"], "n_gpus": world, "B_per_gpu": cfg["B"], "S": cfg["S"], "steps": steps,
            "ms_per_step": dp_ms, "tokens_per_s": world * tokens / (dp_ms * 1e-3),
            "allreduce": {"what": f"NCCL all-reduce (average) of {grad_bytes / 1e6:.0f} MB fp32 gradients "
                                  f"in {n_buckets} buckets, launched from post-accumulate hooks during backward",
                          "exposed_ms_per_step": exposed_ms},
            "ms_per_step_without_allreduce": solo_ms,
            "cuda_graph": {"ms_per_step": graph_ms, "tokens_per_s": world * tokens / (graph_ms * 1e-3),
                           "allreduce_exposed_ms_per_step": graph_exposed_ms,
                           "graphs": 1 if world == 1 else 2},
            "efficiency_vs_1gpu": solo_ms / dp_ms,
            "replica_param_checksum_rel_spread": spread, "final_loss": loss_val}


def run_train_arm(args, cfg):
    import torch
    from tributary_b200.attention import device_status
    from tributary_b200.train import build_masks
    world, rank, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    graph = not args.no_graph  # the step replays from CUDA graphs (two around the all-reduce on N > 1)
    run = TrainRun(cfg, rank, dev, graph=graph)
    for _ in range(args.warmup):
        run()
    barrier(world)
    if device_status(reset=True) != 0:
        raise RuntimeError("device status error during warm-up")
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    step_ms, exposed_ms, loss = run.timed(args.steps, world, finish_events=not graph or world > 1)
    clocks = sampler.stop()
    # end to end: every step copies its cell arrays from pinned host memory and reads the loss back
    h2d = sum(v.numel() * v.element_size() for v in run.host.values())
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        for k, v in run.host.items():
            run.d[k].copy_(v, non_blocking=True)
        loss_val = run().item()
    e1.record()
    barrier(world)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world)
    status = device_status(reset=True)
    if status != 0 or not math.isfinite(loss_val):
        raise RuntimeError(f"device status {status}, loss {loss_val}")
    tokens = cfg["B"] * cfg["S"]
    flops, attn_flops = train_flops(run.model, cfg, build_masks(run.d, TRAIN_KINDS), tokens)
    drift = run.checksum_spread(world)
    peak_tf, _, peak_src = measured_peaks()
    achieved = flops / (step_ms * 1e-3) / 1e12
    n_params = sum(p.numel() for p in run.model.parameters())
    if rank == 0:
        line = {
            "metric": "rt_encoder_train_tokens_per_s", "value": world * tokens / (step_ms * 1e-3), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": cfg["name"], "B_per_gpu": cfg["B"], "global_batch": world * cfg["B"],
                       "S": cfg["S"], "layers": cfg["layers"], "d_model": cfg["d_model"], "heads": cfg["H"],
                       "Dh": cfg["Dh"], "params": n_params, "masks_per_layer": [KIND_NAMES[k] for k in TRAIN_KINDS],
                       "optimizer": "muon (2-D weights) + adamw, global-norm clip 1.0",
                       "l2": "working set (activations of 48 sublayers) far above L2",
                       "parallelism": (f"dp{world}: NCCL all-reduce (average) of fp32 gradients in "
                                       f"{len(run.step.buckets.buffers)} buckets, "
                                       + ("between the backward and update graphs" if graph
                                          else "overlapped with backward"))
                                      if world > 1 else "dp1: one GPU, no collective",
                       "cuda_graph": graph},
            "allreduce_exposed_ms_per_step": exposed_ms,
            "roofline": {"bound": "tensor", "kernel": "whole training step (matmuls + attention)",
                         "achieved": achieved, "peak": peak_tf, "unit": "TFLOP/s", "frac": achieved / peak_tf,
                         "peak_source": peak_src + " bf16 dense (burst)", "traffic": None,
                         "attention_share_of_flops": attn_flops / flops},
            "e2e": {"value": world * tokens / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": 4},
            "gpu_launches": args.steps * (10 + cfg["layers"] * len(TRAIN_KINDS) * 5),
            "clocks": clocks,
            "final_loss": loss_val,
            "replica_param_checksum_rel_spread": drift,
        }
        if not args.no_cpu_baseline:
            v, sample, _ = train_cpu_sample(cfg, args.cpu_seconds)
            line["cpu_baseline"] = {"value": v, "unit": "tokens/s", "cores": len(os.sched_getaffinity(0)),
                                    "kind": "port", "sample": sample}
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


class _CpuOps:
    """The sublayer's gather, QK normalisation, dense masked attention and
    scatter, and the layer's norms, gated residual and SwiGLU activation, in
    plain torch with the reference's semantics (layers.py:16-30, 63-97,
    139-174, 177-200), for the CPU baseline."""

    @staticmethod
    def qk_prepare(qkv, order, tau, heads, head_dim):
        import torch
        b, s, w = qkv.shape
        x = torch.gather(qkv, 1, order[:, :, None].expand(b, s, w)).view(b, s, 3, heads, head_dim)
        x = x.permute(2, 0, 3, 1, 4)
        q = x[0] / x[0].norm(dim=-1, keepdim=True).clamp_min(1e-6) * tau.view(1, heads, 1, 1)
        k = x[1] / x[1].norm(dim=-1, keepdim=True).clamp_min(1e-6)
        return q, k, x[2]

    @staticmethod
    def attention(q, k, v, mask, scale):
        import torch
        s = torch.einsum("bhid,bhjd->bhij", q, k) * scale
        s = torch.where(mask[:, None], s, torch.full_like(s, -1e9))
        return torch.einsum("bhij,bhjd->bhid", torch.softmax(s, -1), v)

    @staticmethod
    def heads_unpermute(o, order):
        import torch
        b, h, s, dh = o.shape
        o = o.permute(0, 2, 1, 3).reshape(b, s, h * dh)
        inv = torch.empty_like(order).scatter_(1, order, torch.arange(s).expand_as(order))
        return torch.gather(o, 1, inv[:, :, None].expand(b, s, h * dh))

    @staticmethod
    def rms_norm(x, gamma, eps):
        import torch.nn.functional as F
        return F.rms_norm(x.float(), (x.shape[-1],), 1.0 + gamma, eps)

    @staticmethod
    def gate_residual(x, out, gate, scale):
        import torch
        return x + (out * scale * torch.sigmoid(gate)).float()

    @staticmethod
    def swiglu(u):
        import torch.nn.functional as F
        f = u.shape[-1] // 2
        return F.silu(u[..., :f]) * u[..., f:]

    @staticmethod
    def residual_add(x, h, scale):
        return x + (h * scale).float()


def train_cpu_sample(cfg, budget_s):
    """The same training step on the host cores: the encoder in fp32 with the
    reference's dense masked attention (layers.py:83-97) under the oracle's
    masks, one sample of the batch, for about budget_s seconds."""
    import torch
    from oracle import rt_oracle as orc  # CPU baseline leg
    from tributary_b200.encoder import RTEncoder
    from tributary_b200.train import TrainStep
    one = dict(cfg, B=1)
    cells = make_train_cells(one, 4321)
    c = cells_to_host_tensors(cells)
    for k in ("target_stype", "cat_start"):
        c[k] = cells[k]
    col = torch.from_numpy(cells["col_table"])
    cat = torch.from_numpy(cells["cat_table"])
    masks = []
    for kind in TRAIN_KINDS:
        from tributary_b200 import batch as rb
        perm = rb.order_for_kind(cells, kind)
        m = orc.permute_mask(orc.mask_for_kind(kind, cells["seq_row_ids"], cells["fk_adj"], cells["column_ids"],
                                               cells["is_padding"]), perm)
        masks.append((torch.from_numpy(perm.astype(np.int64)), torch.from_numpy(m)))
    torch.manual_seed(1234)
    model = RTEncoder(encoder_config(one), ops=_CpuOps())
    step = TrainStep(model, autocast=False)
    t0 = time.perf_counter()
    n = 0
    while n == 0 or time.perf_counter() - t0 < budget_s:
        step(c, masks, col, cat)
        n += 1
    dt = time.perf_counter() - t0
    return n * cfg["S"] / dt, (f"{n} fp32 training steps of the full {cfg['layers']}-layer encoder on 1 sample "
                               f"(S={cfg['S']}), dense masked attention, torch CPU, {torch.get_num_threads()} threads"), dt


def run_train_reference_arm(args, cfg):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    values, times, sample = [], [], ""
    per_step = max(5.0, min(30.0, 150.0 / max(1, args.steps)))
    train_cpu_sample(cfg, 1.0)
    for _ in range(args.steps):
        v, sample, dt = train_cpu_sample(cfg, per_step)
        values.append(v)
        times.append(dt)
    value = statistics.median(values)
    line = {
        "impl": "reference", "metric": "rt_encoder_train_tokens_per_s", "value": value, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        # a step is one bounded sample (whole training steps on one sample of the
        # batch); ms_per_step is the time that sample took, not an extrapolation
        "ms_per_step": 1e3 * statistics.median(times), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": cfg["name"], "B_per_gpu": cfg["B"], "S": cfg["S"], "layers": cfg["layers"]},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": len(os.sched_getaffinity(0)), "kind": "port",
                         "sample": sample + " (jax/XLA-CPU not installable)"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_plan_only(args, cfg):
    """The prepass alone on one GPU: each kind's tile plan rebuilt from the
    workload's device batch, mean CUDA-event time per call (not a bench line)."""
    import torch
    dev = torch.device("cuda", 0)
    wl = Workload(cfg, 1000, dev)
    for _ in range(args.warmup):
        for k in wl.kinds:
            wl.rebuild_plan(k)
    out = {}
    for k in wl.kinds:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            wl.rebuild_plan(k)
        e1.record()
        torch.cuda.synchronize()
        out[KIND_NAMES[k["kind"]]] = e0.elapsed_time(e1) / args.steps * 1000
    print(json.dumps({"workload": cfg["name"], "prepass_us_per_call": out}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="c", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-train", action="store_true",
                    help="attention workloads: skip the data-parallel training-step record")
    ap.add_argument("--no-sweep", action="store_true",
                    help="attention workloads: skip the B=32 S=1024 record and the length x density sweep")
    ap.add_argument("--no-graph", action="store_true",
                    help="--config d: run the step eagerly instead of replaying CUDA graphs")
    ap.add_argument("--train-steps", type=int, default=10,
                    help="timed steps of the training-step record")
    ap.add_argument("--batch", type=int, default=None,
                    help="override the workload's batch size (profiling runs)")
    ap.add_argument("--plan-only", action="store_true",
                    help="attention workloads, one GPU: only the prepass (rt_build_tile_plan of each kind, "
                         "--steps times after --warmup), CUDA-event time per kind; for profiling runs")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    cfg = dict(CONFIGS[args.config])
    if args.batch is not None:
        cfg["B"] = args.batch
        cfg["name"] = cfg["name"].replace("_b%d_" % CONFIGS[args.config]["B"], "_b%d_" % args.batch)
    if cfg.get("train"):
        (run_train_reference_arm if args.impl == "reference" else run_train_arm)(args, cfg)
    elif args.plan_only:
        run_plan_only(args, cfg)
    elif args.impl == "reference":
        run_reference_arm(args, cfg)
    else:
        run_our_arm(args, cfg)


if __name__ == "__main__":
    main()

"""Failure detection of the data-parallel training step, on CPU gloo ranks
(documentation/system_architecture.md:747: a rank that stops must not leave
the others waiting in the gradient exchange forever).

A rank leaves between steps (its process exits without a fault): the
survivor's next step raises RankFailure from the heartbeat, naming the
missing rank, before any collective of that step is launched. A rank that
leaves after the heartbeat but before the gradient all-reduce makes the
survivor's all-reduce fail: RankFailure from GradBuckets.finish, with the
process group aborted."""
import datetime
import json
import os
import tempfile
import time

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from encoder_ref import RefOps, dense_masks, make_cells, tiny_config, to_torch
from tributary_b200.encoder import RTEncoder
from tributary_b200.train import Heartbeat, RankFailure, TrainStep

KINDS = (0, 1, 2, 3)


def _rank(rank, world, init_file, result_file, leave_at):
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    torch.manual_seed(0)
    model = RTEncoder(tiny_config(), ops=RefOps())
    hb = Heartbeat(timeout_s=2.0)
    step = TrainStep(model, heartbeat=hb, allreduce_timeout_s=10.0)
    cells = make_cells(20 + rank)
    c, col, cat = to_torch(cells, "cpu")
    masks = dense_masks(cells, KINDS, "cpu")
    out = {"steps": 0}
    t0 = time.time()
    try:
        for n in range(4):
            if rank == 1 and n == leave_at[0]:
                if leave_at[1] == "after_heartbeat":
                    hb.step(n)  # reaches the step, then leaves before the all-reduce
                os._exit(0)
            t0 = time.time()
            step(c, masks, col, cat)
            out["steps"] += 1
    except RankFailure as e:
        out.update(error="RankFailure", message=str(e), seconds=time.time() - t0)
    if rank == 0:
        with open(result_file, "w") as f:
            json.dump(out, f)
    if dist.is_initialized():  # a RankFailure has already aborted the group
        dist.destroy_process_group()


def _run(leave_at):
    world = 2
    with tempfile.TemporaryDirectory() as d:
        init_file, result_file = os.path.join(d, "init"), os.path.join(d, "result.json")
        ctx = mp.start_processes(_rank, args=(world, init_file, result_file, leave_at), nprocs=world,
                                 start_method="spawn", join=False)
        deadline = time.time() + 120
        while not ctx.join(timeout=5) and time.time() < deadline:
            pass
        with open(result_file) as f:
            return json.load(f)


def test_rank_leaving_between_steps_is_named_by_the_heartbeat():
    out = _run((2, "before_heartbeat"))
    assert out["steps"] == 2
    assert out["error"] == "RankFailure"
    assert "step 2" in out["message"] and "[1]" in out["message"]
    assert out["seconds"] < 15


def test_rank_leaving_before_the_allreduce_fails_the_exchange():
    out = _run((1, "after_heartbeat"))
    assert out["steps"] == 1
    assert out["error"] == "RankFailure"
    assert "all-reduce" in out["message"]
    assert out["seconds"] < 15

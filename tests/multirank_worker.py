"""One rank of the multi-rank CPU tests (tests/test_multirank.py), launched by torchrun
or as plain processes with RANK / WORLD_SIZE / MASTER_* set, over gloo.

    python multirank_worker.py ok   OUT_DIR CKPT_DIR   # bench.py's rank helpers
    python multirank_worker.py gone OUT_DIR            # rank 1 exits before the barrier
    python multirank_worker.py stall OUT_DIR           # rank 1 stays alive but never joins

Each rank writes OUT_DIR/rank<r>.json with what it saw.
"""

import argparse
import contextlib
import copy
import io
import json
import os
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [ROOT, os.path.join(ROOT, "nemotron3-diarization-wgpu_b200")]

import bench  # noqa: E402


def _dump(out_dir, rank, rec):
    with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
        json.dump(rec, f)


def ok(out_dir, ckpt_dir):
    import torch.distributed as dist

    import synth

    world, rank, local = bench.dist_setup("gloo", timeout_s=60)
    rec = {"world": world, "rank": rank, "local": local, "backend": dist.get_backend()}
    # device times differ per rank; every rank must report the slowest
    rec["max"] = bench.max_over_ranks(1.5 + rank, world)
    gathered = [None] * world
    dist.all_gather_object(gathered, {"c4": bench.item_seeds("c4", rank, 3, world),
                                      "c3": bench.item_seeds("c3", rank, 3, world)})
    rec["seeds"] = gathered
    # rank 0 writes the checkpoint; rank 1 must find it complete when checkpoint() returns
    cfg = copy.deepcopy(synth.MODEL_CONFIG)
    cfg["audio_config"]["num_hidden_layers"] = 1
    if rank == 1:
        time.sleep(0.5)  # give rank 0 a head start so that rank 1 really waits at the barrier
    d = bench.checkpoint(rank, world, directory=ckpt_dir, cfg=cfg)
    rec["ckpt"] = d
    rec["ckpt_files"] = sorted(os.listdir(d))
    with open(os.path.join(d, "config.json")) as f:
        rec["ckpt_layers"] = json.load(f)["audio_config"]["num_hidden_layers"]
    # --impl reference: every rank but 0 returns at once, printing nothing
    if rank != 0:
        buf = io.StringIO()
        args = argparse.Namespace(gpus=world, steps=1, warmup=0)
        t0 = time.perf_counter()
        with contextlib.redirect_stdout(buf):
            bench.run_reference(args, world, rank)
        rec["reference_stdout"] = buf.getvalue()
        rec["reference_s"] = time.perf_counter() - t0
    rec["rate"] = bench.job_rate(world, 4, 60.0, 2, bench.max_over_ranks(1000.0 * (rank + 1), world))
    bench.barrier(world)
    dist.destroy_process_group()
    _dump(out_dir, rank, rec)


def gone(out_dir, stall):
    """Rank 1 fails before the barrier: it exits, or (`stall`) it stays alive for 10 s
    without joining.  Rank 0 must get an error from its collective (a closed connection,
    or the process group's 5 s timeout), not wait for good."""
    import torch.distributed as dist

    world, rank, _ = bench.dist_setup("gloo", timeout_s=5)
    if rank == 1:
        _dump(out_dir, rank, {"rank": rank, "left": True})
        if stall:
            time.sleep(10)
        os._exit(7)
    t0 = time.perf_counter()
    rec = {"rank": rank}
    try:
        bench.barrier(world)
        bench.max_over_ranks(1.0, world)
        rec["error"] = None
    except Exception as e:  # the collective's error, reported on the host
        rec["error"] = f"{type(e).__name__}: {e}"[:300]
    rec["wait_s"] = time.perf_counter() - t0
    _dump(out_dir, rank, rec)
    with contextlib.suppress(Exception):
        dist.destroy_process_group()
    os._exit(0)


if __name__ == "__main__":
    if sys.argv[1] == "ok":
        ok(sys.argv[2], sys.argv[3])
    else:
        gone(sys.argv[2], sys.argv[1] == "stall")

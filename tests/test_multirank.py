"""The multi-GPU host logic of bench.py on CPU: two gloo ranks launched the way the
N>1 benchmark is (torchrun, 127.0.0.1).  The data path has no collective: ranks run
disjoint clips, and only the barrier and the max over ranks of the device time cross
processes."""

import json
import os
import socket
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
WORKER = os.path.join(ROOT, "tests", "multirank_worker.py")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _env():
    env = dict(os.environ, MASTER_ADDR="127.0.0.1", OMP_NUM_THREADS="1")
    env.pop("CUDA_VISIBLE_DEVICES", None)
    return env


def _read(out_dir, world):
    recs = []
    for r in range(world):
        with open(os.path.join(out_dir, f"rank{r}.json")) as f:
            recs.append(json.load(f))
    return recs


def test_two_ranks_torchrun(tmp_path):
    out = tmp_path / "out"
    out.mkdir()
    ckpt = tmp_path / "ckpt"
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()), WORKER, "ok", str(out), str(ckpt)]
    p = subprocess.run(cmd, env=_env(), capture_output=True, text=True, timeout=300)
    assert p.returncode == 0, p.stderr[-3000:]
    r0, r1 = _read(str(out), 2)
    assert [r0["rank"], r1["rank"]] == [0, 1] and r0["world"] == r1["world"] == 2
    assert [r0["local"], r1["local"]] == [0, 1] and r0["backend"] == "gloo"
    # max over ranks: both ranks report the slowest rank's value
    assert r0["max"] == r1["max"] == 2.5
    # weak scaling: each rank's clips and sessions are its own
    for key in ("c4", "c3"):
        s0, s1 = r0["seeds"][0][key], r0["seeds"][1][key]
        assert len(s0) == len(s1) == 3 and not set(s0) & set(s1)
        assert r0["seeds"] == r1["seeds"]
    # config 4's 8192 clips and config 3's 256 sessions split evenly: rank 1 owns the second half
    assert r0["seeds"][1]["c4"] == [4096, 4097, 4098] and r0["seeds"][1]["c3"] == [128, 129, 130]
    # one checkpoint, complete on every rank when checkpoint() returns
    assert r0["ckpt"] == r1["ckpt"] == str(ckpt)
    for r in (r0, r1):
        assert r["ckpt_files"] == ["config.json", "model.safetensors", "processor_config.json"]
        assert r["ckpt_layers"] == 1
    assert not [n for n in os.listdir(tmp_path) if ".tmp" in n]  # rank 0's staging directory is gone
    # --impl reference on rank 1: no work, no output
    assert r1["reference_stdout"] == "" and r1["reference_s"] < 1.0
    # whole-job rate: 2 ranks x 4 clips x 60 s x 2 steps over the slowest rank's 2000 ms
    assert r0["rate"] == r1["rate"] == pytest.approx(2 * 4 * 60.0 * 2 / 2.0)


@pytest.mark.parametrize("how", ["gone", "stall"])
def test_rank_that_never_joins(tmp_path, how):
    """A rank that exits before the barrier, or stays alive without joining it: the
    other rank's collective ends with an error on the host, at once or within the
    5 s process-group timeout."""
    port = str(_free_port())
    procs = []
    for r in range(2):
        env = dict(_env(), RANK=str(r), LOCAL_RANK=str(r), WORLD_SIZE="2", MASTER_PORT=port)
        procs.append(subprocess.Popen([sys.executable, WORKER, how, str(tmp_path)], env=env,
                                      stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True))
    codes = []
    for p in procs:
        try:
            p.communicate(timeout=120)
        except subprocess.TimeoutExpired:
            p.kill()
            p.communicate()
        codes.append(p.returncode)
    assert codes == [0, 7]
    r0, r1 = _read(str(tmp_path), 2)
    assert r1["left"] and r0["error"] is not None
    assert r0["wait_s"] < (2 if how == "gone" else 15)


def test_reference_arm_two_ranks(tmp_path):
    """`bench.py --impl reference` under torchrun at N=2, as the driver launches it:
    rank 0 alone times the CPU oracle and prints one JSON line; rank 1 exits 0."""
    env = dict(_env(), TMPDIR=str(tmp_path))  # the bench checkpoint goes under tmp_path
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(ROOT, "bench.py"), "--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "1"]
    p = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stderr[-3000:]
    lines = [ln for ln in p.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["n_gpus"] == 2 and line["steps"] == 1
    assert line["value"] > 0 and line["higher_is_better"] and line["metric"] == "offline RTFx (audio-s/wall-s)"
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": line["unit"], "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}

"""The fp32 noise floor of the frame_check gates on the synthetic checkpoint.

BASELINE's random-init weights (N(0, 0.02), zero biases) make the logits about
N(0, 0.006), so many lie within 1e-7 of the f32 sigmoid's 0.5 decision, and any two
fp32 implementations that round differently disagree there.  This script measures
that with two CPU builds of the same oracle: the plain one (-ffp-contract=off, the
fixtures in tests/golden/full/) and one whose multiply-adds are contracted into
fused FMAs (oracle/liboracle_fma.so), which is just as valid an fp32 evaluation of
the reference's code.  For each fixture it prints the FMA build's logit maxdiff,
its sigmoid>0.5 flips against the plain build, whether the segments are identical,
and every flip's two logits.

    make -C oracle liboracle_fma.so
    python tests/golden/noise_floor.py [fixture ...]     # default: all of tests/golden/full

It runs each fixture's case again on the CPU (about as long as make_full_golden.py),
and records each fixture's result in tests/golden/full/noise_floor.json (maxdiff,
flips, segments identical, the flips' logits), which the GPU tests read: they allow a
decision to differ only where the oracle's logit lies within 4x that fixture's
measured maxdiff of the boundary.
"""

import json
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
FMA_LIB = os.path.join(ROOT, "oracle", "liboracle_fma.so")


def compare(got, want):
    import oracle

    got = np.asarray(got, np.float32).reshape(-1, 8)
    want = np.asarray(want, np.float32).reshape(-1, 8)
    # sigmoid > 0.5 in f32 (src/bin/frame_check.rs:188-190); the sigmoid is the oracle's
    # expf-based one in both builds
    flips = np.argwhere(oracle.sigmoid_above_half(got).reshape(got.shape) !=
                        oracle.sigmoid_above_half(want).reshape(want.shape))
    return {"maxdiff": float(np.abs(got.astype(np.float64) - want.astype(np.float64)).max()),
            "logits": int(want.size), "flips": int(len(flips)),
            "flip_values": [(int(r), int(c), float(want[r, c]), float(got[r, c])) for r, c in flips]}


def run_one(name):
    """One fixture through the FMA-contracted oracle (this process must have loaded it)."""
    sys.path[:0] = [HERE, os.path.join(ROOT, "nemotron3-diarization-wgpu_b200"), os.path.join(ROOT, "oracle")]
    import oracle
    import synth
    from make_full_golden import audio_sha, cases

    assert oracle.LIB_PATH == FMA_LIB
    make, mode = cases()[name]
    z = np.load(os.path.join(HERE, "full", name + ".npz"))
    a = make()
    assert audio_sha(a) == str(z["audio_sha256"])
    d = tempfile.mkdtemp(prefix="n3d_noise_")
    synth.write_checkpoint(d, seed=0)
    om = oracle.OracleModel.load(d)
    r = om.run_offline(a) if mode == "offline" else om.run_streaming(a, mode)
    res = compare(r["logits"], z["logits"])
    segs = lambda l: oracle.extract_speaker_dict(np.asarray(l, np.float32).ravel(), len(l) // 8, 8, 0.01)
    res["segments_identical"] = segs(np.asarray(r["logits"], np.float32).ravel()) == segs(z["logits"].ravel())
    res["name"] = name
    return res


def main(names):
    if len(names) == 1 and names[0].startswith("--one="):
        print(json.dumps(run_one(names[0][6:])), flush=True)
        return
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "liboracle_fma.so"], check=True)
    names = names or sorted(f[:-4] for f in os.listdir(os.path.join(HERE, "full")) if f.endswith(".npz"))
    env = dict(os.environ, N3D_ORACLE_LIB=FMA_LIB)
    out_path = os.path.join(HERE, "full", "noise_floor.json")
    for n in names:
        p = subprocess.run([sys.executable, __file__, "--one=" + n], env=env, capture_output=True, text=True)
        if p.returncode:
            print(n, "failed:", p.stderr[-2000:], flush=True)
            continue
        r = json.loads(p.stdout.strip().splitlines()[-1])
        table = json.load(open(out_path)) if os.path.exists(out_path) else {}
        table[n] = {k: r[k] for k in ("maxdiff", "logits", "flips", "segments_identical", "flip_values")}
        with open(out_path, "w") as f:
            json.dump(dict(sorted(table.items())), f, indent=1)
            f.write("\n")
        print(f"{n:24s} logits {r['logits']:8d}  maxdiff {r['maxdiff']:.3e}  flips {r['flips']}  "
              f"segments identical {r['segments_identical']}", flush=True)
        for row, col, plain, fma in r["flip_values"]:
            print(f"    flip at row {row} speaker {col}: plain oracle {plain:+.3e}, FMA oracle {fma:+.3e}", flush=True)


if __name__ == "__main__":
    main(sys.argv[1:])

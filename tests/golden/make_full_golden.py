"""Regenerate the full-model golden fixtures (tests/golden/full/) from the CPU oracle.

The oracle (oracle/) restates the reference's CPU path.  These fixtures freeze its
RunOutput on the synthetic 31-layer checkpoint (synth.write_checkpoint, seed 0) for
every BASELINE configuration and mode, so that the GPU tests gate the CUDA path
with the reference's frame_check gates (src/bin/frame_check.rs:170-240) without
running the oracle on the GPU box.  Inputs are regenerated from their seeds
(synth.py); each fixture stores the SHA-256 of its audio, so a drift in the
generator shows up as a clear failure instead of a parity miss.

    python tests/golden/make_full_golden.py [name ...]

Takes about 10 minutes on 8 cores.  Cases (audio from synth.py):
  c0_<mode>.npz              config 0 (30 s, 3 speakers) in the three streaming modes
  c4_clip0_offline.npz       config 4 clip 0 (60 s, 61 % overlap, RT60 0.5 s, 8 dB), offline
  c4_clip0_ultra.npz         the same clip, ultra_low_latency
  c4_clip127_offline.npz     config 4 clip 127, offline (the last clip of a 128-clip batch)
  c3_session0_120s.npz       config 3 session 0, first 120 s, ultra_low_latency
  c2_600s_offline.npz        config 2's recipe (4 speakers, band-passed, 15 dB) for 10 min, offline
"""

import hashlib
import os
import sys
import tempfile
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
OUT = os.path.join(HERE, "full")
for p in (os.path.join(ROOT, "nemotron3-diarization-wgpu_b200"), os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

MODES = ("low_latency", "very_low_latency", "ultra_low_latency")


def cases():
    """name -> (audio factory, mode)."""
    import synth

    c = {f"c0_{m}": (synth.config0_audio, m) for m in MODES}
    c["c4_clip0_offline"] = (lambda: synth.config4_clip(0), "offline")
    c["c4_clip0_ultra"] = (lambda: synth.config4_clip(0), "ultra_low_latency")
    c["c4_clip127_offline"] = (lambda: synth.config4_clip(127), "offline")
    c["c3_session0_120s"] = (lambda: synth.config3_session(0, 120.0), "ultra_low_latency")
    c["c2_600s_offline"] = (lambda: synth.config2_audio(600.0), "offline")
    return c


def audio_sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a, np.float32).tobytes()).hexdigest()


def main(names):
    import oracle
    import synth

    d = tempfile.mkdtemp(prefix="n3d_full_")
    synth.write_checkpoint(d, seed=0)
    om = oracle.OracleModel.load(d)
    os.makedirs(OUT, exist_ok=True)
    for name, (make, mode) in cases().items():
        if names and name not in names:
            continue
        a = make()
        t0 = time.time()
        r = om.run_offline(a) if mode == "offline" else om.run_streaming(a, mode)
        path = os.path.join(OUT, name + ".npz")
        np.savez(path, logits=np.asarray(r["logits"], np.float32).reshape(-1, 8), num_frames=r["num_frames"],
                 num_chunks=r["num_chunks"], cache_frames=r["cache_frames"], fifo_frames=r["fifo_frames"],
                 cache_compressed=int(r["cache_compressed"]), mode=mode, audio_sha256=audio_sha(a),
                 samples=a.size)
        print(f"{path}: {os.path.getsize(path)} bytes, {time.time() - t0:.1f} s", flush=True)


if __name__ == "__main__":
    main(sys.argv[1:])

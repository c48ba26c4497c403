"""Regenerate the golden fixtures in this directory from the CPU oracle.

The oracle (oracle/) restates the reference's CPU path; these fixtures freeze its
outputs on small seeded cases so that the parity tests can check the CUDA path
against committed numbers and check the oracle itself against drift.  Inputs are
regenerated from their seeds (synth.py), so only outputs are stored.

    python tests/golden/make_golden.py

Cases (tiny model = the 2-layer, 32-frame-cache variant of tests/conftest.py):
  mel_clip7_1s.npy          log-mel (centred) of synth.clip(7, 1.0 s, 2 speakers)
  tiny_offline_clip12.npz   tiny model, offline, synth.clip(12, 9.0 s, 3)
  tiny_ull_clip11.npz       tiny model, ultra_low_latency, synth.clip(11, 6.0 s, 2)
  linear_17x24x512.npy      tensor::linear, x ~ N(0,1), w ~ N(0, 0.02^2), b ~ N(0,1), seed 17
"""

import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
for p in (os.path.join(ROOT, "tests"), os.path.join(ROOT, "nemotron3-diarization-wgpu_b200"),
          os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def linear_inputs():
    rng = np.random.default_rng(17)
    m, n, k = 17, 24, 512
    x = rng.standard_normal(m * k).astype(np.float32)
    w = (rng.standard_normal(n * k) * 0.02).astype(np.float32)
    b = rng.standard_normal(n).astype(np.float32)
    return x, w, b, m, n, k


def cases(tiny_oracle):
    import oracle
    import synth

    out = {}
    out["mel_clip7_1s.npy"] = tiny_oracle.log_mel(synth.clip(7, 1.0, 2), centered=True)
    for name, fn in (("tiny_offline_clip12.npz", lambda: tiny_oracle.run_offline(synth.clip(12, 9.0, 3))),
                     ("tiny_ull_clip11.npz",
                      lambda: tiny_oracle.run_streaming(synth.clip(11, 6.0, 2), "ultra_low_latency"))):
        r = fn()
        out[name] = dict(logits=np.asarray(r["logits"], np.float32), num_frames=r["num_frames"],
                         num_chunks=r["num_chunks"], cache_frames=r["cache_frames"], fifo_frames=r["fifo_frames"],
                         cache_compressed=int(r["cache_compressed"]))
    x, w, b, m, n, k = linear_inputs()
    out["linear_17x24x512.npy"] = oracle.linear(x, m, k, w, n, b).reshape(m, n)
    return out


def tiny_oracle_model():
    import oracle
    import synth
    from conftest import tiny_config

    d = tempfile.mkdtemp(prefix="n3d_tiny_")
    synth.write_checkpoint(d, seed=0, cfg=tiny_config())
    return oracle.OracleModel.load(d)


def main():
    for name, v in cases(tiny_oracle_model()).items():
        path = os.path.join(HERE, name)
        if isinstance(v, dict):
            np.savez(path, **v)
        else:
            np.save(path, v)
        print(path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()

"""ctypes binding to the CPU oracle (liboracle.so) -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
module, as the checker; the product library never imports it.  It mirrors the
reference's Rust API shape (src/lib.rs:45-64) so parity tests read like the
reference's own: ``OracleModel.run_offline(samples)``,
``OracleModel.run_streaming(samples, mode)``, ``extract_speaker_dict(...)``.
"""

from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
# N3D_ORACLE_LIB selects another build of the same restatement (the FMA-contracted
# variant that tests/golden/noise_floor.py compares against); unset, the plain oracle.
LIB_PATH = os.environ.get("N3D_ORACLE_LIB") or os.path.join(HERE, "liboracle.so")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_fp = C.POINTER(C.c_float)
_sz = C.c_size_t

MODES = {"low_latency": 0, "very_low_latency": 1, "ultra_low_latency": 2}


class Fe(C.Structure):
    _fields_ = [("feature_size", _sz), ("n_fft", _sz), ("hop_length", _sz), ("win_length", _sz),
                ("sampling_rate", _sz), ("preemphasis", C.c_float)]


class CacheCfg(C.Structure):
    _fields_ = [("fifo_length", _sz), ("speaker_cache_length", _sz), ("update_period", _sz),
                ("num_silence_frames", _sz), ("score_threshold", C.c_float),
                ("latest_frames_score_boost", C.c_float), ("num_speakers", _sz), ("subsampling_factor", _sz),
                ("min_positive_scores", _sz), ("num_strong_boosted_frames", _sz), ("num_weak_boosted_frames", _sz)]


class Cfg(C.Structure):
    _fields_ = [("hidden", _sz), ("layers", _sz), ("heads", _sz), ("inter", _sz), ("n_mels", _sz), ("sub", _sz),
                ("rope_theta", C.c_double), ("head_hidden", _sz), ("num_speakers", _sz), ("chunk_length", _sz),
                ("chunk_right_context", _sz), ("cache_stream", CacheCfg), ("cache_offline", CacheCfg), ("fe", Fe),
                ("modes", (_sz * 2) * 3)]


_PP = C.POINTER(_fp)


class Weights(C.Structure):
    _fields_ = [(n, _fp) for n in ("embed_proj", "in_ln_w", "in_ln_b", "fin_ln_w", "fin_ln_b")] + \
               [(n, _PP) for n in ("ln1_w", "ln1_b", "q", "k", "v", "o", "o_b", "ln2_w", "ln2_b", "fc1", "fc1_b",
                                   "fc2", "fc2_b")] + \
               [(n, _fp) for n in ("proj_w", "proj_b", "conv_w", "conv_b", "dense_w", "dense_b", "out_w", "out_b",
                                   "silence", "mel_filters")]


class RunOutput(C.Structure):
    _fields_ = [("logits", _fp), ("num_frames", _sz), ("num_chunks", _sz), ("cache_compressed", C.c_int),
                ("cache_frames", _sz), ("fifo_frames", _sz)]


class StepTrace(C.Structure):
    _fields_ = [("step", _sz), ("cached_frames", _sz), ("window_frames", _sz), ("valid_frames", _sz),
                ("scored_frames", _sz), ("window", _fp), ("encoder_out", _fp), ("step_logits", _fp),
                ("cache_embeds", _fp), ("cache_probs", _fp), ("fifo", _fp), ("cache_frames", _sz),
                ("fifo_frames", _sz), ("cache_compressed", C.c_int)]


class Segment(C.Structure):
    _fields_ = [("start", C.c_float), ("end", C.c_float), ("speaker", _sz)]


STEP_CB = C.CFUNCTYPE(None, C.c_void_p, C.POINTER(StepTrace))


def build() -> str:
    """Compile liboracle.so with the Makefile beside this file (gcc, OpenMP)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(os.path.join(HERE, "n3d_oracle.c")):
            build()
        L = C.CDLL(LIB_PATH)
        L.orc_linear.argtypes = [_f32p, _sz, _sz, _f32p, _sz, C.c_void_p, _f32p]
        L.orc_matmul.argtypes = [_f32p, _sz, _sz, _f32p, _sz, _f32p]
        L.orc_layer_norm.argtypes = [_f32p, _sz, _sz, _f32p, _f32p, _f32p]
        L.orc_gelu.argtypes = [_f32p, _sz, _f32p]
        L.orc_relu.argtypes = [_f32p, _sz, _f32p]
        L.orc_softmax_last.argtypes = [_f32p, _sz, _sz]
        L.orc_hann_periodic_false.argtypes = [_sz, _f32p]
        L.orc_slaney_mel_filterbank.argtypes = [_sz, _sz, _sz, C.c_double, C.c_double, _f32p]
        L.orc_frame_count.argtypes = [_sz, C.POINTER(Fe), C.c_int]
        L.orc_frame_count.restype = _sz
        L.orc_log_mel.argtypes = [_f32p, _sz, C.POINTER(Fe), C.c_int, _f32p, _f32p]
        L.orc_log_mel.restype = _sz
        L.orc_fft.argtypes = [_f32p, _f32p, _sz]
        L.orc_rope_tables.argtypes = [_sz, _sz, C.c_double, _sz, _f32p, _f32p]
        L.orc_apply_rope.argtypes = [_f32p, _sz, _sz, _sz, _f32p, _f32p]
        L.orc_attention.argtypes = [_f32p, _f32p, _f32p, _sz, _sz, _sz, _sz, _f32p]
        L.orc_embed_range.argtypes = [C.POINTER(Cfg), C.POINTER(Weights), _f32p, _sz, _sz, _sz, _f32p]
        L.orc_forward_embeds.argtypes = [C.POINTER(Cfg), C.POINTER(Weights), _f32p, _sz, _sz, _f32p]
        L.orc_head_forward.argtypes = [C.POINTER(Cfg), C.POINTER(Weights), _f32p, _sz, _f32p]
        L.orc_pool_probs.argtypes = [C.POINTER(CacheCfg), _f32p, _sz, _u8p, _sz, _f32p]
        L.orc_num_popped.argtypes = [C.POINTER(CacheCfg), _sz]
        L.orc_num_popped.restype = _sz
        L.orc_frame_scores.argtypes = [C.POINTER(CacheCfg), _f32p, _sz, _f32p]
        L.orc_boost_top.argtypes = [C.POINTER(CacheCfg), _f32p, _sz, _sz, C.c_float]
        L.orc_sigmoid_above_half.argtypes = [_f32p, _sz, _u8p]
        L.orc_compress_picked.argtypes = [C.POINTER(CacheCfg), _f32p, _sz, np.ctypeslib.ndpointer(np.uintp)]
        L.orc_compress_picked.restype = _sz
        L.orc_compress.argtypes = [C.POINTER(CacheCfg), _sz, _f32p, _f32p, _sz, _f32p, _f32p, _f32p]
        L.orc_run_offline.argtypes = [C.POINTER(Cfg), C.POINTER(Weights), _f32p, _sz, C.POINTER(RunOutput),
                                      STEP_CB, C.c_void_p]
        L.orc_run_streaming.argtypes = [C.POINTER(Cfg), C.POINTER(Weights), _f32p, _sz, C.c_int,
                                        C.POINTER(RunOutput), STEP_CB, C.c_void_p]
        L.orc_run_output_free.argtypes = [C.POINTER(RunOutput)]
        L.orc_round2.argtypes = [C.c_float]
        L.orc_round2.restype = C.c_float
        L.orc_extract_speaker_dict.argtypes = [_f32p, _sz, _sz, C.c_float, C.c_void_p, C.c_float,
                                               C.POINTER(Segment), _sz]
        L.orc_extract_speaker_dict.restype = _sz
        L.orc_activity_stats.argtypes = [_f32p, _sz, _sz, C.c_void_p, C.c_float, np.ctypeslib.ndpointer(np.uintp)]
        L.orc_activity_stats.restype = C.c_float
        L.orc_set_threads.argtypes = [C.c_int]
        _lib = L
    return _lib


def f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


# ------------------------------------------------------------------ tensor ops

def linear(x, rows, cols, w, out, bias=None):
    y = np.empty(rows * out, np.float32)
    b = f32(bias) if bias is not None else None
    lib().orc_linear(f32(x), rows, cols, f32(w), out, b.ctypes.data if b is not None else None, y)
    return y


def matmul(a, m, k, b, n):
    c = np.empty(m * n, np.float32)
    lib().orc_matmul(f32(a), m, k, f32(b), n, c)
    return c


def layer_norm(x, rows, cols, w, b):
    y = np.empty(rows * cols, np.float32)
    lib().orc_layer_norm(f32(x), rows, cols, f32(w), f32(b), y)
    return y


def gelu(x):
    x = f32(x)
    y = np.empty_like(x)
    lib().orc_gelu(x, x.size, y)
    return y


def relu(x):
    x = f32(x)
    y = np.empty_like(x)
    lib().orc_relu(x, x.size, y)
    return y


def softmax_last(x, rows, cols):
    x = f32(x).copy()
    lib().orc_softmax_last(x, rows, cols)
    return x


def rope_tables(seq, hd, theta=10000.0, offset=0):
    c = np.empty(seq * hd, np.float32)
    s = np.empty(seq * hd, np.float32)
    lib().orc_rope_tables(seq, hd, theta, offset, c, s)
    return c, s


def apply_rope(x, seq, nh, hd, cos_t, sin_t):
    y = f32(x).copy()
    lib().orc_apply_rope(y, seq, nh, hd, f32(cos_t), f32(sin_t))
    return y


def attention(q, k, v, seq, nh, hd, valid):
    out = np.empty(seq * nh * hd, np.float32)
    lib().orc_attention(f32(q), f32(k), f32(v), seq, nh, hd, valid, out)
    return out


# ------------------------------------------------------------------- front end

def fe_struct(fe: dict) -> Fe:
    return Fe(fe["feature_size"], fe["n_fft"], fe["hop_length"], fe["win_length"], fe["sampling_rate"],
              fe["preemphasis"])


def hann_periodic_false(n):
    out = np.empty(n, np.float32)
    lib().orc_hann_periodic_false(n, out)
    return out


def slaney_mel_filterbank(n_mels, n_fft, sr, fmin, fmax):
    out = np.empty(n_mels * (n_fft // 2 + 1), np.float32)
    lib().orc_slaney_mel_filterbank(n_mels, n_fft, sr, fmin, fmax, out)
    return out


def frame_count(n, fe: dict, centered: bool) -> int:
    f = fe_struct(fe)
    return lib().orc_frame_count(n, C.byref(f), int(centered))


def log_mel(samples, fe: dict, centered: bool, filters):
    f = fe_struct(fe)
    s = f32(samples)
    nfr = lib().orc_frame_count(s.size, C.byref(f), int(centered))
    out = np.zeros(max(nfr, 1) * fe["feature_size"], np.float32)
    lib().orc_log_mel(s, s.size, C.byref(f), int(centered), f32(filters), out)
    return out[: nfr * fe["feature_size"]].reshape(nfr, fe["feature_size"])


def fft(re, im):
    re = f32(re).copy()
    im = f32(im).copy()
    lib().orc_fft(re, im, re.size)
    return re, im


# ----------------------------------------------------------------- cache policy

def cache_cfg(**kw) -> CacheCfg:
    c = CacheCfg()
    for k, v in kw.items():
        setattr(c, k, v)
    return c


def cache_cfg_from_model(cfg: dict, offline: bool) -> CacheCfg:
    """CacheConfig::from_model / ::offline, src/streaming.rs:54-86."""
    s = cfg["streaming_config"]
    ns = s["num_speakers"]
    budget = s["speaker_cache_length"] // ns - s["speaker_cache_silence_frames_per_speaker"]
    fl = lambda r: int(np.floor(np.float32(budget) * np.float32(r)))
    return cache_cfg(
        fifo_length=cfg["fifo_length"] if offline else s["fifo_length"],
        speaker_cache_length=s["speaker_cache_length"],
        update_period=cfg["speaker_cache_update_period"] if offline else s["speaker_cache_update_period"],
        num_silence_frames=s["speaker_cache_silence_frames_per_speaker"],
        score_threshold=s["prediction_score_threshold"],
        latest_frames_score_boost=s["latest_frames_score_boost"],
        num_speakers=ns, subsampling_factor=s["subsampling_factor"],
        min_positive_scores=fl(s["min_positive_scores_rate"]),
        num_strong_boosted_frames=fl(s["strong_boost_rate"]),
        num_weak_boosted_frames=fl(s["weak_boost_rate"]))


def pool_probs(cc: CacheCfg, logits, num_mel_frames, mask):
    m = np.ascontiguousarray(mask, dtype=np.uint8)
    out = np.zeros(max(num_mel_frames // cc.subsampling_factor, 1) * cc.num_speakers, np.float32)
    lib().orc_pool_probs(C.byref(cc), f32(logits), num_mel_frames, m, m.size, out)
    return out[: (num_mel_frames // cc.subsampling_factor) * cc.num_speakers]


def num_popped(cc: CacheCfg, n: int) -> int:
    return lib().orc_num_popped(C.byref(cc), n)


def frame_scores(cc: CacheCfg, probs, num_frames):
    out = np.empty(num_frames * cc.num_speakers, np.float32)
    lib().orc_frame_scores(C.byref(cc), f32(probs), num_frames, out)
    return out


def boost_top(cc: CacheCfg, scores, num_frames, k, boost):
    s = f32(scores).copy()
    lib().orc_boost_top(C.byref(cc), s, num_frames, k, boost)
    return s


def compress_picked(cc: CacheCfg, probs, num_frames):
    picked = np.zeros(cc.speaker_cache_length, np.uintp)
    sentinel = lib().orc_compress_picked(C.byref(cc), f32(probs), num_frames, picked)
    return picked.astype(np.int64), sentinel


def compress(cc: CacheCfg, hidden, embeds, probs, num_frames, silence):
    oe = np.empty(cc.speaker_cache_length * hidden, np.float32)
    op = np.empty(cc.speaker_cache_length * cc.num_speakers, np.float32)
    lib().orc_compress(C.byref(cc), hidden, f32(embeds), f32(probs), num_frames, f32(silence), oe, op)
    return oe, op


# --------------------------------------------------------------------- segments

def round2(v: float) -> float:
    return lib().orc_round2(v)


def sigmoid_above_half(logits) -> np.ndarray:
    """frame_check's per-logit decision, the f32 sigmoid above 0.5 (src/bin/frame_check.rs:188-190)."""
    lg = f32(logits).ravel()
    out = np.zeros(lg.size, np.uint8)
    lib().orc_sigmoid_above_half(lg, lg.size, out)
    return out.astype(bool)


def extract_speaker_dict(logits, num_frames, ns, duration, mask=None, threshold=0.5):
    """[(start, end, speaker)] as src/segments.rs:70-109 returns them."""
    lg = f32(logits)
    m = np.ascontiguousarray(mask, dtype=np.uint8) if mask is not None else None
    mp = m.ctypes.data if m is not None else None
    n = lib().orc_extract_speaker_dict(lg, num_frames, ns, duration, mp, threshold, None, 0)
    buf = (Segment * max(n, 1))()
    lib().orc_extract_speaker_dict(lg, num_frames, ns, duration, mp, threshold, buf, n)
    return [(buf[i].start, buf[i].end, int(buf[i].speaker)) for i in range(n)]


def activity_stats(logits, num_frames, ns, mask=None, threshold=0.5):
    per = np.zeros(ns, np.uintp)
    m = np.ascontiguousarray(mask, dtype=np.uint8) if mask is not None else None
    pct = lib().orc_activity_stats(f32(logits), num_frames, ns, m.ctypes.data if m is not None else None,
                                   threshold, per)
    return pct, [int(v) for v in per]


# ------------------------------------------------------------------------ model

class OracleModel:
    """The reference `Model` (src/model.rs:128-156) on the CPU oracle."""

    def __init__(self, cfg: dict, proc: dict, weights: dict):
        self.cfg, self.proc = cfg, proc
        a, hc = cfg["audio_config"], cfg["head_config"]
        fe = proc["feature_extractor"]
        c = Cfg()
        c.hidden, c.layers, c.heads = a["hidden_size"], a["num_hidden_layers"], a["num_attention_heads"]
        c.inter, c.n_mels, c.sub = a["intermediate_size"], a["num_mel_bins"], proc["subsampling_factor"]
        c.rope_theta = a["rope_parameters"]["rope_theta"]
        c.head_hidden, c.num_speakers = hc["hidden_size"], hc["num_speakers"]
        c.chunk_length, c.chunk_right_context = cfg["chunk_length"], cfg["chunk_right_context"]
        c.cache_stream = cache_cfg_from_model(cfg, offline=False)
        c.cache_offline = cache_cfg_from_model(cfg, offline=True)
        c.fe = fe_struct(fe)
        sm = proc["streaming_modes"]
        for i, k in enumerate(("low_latency", "very_low_latency", "ultra_low_latency")):
            c.modes[i][0], c.modes[i][1] = sm[k]
        self.c = c
        self._keep = []

        def arr(name):
            x = f32(weights[name])
            self._keep.append(x)
            return x.ctypes.data_as(_fp)

        def layer_arr(suffix):
            ptrs = (_fp * c.layers)(*[arr(f"model.audio_tower.layers.{i}.{suffix}") for i in range(c.layers)])
            self._keep.append(ptrs)
            return C.cast(ptrs, _PP)

        p = "model.audio_tower"
        w = Weights()
        w.embed_proj = arr(f"{p}.embedder.projection.weight")
        w.in_ln_w, w.in_ln_b = arr(f"{p}.input_layer_norm.weight"), arr(f"{p}.input_layer_norm.bias")
        w.fin_ln_w, w.fin_ln_b = arr(f"{p}.layer_norm.weight"), arr(f"{p}.layer_norm.bias")
        for fld, suf in (("ln1_w", "layer_norm1.weight"), ("ln1_b", "layer_norm1.bias"),
                         ("q", "self_attn.q_proj.weight"), ("k", "self_attn.k_proj.weight"),
                         ("v", "self_attn.v_proj.weight"), ("o", "self_attn.o_proj.weight"),
                         ("o_b", "self_attn.o_proj.bias"), ("ln2_w", "layer_norm2.weight"),
                         ("ln2_b", "layer_norm2.bias"), ("fc1", "mlp.fc1.weight"), ("fc1_b", "mlp.fc1.bias"),
                         ("fc2", "mlp.fc2.weight"), ("fc2_b", "mlp.fc2.bias")):
            setattr(w, fld, layer_arr(suf))
        w.proj_w, w.proj_b = arr("model.proj.weight"), arr("model.proj.bias")
        w.conv_w, w.conv_b = arr("model.upsampler.conv.weight"), arr("model.upsampler.conv.bias")
        w.dense_w, w.dense_b = arr("classifier.dense.weight"), arr("classifier.dense.bias")
        w.out_w, w.out_b = arr("classifier.out_proj.weight"), arr("classifier.out_proj.bias")
        w.silence = arr("silence_embeds")
        filters = slaney_mel_filterbank(fe["feature_size"], fe["n_fft"], fe["sampling_rate"], 0.0,
                                        fe["sampling_rate"] / 2.0)
        self.filters = filters
        w.mel_filters = filters.ctypes.data_as(_fp)
        self.w = w

    @classmethod
    def load(cls, directory: str) -> "OracleModel":
        import json
        import sys

        sys.path.insert(0, os.path.join(os.path.dirname(HERE), "nemotron3-diarization-wgpu_b200"))
        from synth import load_safetensors

        with open(os.path.join(directory, "config.json")) as f:
            cfg = json.load(f)
        with open(os.path.join(directory, "processor_config.json")) as f:
            proc = json.load(f)
        return cls(cfg, proc, load_safetensors(os.path.join(directory, "model.safetensors")))

    @property
    def num_speakers(self) -> int:
        return self.c.num_speakers

    def _collect(self, out: RunOutput):
        ns = self.c.num_speakers
        n = out.num_frames * ns
        logits = np.ctypeslib.as_array(out.logits, shape=(n,)).copy() if n else np.zeros(0, np.float32)
        res = dict(logits=logits.reshape(out.num_frames, ns), num_frames=out.num_frames,
                   num_chunks=out.num_chunks, cache_compressed=bool(out.cache_compressed),
                   cache_frames=out.cache_frames, fifo_frames=out.fifo_frames)
        lib().orc_run_output_free(C.byref(out))
        return res

    def _trace_cb(self, traces):
        h, sub, ns = self.c.hidden, self.c.sub, self.c.num_speakers

        def cb(_user, tp):
            t = tp.contents
            wf = t.window_frames
            arr = lambda p, n: np.ctypeslib.as_array(p, shape=(n,)).copy() if n else np.zeros(0, np.float32)
            traces.append(dict(
                cached_frames=t.cached_frames, window_frames=wf, valid_frames=t.valid_frames,
                scored_frames=t.scored_frames, window=arr(t.window, wf * h).reshape(wf, h),
                encoder_out=arr(t.encoder_out, wf * h).reshape(wf, h),
                step_logits=arr(t.step_logits, wf * sub * ns).reshape(wf * sub, ns),
                cache_embeds=arr(t.cache_embeds, t.cache_frames * h).reshape(t.cache_frames, h),
                cache_probs=arr(t.cache_probs, t.cache_frames * ns).reshape(t.cache_frames, ns),
                fifo=arr(t.fifo, t.fifo_frames * h).reshape(t.fifo_frames, h),
                cache_compressed=bool(t.cache_compressed)))

        return STEP_CB(cb)

    def run_offline(self, samples, traces: list | None = None):
        out = RunOutput()
        cb = self._trace_cb(traces) if traces is not None else STEP_CB()
        s = f32(samples)
        lib().orc_run_offline(C.byref(self.c), C.byref(self.w), s, s.size, C.byref(out), cb, None)
        return self._collect(out)

    def run_streaming(self, samples, mode: str, traces: list | None = None):
        out = RunOutput()
        cb = self._trace_cb(traces) if traces is not None else STEP_CB()
        s = f32(samples)
        rc = lib().orc_run_streaming(C.byref(self.c), C.byref(self.w), s, s.size, MODES[mode], C.byref(out), cb,
                                     None)
        res = self._collect(out)
        if rc != 0:
            raise ValueError("audio too short for the streaming look-ahead")
        return res

    def log_mel(self, samples, centered=True):
        return log_mel(samples, self.proc["feature_extractor"], centered, self.filters)

    def embed_range(self, mel, num_frames, lo, hi):
        out = np.empty((hi - lo) * self.c.hidden, np.float32)
        lib().orc_embed_range(C.byref(self.c), C.byref(self.w), f32(mel), num_frames, lo, hi, out)
        return out.reshape(hi - lo, self.c.hidden)

    def forward_embeds(self, embeds, valid):
        e = f32(embeds)
        g = e.size // self.c.hidden
        out = np.empty(g * self.c.hidden, np.float32)
        lib().orc_forward_embeds(C.byref(self.c), C.byref(self.w), e, g, valid, out)
        return out.reshape(g, self.c.hidden)

    def head_forward(self, enc, frames):
        out = np.empty(frames * self.c.sub * self.c.num_speakers, np.float32)
        lib().orc_head_forward(C.byref(self.c), C.byref(self.w), f32(enc), frames, out)
        return out.reshape(frames * self.c.sub, self.c.num_speakers)

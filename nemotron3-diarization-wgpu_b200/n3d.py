"""Python binding of the C ABI (include/n3d.h) over libn3d.so.

It mirrors the reference crate's public API (src/lib.rs:45-64) so callers and
tests read like the reference's own code:

    model = Model.load_gpu(checkpoint_dir)          # Model::load_gpu
    out = model.run_offline(samples)                # Model::run_offline
    out = model.run_streaming(samples, "ultra_low_latency")
    segs = extract_speaker_dict(out.logits, out.num_frames, model.num_speakers, 0.01)

There is no CPU fallback: if libn3d.so is missing or no B200 is visible the
calls raise.
"""

from __future__ import annotations

import ctypes as C
import os
import weakref
import re
import subprocess
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libn3d.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "n3d.h")

MODES = {"low_latency": 0, "very_low_latency": 1, "ultra_low_latency": 2, "offline": 3}
STATUS = {0: "OK", 1: "Io", 2: "Json", 3: "Safetensors", 4: "TensorDtype", 5: "MissingTensor", 6: "TensorShape",
          7: "UnsupportedAudio", 8: "Npy", 9: "Gpu", 10: "Cuda", 11: "Timeout", 12: "NoDevice",
          13: "InvalidArgument"}

_sz = C.c_size_t
_fp = C.POINTER(C.c_float)


class DiarizationError(RuntimeError):
    """A non-OK n3d_status; `.kind` names the DiarizationError variant (src/error.rs:7-45)."""

    def __init__(self, status: int, message: str):
        self.status = status
        self.kind = STATUS.get(status, str(status))
        super().__init__(f"{self.kind}: {message}")


class _RunOutput(C.Structure):
    _fields_ = [("logits", _fp), ("num_frames", _sz), ("num_speakers", _sz), ("num_chunks", _sz),
                ("cache_compressed", C.c_int), ("cache_frames", _sz), ("fifo_frames", _sz)]


class _Segment(C.Structure):
    _fields_ = [("start", C.c_float), ("end", C.c_float), ("speaker", _sz)]


class _ModeParams(C.Structure):
    _fields_ = [(n, _sz) for n in ("hop_length", "n_fft", "subsampling", "mel_frames_per_chunk",
                                   "mel_frames_per_step", "lookahead_encoder_frames", "first_chunk_samples",
                                   "samples_per_chunk", "latency_ms")]


class _Chunk(C.Structure):
    _fields_ = [("start", _sz), ("len", _sz), ("centered", C.c_int), ("num_mel_frames", _sz), ("lookahead", _sz)]


class _StepPlan(C.Structure):
    _fields_ = [("cached_frames", _sz), ("window_frames", _sz), ("valid_frames", _sz), ("scored_frames", _sz),
                ("cache_frames", _sz), ("fifo_frames", _sz), ("cache_compressed", C.c_int)]


class CacheConfig(C.Structure):
    """CacheConfig (src/streaming.rs:39-52), as n3d_cache_config."""
    _fields_ = [("fifo_length", _sz), ("speaker_cache_length", _sz), ("update_period", _sz),
                ("num_silence_frames", _sz), ("score_threshold", C.c_float), ("latest_frames_score_boost", C.c_float),
                ("num_speakers", _sz), ("subsampling_factor", _sz), ("min_positive_scores", _sz),
                ("num_strong_boosted_frames", _sz), ("num_weak_boosted_frames", _sz)]


class _KernelStats(C.Structure):
    _fields_ = [("name", C.c_char_p), ("launches", _sz), ("ms", C.c_double), ("flops", C.c_double),
                ("bytes", C.c_double)]


@dataclass
class RunOutput:
    """RunOutput (src/model.rs:43-53)."""
    logits: np.ndarray  # [num_frames, num_speakers]
    num_frames: int
    num_chunks: int
    cache_compressed: bool
    cache_frames: int
    fifo_frames: int


@dataclass(frozen=True)
class Segment:
    """Segment (src/segments.rs:9-14): one speaker's active span, in seconds."""
    start: float
    end: float
    speaker: int


def build() -> str:
    """Compile libn3d.so for sm_100a with the Makefile beside this file."""
    subprocess.run(["make", "-s", "-C", HERE, "-j8"], check=True)
    return LIB_PATH


def header_functions() -> list[str]:
    """Names of every function include/n3d.h declares."""
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(n3d_[a-z_0-9]+)\s*\(", src)))


_lib = None


def lib() -> C.CDLL:
    """The loaded libn3d.so with every entry point's argument and result types set.
    Raises OSError when the library is not built: there is no CPU fallback."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise OSError(f"{LIB_PATH} is missing: build it with `make -C {HERE}` (no CPU fallback exists)")
    L = C.CDLL(LIB_PATH)
    vp, fpp = C.c_void_p, _fp
    sig = {
        "n3d_model_load_gpu": ([C.c_char_p, C.c_int, C.POINTER(vp)], C.c_int),
        "n3d_model_free": ([vp], None),
        "n3d_model_set_stream": ([vp, vp], C.c_int),
        "n3d_num_speakers": ([vp], _sz),
        "n3d_hidden_size": ([vp], _sz),
        "n3d_model_describe": ([vp], C.c_char_p),
        "n3d_run_offline": ([vp, fpp, _sz, C.POINTER(_RunOutput)], C.c_int),
        "n3d_run_streaming": ([vp, fpp, _sz, C.c_int, C.POINTER(_RunOutput)], C.c_int),
        "n3d_run_output_free": ([C.POINTER(_RunOutput)], None),
        "n3d_run_batch": ([vp, C.c_int, C.POINTER(fpp), C.POINTER(_sz), _sz, C.POINTER(_RunOutput)], C.c_int),
        "n3d_batch_out_frames": ([vp, C.c_int, C.POINTER(_sz), _sz, C.POINTER(_sz)], C.c_int),
        "n3d_run_batch_device": ([vp, C.c_int, vp, C.POINTER(_sz), C.POINTER(_sz), _sz, vp, C.POINTER(_sz)],
                                 C.c_int),
        "n3d_session_open": ([vp, C.c_int, C.POINTER(vp)], C.c_int),
        "n3d_session_push": ([vp, fpp, _sz, C.POINTER(_RunOutput)], C.c_int),
        "n3d_session_close": ([vp, C.POINTER(_RunOutput)], C.c_int),
        "n3d_session_free": ([vp], None),
        "n3d_sessions_push": ([C.POINTER(vp), C.POINTER(fpp), C.POINTER(_sz), _sz, C.c_int, C.POINTER(_RunOutput)],
                              C.c_int),
        "n3d_log_mel": ([vp, fpp, _sz, C.c_int, fpp, _sz, C.POINTER(_sz)], C.c_int),
        "n3d_embed_range": ([vp, fpp, _sz, _sz, _sz, fpp], C.c_int),
        "n3d_forward_embeds": ([vp, fpp, _sz, _sz, fpp], C.c_int),
        "n3d_head_forward": ([vp, fpp, _sz, fpp], C.c_int),
        "n3d_forward_window": ([vp, fpp, _sz, _sz, fpp], C.c_int),
        "n3d_extract_speaker_dict": ([fpp, _sz, _sz, C.c_float, vp, C.c_float, C.POINTER(C.POINTER(_Segment)),
                                      C.POINTER(_sz)], C.c_int),
        "n3d_segments_free": ([C.POINTER(_Segment)], None),
        "n3d_activity_stats": ([fpp, _sz, _sz, vp, C.c_float, C.POINTER(_sz)], C.c_float),
        "n3d_frame_duration": ([_sz, C.c_uint32], C.c_float),
        "n3d_config_load": ([C.c_char_p, C.POINTER(vp)], C.c_int),
        "n3d_config_free": ([vp], None),
        "n3d_mode_params_resolve": ([vp, C.c_int, C.POINTER(_ModeParams)], C.c_int),
        "n3d_streaming_chunks": ([vp, _sz, C.c_int, C.POINTER(_Chunk), _sz, C.POINTER(_sz)], C.c_int),
        "n3d_schedule": ([vp, C.c_int, _sz, C.POINTER(_StepPlan), _sz, C.POINTER(_sz), C.POINTER(_RunOutput)],
                         C.c_int),
        "n3d_linear": ([C.c_int, vp, _sz, _sz, vp, _sz, vp, vp], C.c_int),
        "n3d_linear_noalloc": ([C.c_int, vp, _sz, _sz, vp, _sz, vp, vp, vp], C.c_int),
        "n3d_layer_norm": ([C.c_int, vp, _sz, _sz, vp, vp, vp], C.c_int),
        "n3d_attention": ([C.c_int, vp, vp, vp, _sz, _sz, _sz, _sz, C.c_int, C.c_double, vp], C.c_int),
        "n3d_cache_compress": ([C.c_int, C.POINTER(CacheConfig), fpp, _sz, vp, _sz, vp, C.POINTER(_sz),
                                C.POINTER(_sz), C.POINTER(_sz), vp, vp], C.c_int),
        "n3d_selftest_wait_timeout": ([C.c_int, C.c_double, C.POINTER(C.c_double)], C.c_int),
        "n3d_bench_linear": ([C.c_int, _sz, _sz, _sz, C.c_int, C.POINTER(C.c_double)], C.c_int),
        "n3d_bench_attention": ([C.c_int, _sz, _sz, _sz, C.c_int, C.POINTER(C.c_double)], C.c_int),
        "n3d_bench_layer_norm": ([C.c_int, _sz, _sz, C.c_int, C.POINTER(C.c_double)], C.c_int),
        "n3d_profile_enable": ([vp, C.c_int], C.c_int),
        "n3d_profile_read": ([vp, C.POINTER(_KernelStats), _sz], _sz),
        "n3d_step_timing_enable": ([vp, C.c_int], C.c_int),
        "n3d_step_times": ([vp, C.POINTER(C.c_double), _sz], _sz),
        "n3d_last_error": ([], C.c_char_p),
        "n3d_version": ([], C.c_char_p),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res
    _lib = L
    return L


def _check(status: int) -> None:
    if status != 0:
        raise DiarizationError(status, lib().n3d_last_error().decode())


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(_fp)


def _free_output(o: _RunOutput) -> None:
    lib().n3d_run_output_free(C.byref(o))


def _collect(o: _RunOutput) -> RunOutput:
    """The output's logits as a numpy array without a copy: the array views the
    library-allocated buffer, which is released (n3d_run_output_free) once the array
    and every view of it are gone."""
    n = o.num_frames * o.num_speakers
    if n:
        buf = (C.c_float * n).from_address(C.cast(o.logits, C.c_void_p).value)
        weakref.finalize(buf, _free_output, _RunOutput.from_buffer_copy(o))
        logits = np.ctypeslib.as_array(buf)
    else:
        logits = np.zeros(0, np.float32)
        lib().n3d_run_output_free(C.byref(o))
    return RunOutput(logits.reshape(o.num_frames, o.num_speakers), int(o.num_frames), int(o.num_chunks),
                     bool(o.cache_compressed), int(o.cache_frames), int(o.fifo_frames))


def _struct_dict(st) -> dict:
    return {name: getattr(st, name) for name, _ in st._fields_}


class Config:
    """config.json + processor_config.json of a checkpoint (load_configs,
    src/config.rs:221-225) and the chunk arithmetic the runs follow.  Host only: no
    GPU is needed."""

    def __init__(self, handle: int):
        self._h = C.c_void_p(handle)

    @classmethod
    def load(cls, directory: str) -> "Config":
        """load_configs (src/config.rs:221-225) through n3d_config_load."""
        h = C.c_void_p()
        _check(lib().n3d_config_load(directory.encode(), C.byref(h)))
        return cls(h.value)

    def close(self) -> None:
        """Release the configuration (n3d_config_free)."""
        if self._h:
            lib().n3d_config_free(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def mode_params(self, mode: str) -> dict:
        """ModeParams::resolve (src/config.rs:152-195) as a dict of its fields."""
        p = _ModeParams()
        _check(lib().n3d_mode_params_resolve(self._h, MODES[mode], C.byref(p)))
        return _struct_dict(p)

    def streaming_chunks(self, n_samples: int, mode: str) -> list[dict]:
        """Model::streaming_chunks (src/model.rs:343-365) without the mel features."""
        n = _sz()
        _check(lib().n3d_streaming_chunks(self._h, n_samples, MODES[mode], None, 0, C.byref(n)))
        arr = (_Chunk * max(n.value, 1))()
        _check(lib().n3d_streaming_chunks(self._h, n_samples, MODES[mode], arr, n.value, C.byref(n)))
        return [_struct_dict(arr[i]) for i in range(n.value)]

    def schedule(self, n_samples: int, mode: str) -> tuple[list[dict], dict]:
        """The chunk-loop steps of a run (ChunkTrace counts, src/model.rs:57-75) and the
        RunOutput counts it will return (without logits)."""
        n = _sz()
        tot = _RunOutput()
        _check(lib().n3d_schedule(self._h, MODES[mode], n_samples, None, 0, C.byref(n), C.byref(tot)))
        arr = (_StepPlan * max(n.value, 1))()
        _check(lib().n3d_schedule(self._h, MODES[mode], n_samples, arr, n.value, C.byref(n), None))
        steps = [_struct_dict(arr[i]) for i in range(n.value)]
        for st in steps:
            st["cache_compressed"] = bool(st["cache_compressed"])
        totals = {k: v for k, v in _struct_dict(tot).items() if k != "logits"}
        totals["cache_compressed"] = bool(totals["cache_compressed"])
        return steps, totals


class Model:
    """The reference `Model` (src/model.rs:128-365) on a B200."""

    def __init__(self, handle: int, device: int):
        self._h = C.c_void_p(handle)
        self.device = device
        self._sessions = weakref.WeakSet()

    @classmethod
    def load_gpu(cls, directory: str, device: int = 0) -> "Model":
        """Model::load_gpu (src/model.rs:160-166): config.json, processor_config.json and
        model.safetensors from `directory`, with the weights resident on `device`."""
        h = C.c_void_p()
        _check(lib().n3d_model_load_gpu(directory.encode(), device, C.byref(h)))
        return cls(h.value, device)

    def close(self) -> None:
        """Free the model (n3d_model_free), after any sessions still open on it."""
        if self._h:
            for ss in list(self._sessions):  # sessions must go before their model
                ss.free()
            lib().n3d_model_free(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_stream(self, stream_handle: int | None) -> None:
        """Run on a caller-owned cudaStream_t (e.g. torch.cuda.current_stream().cuda_stream)."""
        _check(lib().n3d_model_set_stream(self._h, C.c_void_p(stream_handle) if stream_handle else None))

    @property
    def num_speakers(self) -> int:
        """Model::num_speakers (src/model.rs:211-213)."""
        return lib().n3d_num_speakers(self._h)

    @property
    def hidden_size(self) -> int:
        """Model::hidden_size (src/model.rs:215-217)."""
        return lib().n3d_hidden_size(self._h)

    def describe(self) -> str:
        """Model::gpu_describe (src/model.rs:207-209): the device and this build."""
        return lib().n3d_model_describe(self._h).decode()

    def run_offline(self, samples) -> RunOutput:
        """Model::run_offline (src/model.rs:232-234) on 16 kHz mono samples."""
        s = _f32(samples)
        o = _RunOutput()
        _check(lib().n3d_run_offline(self._h, _ptr(s), s.size, C.byref(o)))
        return _collect(o)

    def run_streaming(self, samples, mode: str) -> RunOutput:
        """Model::run_streaming (src/model.rs:313-336) in "low_latency",
        "very_low_latency" or "ultra_low_latency"."""
        s = _f32(samples)
        o = _RunOutput()
        _check(lib().n3d_run_streaming(self._h, _ptr(s), s.size, MODES[mode], C.byref(o)))
        return _collect(o)

    def run_batch(self, clips, mode: str = "offline") -> list[RunOutput]:
        """n3d_run_batch: many clips in one call; each result equals the clip's own run."""
        arrs = [_f32(c) for c in clips]
        n = len(arrs)
        ptrs = (_fp * max(n, 1))(*[_ptr(a) for a in arrs])
        lens = (_sz * max(n, 1))(*[a.size for a in arrs])
        outs = (_RunOutput * max(n, 1))()
        _check(lib().n3d_run_batch(self._h, MODES[mode], ptrs, lens, n, outs))
        return [_collect(outs[i]) for i in range(n)]

    def open_session(self, mode: str) -> "Session":
        """An incremental streaming session (n3d_session_open)."""
        h = C.c_void_p()
        _check(lib().n3d_session_open(self._h, MODES[mode], C.byref(h)))
        ss = Session(h, self)
        self._sessions.add(ss)
        return ss

    def sessions_push(self, sessions, pieces, close: bool = False) -> list[RunOutput]:
        """n3d_sessions_push: pieces[i] appended to sessions[i]; the new rows of each."""
        arrs = [_f32(p) for p in pieces]
        n = len(sessions)
        hs = (C.c_void_p * max(n, 1))(*[ss._h for ss in sessions])
        ptrs = (_fp * max(n, 1))(*[_ptr(a) for a in arrs])
        lens = (_sz * max(n, 1))(*[a.size for a in arrs])
        outs = (_RunOutput * max(n, 1))()
        _check(lib().n3d_sessions_push(hs, ptrs, lens, n, int(close), outs))
        return [_collect(outs[i]) for i in range(n)]

    def batch_out_frames(self, lens, mode: str = "offline") -> list[int]:
        """Logit rows each clip of the given lengths returns in `mode` (n3d_batch_out_frames)."""
        n = len(lens)
        arr = (_sz * max(n, 1))(*lens)
        out = (_sz * max(n, 1))()
        _check(lib().n3d_batch_out_frames(self._h, MODES[mode], arr, n, out))
        return [int(out[i]) for i in range(n)]

    def run_batch_device(self, mode: str, d_audio: int, offsets, lens, d_logits: int, out_offsets) -> None:
        """n3d_run_batch_device: clips already in device memory (d_audio at `offsets`),
        logits written to device memory at `out_offsets` rows of d_logits."""
        n = len(lens)
        _check(lib().n3d_run_batch_device(self._h, MODES[mode], C.c_void_p(d_audio), (_sz * max(n, 1))(*offsets),
                                          (_sz * max(n, 1))(*lens), n, C.c_void_p(d_logits),
                                          (_sz * max(n, 1))(*out_offsets)))

    # ---- profiling (device time per kernel class, CUDA events on the model's stream)
    def profile_enable(self, on: bool = True) -> None:
        """Time every launch of later runs with CUDA events (n3d_profile_enable; resets)."""
        _check(lib().n3d_profile_enable(self._h, int(on)))

    def profile_read(self) -> dict:
        """Per kernel class: launches, device ms, algorithmic FLOP and bytes (n3d_profile_read)."""
        buf = (_KernelStats * 16)()
        n = lib().n3d_profile_read(self._h, buf, 16)
        return {buf[i].name.decode(): dict(launches=int(buf[i].launches), ms=buf[i].ms, flops=buf[i].flops,
                                           bytes=buf[i].bytes) for i in range(n)}

    def step_timing_enable(self, on: bool = True) -> None:
        """Record the device time of each chunk-loop step of later runs (n3d_step_timing_enable)."""
        _check(lib().n3d_step_timing_enable(self._h, int(on)))

    def step_times(self) -> list[float]:
        """The recorded chunk-loop step times, ms (n3d_step_times)."""
        n = lib().n3d_step_times(self._h, None, 0)
        buf = (C.c_double * max(n, 1))()
        lib().n3d_step_times(self._h, buf, n)
        return [buf[i] for i in range(n)]

    # ---- stages (GpuEngine, src/gpu_engine.rs)
    def log_mel(self, samples, centered: bool = True) -> np.ndarray:
        """log_mel (src/mel.rs:160-225) on the device: [frames, 128]."""
        s = _f32(samples)
        cap = (s.size // 160 + 2) * 128
        out = np.zeros(max(cap, 1), np.float32)
        frames = _sz()
        _check(lib().n3d_log_mel(self._h, _ptr(s), s.size, int(centered), _ptr(out), out.size, C.byref(frames)))
        return out[: frames.value * 128].reshape(frames.value, 128)

    def embed_range(self, mel, num_frames: int, lo: int, hi: int) -> np.ndarray:
        """GpuEngine::embed_mel_range (src/gpu_engine.rs:1335-1379): groups lo..hi."""
        m = _f32(mel) if num_frames else np.zeros(1, np.float32)
        out = np.zeros((hi - lo) * self.hidden_size, np.float32)
        _check(lib().n3d_embed_range(self._h, _ptr(m), num_frames, lo, hi, _ptr(out)))
        return out.reshape(hi - lo, self.hidden_size)

    def forward_embeds(self, embeds, valid: int) -> np.ndarray:
        """GpuEngine::forward_embeds (src/gpu_engine.rs:1506): the tower over a window
        whose first `valid` frames are unmasked."""
        e = _f32(embeds)
        frames = e.size // self.hidden_size
        out = np.zeros(e.size, np.float32)
        _check(lib().n3d_forward_embeds(self._h, _ptr(e), frames, valid, _ptr(out)))
        return out.reshape(frames, self.hidden_size)

    def head_forward(self, encoder_out, frames: int) -> np.ndarray:
        """GpuEngine::head_forward (src/gpu_engine.rs:1695): [frames * 8, speakers] logits."""
        e = _f32(encoder_out)
        out = np.zeros(frames * 8 * self.num_speakers, np.float32)
        _check(lib().n3d_head_forward(self._h, _ptr(e), frames, _ptr(out)))
        return out.reshape(frames * 8, self.num_speakers)

    def forward_window(self, embeds, valid: int) -> np.ndarray:
        """GpuEngine::forward_window (src/gpu_engine.rs:1516-1520): tower and head."""
        e = _f32(embeds)
        frames = e.size // self.hidden_size
        out = np.zeros(frames * 8 * self.num_speakers, np.float32)
        _check(lib().n3d_forward_window(self._h, _ptr(e), frames, valid, _ptr(out)))
        return out.reshape(frames * 8, self.num_speakers)


class Session:
    """A streaming session: push audio as it arrives, get each completed chunk's logits
    rows; close() runs the final chunk.  Concatenated, the rows equal run_streaming."""

    def __init__(self, handle, model: Model):
        self._h = handle
        self._model = model  # the model outlives its sessions

    def push(self, samples) -> RunOutput:
        """Append samples; the logit rows of every chunk they complete."""
        s = _f32(samples)
        o = _RunOutput()
        _check(lib().n3d_session_push(self._h, _ptr(s), s.size, C.byref(o)))
        return _collect(o)

    def close(self) -> RunOutput:
        """Run the final centred chunk; its rows, and the run's totals."""
        o = _RunOutput()
        _check(lib().n3d_session_close(self._h, C.byref(o)))
        return _collect(o)

    def free(self) -> None:
        """Release the session's device state (n3d_session_free)."""
        if self._h:
            lib().n3d_session_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def extract_speaker_dict(logits, num_frames: int, num_speakers: int, duration: float, mask=None,
                         threshold: float = 0.5) -> list[Segment]:
    """extract_speaker_dict (src/segments.rs:70-109)."""
    lg = _f32(logits) if num_frames and num_speakers else np.zeros(1, np.float32)
    m = np.ascontiguousarray(mask, dtype=np.uint8) if mask is not None else None
    out = C.POINTER(_Segment)()
    n = _sz()
    _check(lib().n3d_extract_speaker_dict(_ptr(lg), num_frames, num_speakers, duration,
                                          m.ctypes.data if m is not None else None, threshold, C.byref(out),
                                          C.byref(n)))
    segs = [Segment(out[i].start, out[i].end, int(out[i].speaker)) for i in range(n.value)]
    lib().n3d_segments_free(out)
    return segs


def activity_stats(logits, num_frames: int, num_speakers: int, mask=None, threshold: float = 0.5):
    """activity_stats (src/segments.rs:113-141): (speech percentage, per-speaker frame counts)."""
    lg = _f32(logits) if num_frames and num_speakers else np.zeros(1, np.float32)
    m = np.ascontiguousarray(mask, dtype=np.uint8) if mask is not None else None
    per = (_sz * max(num_speakers, 1))()
    pct = lib().n3d_activity_stats(_ptr(lg), num_frames, num_speakers, m.ctypes.data if m is not None else None,
                                   threshold, per)
    return pct, [int(per[i]) for i in range(num_speakers)]


def frame_duration(hop_length: int = 160, sampling_rate: int = 16000) -> float:
    """frame_duration (src/segments.rs:36-38): seconds per logit row."""
    return lib().n3d_frame_duration(hop_length, sampling_rate)


def linear(device: int, d_x: int, rows: int, cols: int, d_w: int, out: int, d_bias: int | None, d_y: int) -> None:
    """tensor::linear on device pointers (fp16-split tcgen05 GEMM)."""
    _check(lib().n3d_linear(device, d_x, rows, cols, d_w, out, d_bias, d_y))


def linear_noalloc(device: int, d_x: int, rows: int, cols: int, d_w: int, out: int, d_bias: int | None, d_y: int,
                   stream: int | None = None) -> None:
    """tensor::linear for callers that cannot allocate device memory: the operand
    split uses the library's fixed 16 MiB device scratch (limit: rows*cols +
    out*cols at most 4194240; calls overlapping on the GPU race)."""
    _check(lib().n3d_linear_noalloc(device, d_x, rows, cols, d_w, out, d_bias, d_y, stream))


def layer_norm(device: int, d_x: int, rows: int, cols: int, d_w: int, d_b: int, d_y: int) -> None:
    """tensor::layer_norm (src/tensor.rs:97-110) on device pointers; cols 512 or 1024."""
    _check(lib().n3d_layer_norm(device, d_x, rows, cols, d_w, d_b, d_y))


def attention(device: int, d_q: int, d_k: int, d_v: int, seq: int, heads: int, head_dim: int, valid: int,
              d_out: int, rope: bool = True, theta: float = 10000.0) -> None:
    """RoPE then masked attention (src/encoder.rs:163-185, 281-329) on device pointers."""
    _check(lib().n3d_attention(device, d_q, d_k, d_v, seq, heads, head_dim, valid, int(rope), theta, d_out))


def cache_compress(device: int, cfg: CacheConfig, probs, frames: int, embeds=None, hidden: int = 0, silence=None):
    """SpeakerCache::trace_compress / compress (src/streaming.rs:353-482) on the device,
    through the chunk loop's own selection and gather code.  Returns (picked, sentinel)
    and, when `embeds` is given, also the gathered (embeds [L, hidden], probs [L, ns])."""
    p = _f32(probs)
    L = cfg.speaker_cache_length
    picked = (_sz * max(L, 1))()
    sentinel, count = _sz(), _sz()
    ns = cfg.num_speakers
    if embeds is not None:
        e, sil = _f32(embeds), _f32(silence)
        oe = np.empty(L * hidden, np.float32)
        op = np.empty(L * ns, np.float32)
        _check(lib().n3d_cache_compress(device, C.byref(cfg), _ptr(p), frames, e.ctypes.data, hidden, sil.ctypes.data,
                                        picked, C.byref(sentinel), C.byref(count), oe.ctypes.data, op.ctypes.data))
    else:
        _check(lib().n3d_cache_compress(device, C.byref(cfg), _ptr(p), frames, None, 0, None, picked,
                                        C.byref(sentinel), C.byref(count), None, None))
    n = count.value
    out = np.array(picked[:n], np.int64), sentinel.value
    if embeds is not None:
        return out + (oe[:n * hidden].reshape(n, hidden), op[:n * ns].reshape(n, ns))
    return out


def bench_linear(device: int, rows: int, cols: int, out: int, iters: int = 20) -> float:
    """Mean device ms of one launch of n3d_linear's GEMM on resident synthetic operands."""
    ms = C.c_double()
    _check(lib().n3d_bench_linear(device, rows, cols, out, iters, C.byref(ms)))
    return ms.value


def bench_attention(device: int, seq: int, heads: int, head_dim: int, iters: int = 20) -> float:
    """Mean device ms of one attention launch over all `seq` keys on resident operands."""
    ms = C.c_double()
    _check(lib().n3d_bench_attention(device, seq, heads, head_dim, iters, C.byref(ms)))
    return ms.value


def bench_layer_norm(device: int, rows: int, cols: int, iters: int = 20) -> float:
    """Mean device ms of one LayerNorm launch (fp32 in and out)."""
    ms = C.c_double()
    _check(lib().n3d_bench_layer_norm(device, rows, cols, iters, C.byref(ms)))
    return ms.value


def selftest_wait_timeout(device: int, limit_ms: float) -> tuple[int, str, float]:
    """Run one bounded device wait on a flag nothing sets (n3d_selftest_wait_timeout).
    Returns (status, message, waited_ms); the status is Timeout when the wait gave up."""
    w = C.c_double()
    st = lib().n3d_selftest_wait_timeout(device, limit_ms, C.byref(w))
    return st, lib().n3d_last_error().decode(), w.value

"""The oracle's chunk loop against a Python restatement of the reference's
(src/model.rs:236-365, 371-538; SpeakerCache::update and num_popped,
src/streaming.rs:202-284), built on the oracle's own stage functions.  Those stages
are checked separately against float64 restatements and the reference's known answers.

What this pins is the loop's data movement:
* offline: the zero mel row appended after the valid frames, the spans of
  chunk_length groups plus right context, and the per-group mask;
* streaming: the chunk geometry and the per-chunk mel and embeddings;
* each window as cache ++ FIFO ++ chunk ++ look-ahead, its valid count, and the logit
  rows kept;
* FIFO append and pop, and cache probabilities taken from the step until the first
  compression and from the cache after it;
* the final truncation.
The loop moves data and does no arithmetic of its own, so the bar is bit for bit: logits
and every RunOutput field."""

import numpy as np
import pytest

import oracle
import synth

MODES = {"low_latency": 0, "very_low_latency": 1, "ultra_low_latency": 2}


@pytest.fixture(scope="module")
def tiny(tiny_checkpoint_dir, tiny_oracle):
    silence = synth.load_safetensors(tiny_checkpoint_dir + "/model.safetensors")["silence_embeds"]
    return tiny_oracle, np.asarray(silence, np.float32)


class Cache:
    """SpeakerCache (src/streaming.rs:180-284) over the oracle's pool_probs and compress."""

    def __init__(self, cc, hidden, silence):
        self.cc, self.hidden, self.silence = cc, hidden, silence
        self.embeds = np.zeros((0, hidden), np.float32)
        self.probs = np.zeros((0, cc.num_speakers), np.float32)
        self.fifo = np.zeros((0, hidden), np.float32)
        self.compressed = False

    def num_popped(self, n):
        if n <= self.cc.fifo_length:
            return 0
        return min(max(self.cc.update_period, n - self.cc.fifo_length), n)

    def update(self, window, logits, n_chunk, step_mask):
        cc, ns, sub = self.cc, self.cc.num_speakers, self.cc.subsampling_factor
        nin = window.shape[0]
        probs = oracle.pool_probs(cc, logits.reshape(-1), nin * sub, step_mask).reshape(-1, ns)
        n_cache, start = self.embeds.shape[0], self.embeds.shape[0] + self.fifo.shape[0]
        fifo = np.concatenate([self.fifo, window[start:start + n_chunk]])
        popped = self.num_popped(fifo.shape[0])
        if popped > 0:
            fifo_probs = probs[n_cache:n_cache + fifo.shape[0]]
            stored = self.probs if self.compressed else probs[:n_cache]
            ce = np.concatenate([self.embeds, fifo[:popped]])
            cp = np.concatenate([stored, fifo_probs[:popped]])
            fifo = fifo[popped:]
            if ce.shape[0] > cc.speaker_cache_length:
                e, p = oracle.compress(cc, self.hidden, ce.reshape(-1), cp.reshape(-1), ce.shape[0], self.silence)
                ce, cp = e.reshape(-1, self.hidden), p.reshape(-1, ns)
                self.compressed = True
            self.embeds, self.probs = ce, cp
        self.fifo = fifo


def _step(om, cache, embeds, mask, n_chunk, cap, out):
    sub, ns = om.c.sub, om.c.num_speakers
    cached = cache.embeds.shape[0] + cache.fifo.shape[0]
    window = np.concatenate([cache.embeds, cache.fifo, embeds]).astype(np.float32)
    step_mask = [True] * cached + list(mask)
    valid = sum(step_mask)
    logits = om.head_forward(om.forward_embeds(window, valid), window.shape[0])
    cache.update(window, logits, n_chunk, step_mask)
    s, e = cached * sub, (cached + n_chunk) * sub
    out.append(logits[s:s + min(e - s, cap)])


def _run_offline(om, silence, samples):
    sub, fe = om.c.sub, om.proc["feature_extractor"]
    valid = oracle.frame_count(len(samples), fe, True)
    mel = np.zeros((valid + 1, fe["feature_size"]), np.float32)  # the over-emitted frame, zeroed
    mel[:valid] = om.log_mel(samples, True)[:valid]
    groups = -(-(valid + 1) // sub)
    cache = Cache(oracle.cache_cfg_from_model(om.cfg, offline=True), om.c.hidden, silence)
    out, n_chunks, start = [], 0, 0
    while start < groups:
        end = min(start + om.cfg["chunk_length"], groups)
        lo, hi = start, min(end + om.cfg["chunk_right_context"], groups)
        embeds = om.embed_range(mel, valid + 1, lo, hi)
        _step(om, cache, embeds, [g * sub < valid for g in range(lo, hi)], end - start, 1 << 62, out)
        n_chunks += 1
        start += om.cfg["chunk_length"]
    logits = np.concatenate(out)[:valid + 1]
    return logits, n_chunks, cache


def _run_streaming(om, silence, samples, mode):
    sub, fe = om.c.sub, om.proc["feature_extractor"]
    cl, rc = om.proc["streaming_modes"][mode]
    hop, n_fft, win = fe["hop_length"], fe["n_fft"], fe["win_length"]
    mel_chunk, mel_step = (cl + rc) * sub, cl * sub
    first, per_chunk = (mel_chunk - 1) * hop + win // 2, mel_chunk * hop + win
    chunks = [(samples[:min(first, len(samples))], True, rc)]
    idx = mel_step
    start = idx * hop - n_fft // 2
    while start + per_chunk <= len(samples):
        chunks.append((samples[start:start + per_chunk], False, rc))
        idx += mel_step
        start = idx * hop - n_fft // 2
    chunks.append((samples[min(start, len(samples)):], True, 0))
    cache = Cache(oracle.cache_cfg_from_model(om.cfg, offline=False), om.c.hidden, silence)
    out = []
    for audio, centered, la in chunks:
        nm = oracle.frame_count(len(audio), fe, centered)
        mel = om.log_mel(audio, centered)
        groups = -(-nm // sub)
        if groups < la:
            return None  # too short for the look-ahead (the oracle reports it)
        embeds = om.embed_range(mel, nm, 0, groups)
        _step(om, cache, embeds, [True] * groups, groups - la, nm, out)
    return np.concatenate(out), len(chunks), cache


@pytest.mark.parametrize("seconds", [0.3, 2.2, 7.5, 19.3])
def test_offline_loop(tiny, seconds):
    om, silence = tiny
    a = synth.clip(21, seconds, 3)
    got = om.run_offline(a)
    logits, n_chunks, cache = _run_offline(om, silence, a)
    assert np.array_equal(got["logits"], logits)
    assert (got["num_frames"], got["num_chunks"]) == (logits.shape[0], n_chunks)
    assert (got["cache_compressed"], got["cache_frames"], got["fifo_frames"]) == \
        (cache.compressed, cache.embeds.shape[0], cache.fifo.shape[0])
    assert cache.compressed == (seconds > 7)  # the two long clips reach compression


@pytest.mark.parametrize("mode", list(MODES))
@pytest.mark.parametrize("seconds", [1.1, 6.0, 15.7])
def test_streaming_loop(tiny, mode, seconds):
    om, silence = tiny
    a = synth.clip(22, seconds, 3)
    got = om.run_streaming(a, mode)
    logits, n_chunks, cache = _run_streaming(om, silence, a, mode)
    assert np.array_equal(got["logits"], logits)
    assert (got["num_frames"], got["num_chunks"]) == (logits.shape[0], n_chunks)
    assert (got["cache_compressed"], got["cache_frames"], got["fifo_frames"]) == \
        (cache.compressed, cache.embeds.shape[0], cache.fifo.shape[0])
    assert cache.compressed or seconds < 6  # the long runs exercise compression

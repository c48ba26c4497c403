"""The oracle's embedder, encoder tower and head against an independent float64
restatement in numpy of the reference's code (CPU only).

The known-answer tests pin the oracle's individual operations; these check how it
composes them, on a 2-layer model whose weights, biases and LayerNorm parameters are
all random (the synthetic checkpoint's zero biases and unit gains would hide a missing
term):
* the embedder's 8-frame stacking with zero padding past the last frame
  (src/encoder.rs:126-146);
* the tower: input LayerNorm, RoPE tables (src/encoder.rs:163-185), pre-norm blocks
  with masked-key attention and both residuals (src/encoder.rs:236-329), final
  LayerNorm;
* the head: projection, k=3 convolution with one zero frame each side, sub-pixel
  reshape, ReLU, dense, ReLU, out_proj (src/head.rs:92-157).
Tolerances are fp32-vs-float64 rounding, far inside the reference's stage gates
(encoder 1e-2, head 2e-2)."""

import copy

import numpy as np
import pytest

import oracle
import synth

P = "model.audio_tower"


@pytest.fixture(scope="module")
def model():
    cfg = copy.deepcopy(synth.MODEL_CONFIG)
    cfg["audio_config"]["num_hidden_layers"] = 2
    rng = np.random.default_rng(77)
    w = {}
    for name, shape, kind in synth.tensor_specs(cfg):
        if kind == "g":
            w[name] = (1.0 + 0.2 * rng.standard_normal(shape)).astype(np.float32)
        else:
            std = 0.05 if kind == "w" else 0.1
            w[name] = (std * rng.standard_normal(shape)).astype(np.float32)
    return oracle.OracleModel(cfg, synth.PROCESSOR_CONFIG, w), cfg, {k: v.astype(np.float64) for k, v in w.items()}


def _ln(x, g, b):
    mu = x.mean(-1, keepdims=True)
    var = ((x - mu) ** 2).mean(-1, keepdims=True)
    return (x - mu) / np.sqrt(var + 1e-5) * g + b


def _rope(seq, hd, theta):
    inv = (1.0 / theta ** (2.0 * np.arange(hd // 2) / hd)).astype(np.float32)  # f64 -> f32, as the reference
    ang = np.arange(seq, dtype=np.float32)[:, None] * inv[None, :]             # f32 product
    ang = np.concatenate([ang, ang], 1).astype(np.float64)
    return np.cos(ang), np.sin(ang)


def _tower64(cfg, w, embeds, valid):
    a = cfg["audio_config"]
    h, nh = a["hidden_size"], a["num_attention_heads"]
    hd = h // nh
    S = embeds.shape[0]
    x = _ln(embeds, w[f"{P}.input_layer_norm.weight"], w[f"{P}.input_layer_norm.bias"])
    cos, sin = _rope(S, hd, a["rope_parameters"]["rope_theta"])

    def rope(t):
        t = t.reshape(S, nh, hd)
        half = hd // 2
        rot = np.concatenate([-t[..., half:], t[..., :half]], -1)
        return t * cos[:, None, :] + rot * sin[:, None, :]

    for i in range(a["num_hidden_layers"]):
        b = f"{P}.layers.{i}"
        n1 = _ln(x, w[f"{b}.layer_norm1.weight"], w[f"{b}.layer_norm1.bias"])
        q = rope(n1 @ w[f"{b}.self_attn.q_proj.weight"].T)
        k = rope(n1 @ w[f"{b}.self_attn.k_proj.weight"].T)
        v = (n1 @ w[f"{b}.self_attn.v_proj.weight"].T).reshape(S, nh, hd)
        s = np.einsum("qhd,khd->hqk", q, k)[:, :, :valid] / np.sqrt(hd)
        p = np.exp(s - s.max(-1, keepdims=True))
        p /= p.sum(-1, keepdims=True)
        ctx = np.einsum("hqk,khd->qhd", p, v[:valid]).reshape(S, h)
        x = x + ctx @ w[f"{b}.self_attn.o_proj.weight"].T + w[f"{b}.self_attn.o_proj.bias"]
        n2 = _ln(x, w[f"{b}.layer_norm2.weight"], w[f"{b}.layer_norm2.bias"])
        from scipy.special import erf

        f1 = n2 @ w[f"{b}.mlp.fc1.weight"].T + w[f"{b}.mlp.fc1.bias"]
        f1 = 0.5 * f1 * (1.0 + erf(f1 / np.sqrt(2.0)))
        x = x + f1 @ w[f"{b}.mlp.fc2.weight"].T + w[f"{b}.mlp.fc2.bias"]
    return _ln(x, w[f"{P}.layer_norm.weight"], w[f"{P}.layer_norm.bias"])


def _head64(cfg, w, enc):
    hh, up = cfg["head_config"]["hidden_size"], cfg["audio_config"]["subsampling_factor"]
    S = enc.shape[0]
    proj = enc @ w["model.proj.weight"].T + w["model.proj.bias"]
    pad = np.concatenate([np.zeros((1, hh)), proj, np.zeros((1, hh))])
    cw = w["model.upsampler.conv.weight"]  # [hh * up, hh, 3]
    conv = sum(pad[j:j + S] @ cw[:, :, j].T for j in range(3)) + w["model.upsampler.conv.bias"]
    shaped = conv.reshape(S * up, hh)       # row t*up + j is sub-pixel j of frame t
    r1 = np.maximum(shaped, 0)
    d = np.maximum(r1 @ w["classifier.dense.weight"].T + w["classifier.dense.bias"], 0)
    return d @ w["classifier.out_proj.weight"].T + w["classifier.out_proj.bias"]


@pytest.mark.parametrize("num_frames,lo,hi", [(100, 0, 13), (100, 5, 13), (3, 0, 1), (64, 2, 8)])
def test_embedder(model, num_frames, lo, hi):
    om, cfg, w = model
    rng = np.random.default_rng(num_frames + lo)
    mel = rng.standard_normal((num_frames, 128)).astype(np.float32)
    got = om.embed_range(mel, num_frames, lo, hi)
    padded = np.zeros(((hi + 1) * 8, 128))
    padded[:num_frames] = mel
    stacked = padded[lo * 8:hi * 8].reshape(hi - lo, 8 * 128)  # frames past num_frames stay zero
    want = stacked @ w[f"{P}.embedder.projection.weight"].T
    assert np.abs(got - want).max() < 1e-4


@pytest.mark.parametrize("S,valid", [(37, 37), (37, 29), (1, 1), (96, 64)])
def test_tower(model, S, valid):
    om, cfg, w = model
    e = np.random.default_rng(S * 100 + valid).standard_normal((S, 512)).astype(np.float32)
    got = om.forward_embeds(e, valid)
    want = _tower64(cfg, w, e.astype(np.float64), valid)
    assert np.abs(got - want).max() < 2e-4


@pytest.mark.parametrize("S", [1, 2, 23])
def test_head(model, S):
    om, cfg, w = model
    enc = np.random.default_rng(S).standard_normal((S, 512)).astype(np.float32)
    got = om.head_forward(enc, S)
    want = _head64(cfg, w, enc.astype(np.float64))
    assert got.shape == want.shape
    assert np.abs(got - want).max() < 1e-4 * max(1.0, np.abs(want).max())

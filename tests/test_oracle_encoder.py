"""The speech-tokenizer encoder restatement in the oracle (the voice-clone
path's Qwen3TtsAudioCodecEncoder, codec/network/encoder.rs; built as
codec/config.rs:136-346 builds it).  The reference ships no golden vectors
for the encoder, so its numerics are unpinned; these tests pin what the
reference's structure fixes exactly:

* frame counts from the conv1d_padding rules (conv.rs:44-64) for ragged
  sample counts;
* the residual vector quantizer (encoder.rs:319-368, codebook.rs:4-41) on a
  hand-built codebook: exact hits, first index on ties, clamped cluster usage,
  greedy residuals;
* causality: every convolution pads on the left and the transformer masks
  future keys, so a prefix of the audio encodes to the same codes except the
  last frame, whose stride windows the prefix cuts (bit-exact, same order of
  operations);
* semantic codes come first, and asking for fewer codebooks returns a prefix
  of the rows;
* the hidden state the quantizers read matches an independent float64 numpy
  restatement of the backbone, transformer and downsample (1e-5 relative).
"""
import numpy as np
import pytest

import oracle as O
import synthetic as S


@pytest.fixture(scope="module")
def enc():
    cfg = S.CodecEncoderConfig().small()
    return cfg, O.OracleCodecEncoder(cfg, S.make_codec_encoder_weights(cfg, seed=0))


def _wave(n, seed=1):
    g = np.random.default_rng([seed, 5])
    t = np.arange(n, dtype=np.float32) / 24000.0
    return (0.3 * np.sin(2 * np.pi * 220.0 * t) + 0.05 * g.standard_normal(n)).astype(np.float32)


@pytest.mark.parametrize("n", [1, 11, 12, 13, 25, 2400, 2417])
def test_encoder_frames_and_code_range(enc, n):
    cfg, e = enc
    codes = e.encode(_wave(n))
    assert codes.shape == (cfg.n_q, cfg.frames(n))
    assert codes.min() >= 0 and codes.max() < cfg.codebook_size


def test_full_size_frame_rate():
    """Mimi-style shape: 960 samples per step, then stride 2: 12.5 frames per
    second at 24 kHz (1920 samples per frame, the decoder's rate)."""
    cfg = S.CodecEncoderConfig()
    assert cfg.frames(24000 * 4) == 50 and cfg.frames(1920 * 7) == 7


def test_encoder_is_causal(enc):
    cfg, e = enc
    wave = _wave(3000, seed=2)
    full = e.encode(wave)
    for n1 in (1000, 1210, 2999):
        part = e.encode(wave[:n1])
        T1 = part.shape[1]
        np.testing.assert_array_equal(part[:, :T1 - 1], full[:, :T1 - 1])


def test_fewer_codebooks_are_a_prefix(enc):
    cfg, e = enc
    wave = _wave(2400, seed=3)
    all_rows = e.encode(wave)
    for n_valid in (1, 2, cfg.n_q - 1):
        np.testing.assert_array_equal(e.encode(wave, n_valid=n_valid), all_rows[:n_valid])
    with pytest.raises(ValueError):
        e.encode(wave, n_valid=0)  # no semantic layer: the reference's InvalidInput


def test_rvq_encode_kat():
    """Two greedy layers on a hand-built codebook, against a numpy argmin
    (first index on ties): row 4 duplicates row 1, row 5 has zero usage
    (clamped to 1e-6, so its centroid sits 9e6 out and is never chosen)."""
    vq, cb = 4, 6
    embed_sum = np.array([[3, 0, 0, 0], [0, 1, 0, 0], [0, 0, 4, 0], [0, 0, 0, 1],
                          [0, 1, 0, 0], [9, 9, 9, 9]], np.float32)
    usage = np.array([1, 1, 2, 1, 1, 0], np.float32)
    layer2 = np.zeros((cb, vq), np.float32)
    layer2[:4] = np.eye(4, dtype=np.float32)  # e_0..e_3, then two zero rows
    x = np.array([[3, 0, 0, 9], [0, 1, 0, 9], [0, 0, 2.2, 9], [0.9, 0, 0, 9]], np.float32)  # [vq][T]
    codes, res = O.rvq_encode([embed_sum, layer2], [usage, np.ones(cb, np.float32)], x)
    r = x.astype(np.float64).copy()
    want = []
    for es, us in ((embed_sum, usage), (layer2, np.ones(cb, np.float32))):
        cent = es.astype(np.float64) / np.maximum(us, 1e-6)[:, None]
        d = ((r.T[:, None, :] - cent[None]) ** 2).sum(-1)
        ids = d.argmin(1)
        want.append(ids)
        r -= cent[ids].T
    np.testing.assert_array_equal(codes, np.array(want))
    np.testing.assert_allclose(res, r, atol=1e-5)
    assert codes[0, 1] == 1, "a tie goes to the first index"
    assert 5 not in codes[0], "a zero-usage row is never chosen"
    np.testing.assert_array_equal(codes[0], [0, 1, 2, 0])
    np.testing.assert_array_equal(codes[1], [3, 4, 4, 1])


def _conv_np(x, w, b, stride, edge):
    """conv1d_padding + pad_1d + Conv1d (conv.rs:44-83) in float64."""
    L, k = x.shape[1], w.shape[2]
    pt = max(k - stride, 0)
    padded = L + pt
    missing = max(k - padded, 0)
    extra = missing if missing > 0 else (stride - (padded - k) % stride) % stride
    xp = np.pad(x, ((0, 0), (pt, extra)), mode="edge" if edge else "constant")
    Lo = (L + pt + extra - k) // stride + 1
    win = xp[:, np.arange(Lo)[:, None] * stride + np.arange(k)[None]]  # [ci][Lo][k]
    y = np.einsum("oik,itk->ot", w, win)
    return y + (b[:, None] if b is not None else 0.0)


def encoder_hidden_numpy(cfg, w):
    from scipy.special import erf
    W = lambda n: w[n].astype(np.float64)
    elu = lambda v: np.where(v > 0, v, np.expm1(v))
    p = "encoder.encoder.layers"

    def run(wave):
        x = _conv_np(wave[None].astype(np.float64), W(f"{p}.0.conv.weight"), W(f"{p}.0.conv.bias"), 1, False)
        li = 1
        for r in reversed(cfg.upsampling_ratios):
            h = _conv_np(elu(x), W(f"{p}.{li}.conv_in.conv.weight"), W(f"{p}.{li}.conv_in.conv.bias"), 1, False)
            x = x + _conv_np(elu(h), W(f"{p}.{li}.conv_out.conv.weight"), W(f"{p}.{li}.conv_out.conv.bias"), 1,
                             False)
            x = _conv_np(elu(x), W(f"{p}.{li + 2}.conv.weight"), W(f"{p}.{li + 2}.conv.bias"), r, False)
            li += 3
        x = _conv_np(elu(x), W(f"{p}.{li + 1}.conv.weight"), W(f"{p}.{li + 1}.conv.bias"), 1, False)
        h = x.T  # [T][H]
        T, hd = h.shape[0], cfg.head_dim
        inv = cfg.theta ** (-np.arange(0, hd, 2) / hd)
        ang = np.arange(T)[:, None] * inv[None]
        cs, sn = np.cos(ang), np.sin(ang)

        def rope(v):  # [T][heads][hd], adjacent pairs
            a, b = v[..., 0::2], v[..., 1::2]
            out = np.empty_like(v)
            out[..., 0::2] = a * cs[:, None] - b * sn[:, None]
            out[..., 1::2] = b * cs[:, None] + a * sn[:, None]
            return out

        def ln(v, g, bb):
            mu = v.mean(-1, keepdims=True)
            var = ((v - mu) ** 2).mean(-1, keepdims=True)
            return (v - mu) / np.sqrt(var + cfg.norm_eps) * g + bb

        for l in range(cfg.n_layers):
            q_ = f"encoder.encoder_transformer.layers.{l}"
            n = ln(h, W(f"{q_}.input_layernorm.weight"), W(f"{q_}.input_layernorm.bias"))
            q = rope((n @ W(f"{q_}.self_attn.q_proj.weight").T).reshape(T, cfg.n_heads, hd))
            k = rope((n @ W(f"{q_}.self_attn.k_proj.weight").T).reshape(T, cfg.n_kv, hd))
            v = (n @ W(f"{q_}.self_attn.v_proj.weight").T).reshape(T, cfg.n_kv, hd)
            rep = cfg.n_heads // cfg.n_kv
            k, v = np.repeat(k, rep, axis=1), np.repeat(v, rep, axis=1)
            s = np.einsum("thd,shd->hts", q, k) / np.sqrt(hd)
            s = np.where(np.triu(np.ones((T, T), bool), 1)[None], -np.inf, s)
            a = np.exp(s - s.max(-1, keepdims=True))
            a /= a.sum(-1, keepdims=True)
            o = np.einsum("hts,shd->thd", a, v).reshape(T, -1) @ W(f"{q_}.self_attn.o_proj.weight").T
            h = h + o * W(f"{q_}.self_attn_layer_scale.scale")
            n = ln(h, W(f"{q_}.post_attention_layernorm.weight"), W(f"{q_}.post_attention_layernorm.bias"))
            f = n @ W(f"{q_}.mlp.fc1.weight").T
            f = 0.5 * f * (1 + erf(f / np.sqrt(2)))
            h = h + (f @ W(f"{q_}.mlp.fc2.weight").T) * W(f"{q_}.mlp_layer_scale.scale")
        return _conv_np(h.T, W("encoder.downsample.conv.weight"), None, 2, True)

    return run


@pytest.mark.parametrize("n", [500, 2417])
def test_encoder_hidden_matches_numpy(enc, n):
    """Backbone, causal transformer and edge-padded downsample against an
    independent float64 numpy restatement (f32 vs f64 arithmetic only)."""
    cfg, e = enc
    w = S.make_codec_encoder_weights(cfg, seed=0)
    wave = _wave(n, seed=4)
    got = e.hidden(wave)
    ref = encoder_hidden_numpy(cfg, w)(wave)
    assert got.shape == ref.shape == (cfg.hidden, cfg.frames(n))
    assert np.abs(got - ref).max() <= 1e-5 * np.abs(ref).max()

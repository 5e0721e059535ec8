"""The speaker encoder restatement in the oracle (the voice-clone path's
x-vector: speaker/infer/feature.rs for the log-mel front end, the ECAPA-TDNN
of speaker/network/*.rs).  No reference vectors exist for it, so the C
restatement is checked against a second, independent float64 numpy
restatement of the same reference code: the reflect-padded STFT (numpy's
FFT standing in for rustfft 6.4.1, both the plain DFT), the mel filters with
area normalisation, and the network (reflect-padded TDNN blocks,
Res2Net branch order, squeeze-excitation, attentive statistics pooling).
Tolerances cover the f32 vs f64 arithmetic only.
"""
import numpy as np
import pytest

import oracle as O
import synthetic as S


def _audio(n, seed=0):
    g = np.random.default_rng([seed, 9])
    t = np.arange(n) / 24000.0
    return (0.3 * np.sin(2 * np.pi * 440 * t) + 0.2 * np.sin(2 * np.pi * 3100 * t)
            + 0.05 * g.standard_normal(n)).astype(np.float32)


def mel_numpy(x, n_mels=128, sr=24000):
    n_fft, hop = 1024, 256
    pad = (n_fft - hop) // 2
    n = len(x)
    left = [x[min(i, n - 1)] for i in range(pad, 0, -1)]
    right = [x[min(max(n - 2 - i, 0), n - 1)] for i in range(pad)]
    p = np.concatenate([left, x, right]).astype(np.float64)
    frames = (len(p) - n_fft) // hop + 1
    win = 0.5 - 0.5 * np.cos(2 * np.pi * np.arange(n_fft) / n_fft)
    spec = np.stack([np.fft.rfft(p[t * hop:t * hop + n_fft] * win) for t in range(frames)])
    mag = np.sqrt(np.abs(spec) ** 2 + 1e-9)
    to_mel = lambda f: 2595.0 * np.log10(1.0 + f / 700.0)
    hz = 700.0 * (10 ** (np.linspace(to_mel(0.0), to_mel(sr / 2), n_mels + 2) / 2595.0) - 1.0)
    f = np.arange(n_fft // 2 + 1) * sr / n_fft
    fb = np.zeros((n_mels, len(f)))
    for m in range(n_mels):
        l, c, r = hz[m:m + 3]
        up = (f >= l) & (f <= c)
        dn = (f > c) & (f <= r)
        fb[m, up] = (f[up] - l) / (c - l)
        fb[m, dn] = (r - f[dn]) / (r - c)
        fb[m] *= 2.0 / (r - l)
    return np.log(np.maximum(mag @ fb.T, 1e-5)).T


@pytest.mark.parametrize("n", [256, 1000, 24000])
def test_mel_matches_numpy(n):
    x = _audio(n)
    got = O.speaker_mel(x)
    ref = mel_numpy(x)
    assert got.shape == ref.shape == (128, S.SpeakerEncoderConfig().frames(n))
    assert np.abs(got - ref).max() < 2e-4
    with pytest.raises(ValueError):
        O.speaker_mel(x[:255])


def _tdnn(x, w, b, dil):
    k = w.shape[2]
    total = dil * (k - 1)
    pl, pr = total // 2, total - total // 2
    T = x.shape[1]
    xp = np.concatenate([x[:, 1:pl + 1][:, ::-1], x, x[:, T - 1 - pr:T - 1][:, ::-1]], axis=1)
    y = np.stack([np.einsum("oi,it->ot", w[:, :, j], xp[:, j * dil:j * dil + T]) for j in range(k)]).sum(0)
    return np.maximum(y + b[:, None], 0.0)


def speaker_numpy(cfg, w, mel):
    p = "speaker_encoder"
    W = lambda n: w[f"{n}.weight"].astype(np.float64)
    B = lambda n: w[f"{n}.bias"].astype(np.float64)
    x = _tdnn(mel.astype(np.float64), W(f"{p}.blocks.0.conv"), B(f"{p}.blocks.0.conv"), cfg.enc_dilations[0])
    outs = []
    for i in range(1, 4):
        b = f"{p}.blocks.{i}"
        h = _tdnn(x, W(f"{b}.tdnn1.conv"), B(f"{b}.tdnn1.conv"), 1)
        ch = np.split(h, cfg.enc_res2net_scale, axis=0)
        ys, prev = [ch[0]], None
        for j in range(1, cfg.enc_res2net_scale):
            inp = ch[j] if j == 1 else ch[j] + prev
            prev = _tdnn(inp, W(f"{b}.res2net_block.blocks.{j - 1}.conv"),
                         B(f"{b}.res2net_block.blocks.{j - 1}.conv"), cfg.enc_dilations[i])
            ys.append(prev)
        h = _tdnn(np.concatenate(ys), W(f"{b}.tdnn2.conv"), B(f"{b}.tdnn2.conv"), 1)
        s = h.mean(1)
        z = np.maximum(W(f"{b}.se_block.conv1")[:, :, 0] @ s + B(f"{b}.se_block.conv1"), 0.0)
        sc = 1.0 / (1.0 + np.exp(-(W(f"{b}.se_block.conv2")[:, :, 0] @ z + B(f"{b}.se_block.conv2"))))
        x = h * sc[:, None] + x
        outs.append(x)
    h = _tdnn(np.concatenate(outs), W(f"{p}.mfa.conv"), B(f"{p}.mfa.conv"), cfg.enc_dilations[4])
    T = h.shape[1]
    mu = h.mean(1)
    sd = np.sqrt(np.maximum((h ** 2).mean(1) - mu ** 2, 0.0) + 1e-5)
    a = np.tanh(_tdnn(np.concatenate([h, np.repeat(mu[:, None], T, 1), np.repeat(sd[:, None], T, 1)]),
                      W(f"{p}.asp.tdnn.conv"), B(f"{p}.asp.tdnn.conv"), 1))
    logits = W(f"{p}.asp.conv")[:, :, 0] @ a + B(f"{p}.asp.conv")[:, None]
    att = np.exp(logits - logits.max(1, keepdims=True))
    att /= att.sum(1, keepdims=True)
    wm = (h * att).sum(1)
    ws = np.sqrt(np.maximum((h ** 2 * att).sum(1) - wm ** 2, 0.0) + 1e-5)
    return W(f"{p}.fc")[:, :, 0] @ np.concatenate([wm, ws]) + B(f"{p}.fc")


@pytest.fixture(scope="module")
def small_speaker():
    cfg = S.SpeakerEncoderConfig().small()
    w = S.make_speaker_weights(cfg, seed=0)
    return cfg, w, O.OracleSpeaker(cfg, w)


@pytest.mark.parametrize("T", [5, 40])
def test_speaker_network_matches_numpy(small_speaker, T):
    cfg, w, sp = small_speaker
    mel = np.random.default_rng([T, 4]).standard_normal((cfg.mel_dim, T)).astype(np.float32)
    got = sp.forward(mel)
    ref = speaker_numpy(cfg, w, mel)
    assert got.shape == (cfg.enc_dim,)
    assert np.abs(got - ref).max() <= 1e-5 * max(1.0, np.abs(ref).max())


def test_speaker_embed_is_mel_then_network(small_speaker):
    cfg, w, sp = small_speaker
    x = _audio(6000, seed=3)
    mel = O.speaker_mel(x, n_mels=cfg.mel_dim)
    np.testing.assert_array_equal(sp.embed(x), sp.forward(mel))
    with pytest.raises(ValueError):
        sp.forward(mel[:, :2])  # a k5 TDNN needs 3 frames for its reflect padding

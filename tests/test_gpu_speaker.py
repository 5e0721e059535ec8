"""ECAPA-TDNN speaker encoder of the voice-clone path on the device
(q3t_speaker_*, the reference's LoadedQwen3TtsSpeakerEncoder::
encode_embedding, speaker/infer/mod.rs:11-20) against the oracle's
restatement (oracle.c orc_speaker_mel / orc_speaker_forward), same seeded
weights and audio:

* log-mel features: the device takes the 1024-point DFT as direct f64 sums,
  the oracle as a radix-2 FFT (both f64, both cast to f32 before the
  magnitude); max abs difference of the logs <= 1e-4;
* x-vector: relative L2 error <= 1e-4 against the f32 oracle (summation
  order and fused multiply-adds only), for clips of 10 frames to 3 s;
* clips too short for the TDNN blocks' reflect padding fail on both sides
  (INVALID_INPUT here, the oracle's error there);
* repeat calls are bit-identical;
* the reduced and the full-size (512-channel, 1024-dim) encoder.
"""
import numpy as np
import pytest

import oracle as O
import q3t
import synthetic as S

pytestmark = pytest.mark.gpu


def _audio(n, seed=0):
    g = np.random.default_rng([seed, 9])
    t = np.arange(n) / 24000.0
    return (0.3 * np.sin(2 * np.pi * 440 * t) + 0.2 * np.sin(2 * np.pi * 3100 * t)
            + 0.05 * g.standard_normal(n)).astype(np.float32)


def _rel(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module")
def small():
    cfg = S.SpeakerEncoderConfig().small()
    w = S.make_speaker_weights(cfg, seed=0)
    e = q3t.SpeakerEncoder(cfg, w)
    yield cfg, e, O.OracleSpeaker(cfg, w)
    e.close()


@pytest.mark.parametrize("n", [256, 1000, 7001, 24000])
def test_small_mel_matches_oracle(small, n):
    cfg, e, _ = small
    x = _audio(n, seed=n)
    got, ref = e.mel(x), O.speaker_mel(x, n_mels=cfg.mel_dim)
    assert got.shape == ref.shape == (cfg.mel_dim, cfg.frames(n))
    assert np.abs(got - ref).max() <= 1e-4


@pytest.mark.parametrize("n", [2560, 7001, 24000, 72000])
def test_small_embedding_matches_oracle(small, n):
    cfg, e, oe = small
    x = _audio(n, seed=n + 1)
    got, ref = e.embed(x), oe.embed(x)
    assert got.shape == ref.shape == (cfg.enc_dim,)
    assert np.isfinite(got).all()
    assert _rel(got, ref) <= 1e-4, _rel(got, ref)
    np.testing.assert_array_equal(e.embed(x), got)


def test_small_too_short_clips_are_rejected(small):
    cfg, e, oe = small
    # 4 frames: block 3's Res2Net convs (kernel 3, dilation 4) need 5
    x = _audio(1100, seed=3)
    assert cfg.frames(len(x)) == 4
    with pytest.raises(ValueError):
        oe.embed(x)
    with pytest.raises(q3t.Q3TError) as err:
        e.embed(x)
    assert err.value.status == q3t.INVALID_INPUT
    with pytest.raises(q3t.Q3TError) as err:
        e.embed(x[:255])
    assert err.value.status == q3t.INVALID_INPUT
    # the encoder still works after the rejections
    y = _audio(4000, seed=4)
    assert _rel(e.embed(y), oe.embed(y)) <= 1e-4


def test_full_size_speaker_encoder_matches_oracle():
    cfg = S.SpeakerEncoderConfig()
    w = S.make_speaker_weights(cfg, seed=0)
    e = q3t.SpeakerEncoder(cfg, w)
    try:
        oe = O.OracleSpeaker(cfg, w)
        x = _audio(72000, seed=7)
        mel, omel = e.mel(x), O.speaker_mel(x)
        assert np.abs(mel - omel).max() <= 1e-4
        got, ref = e.embed(x), oe.embed(x)
        rel = _rel(got, ref)
        print(f"full-size speaker encoder, 3 s: x-vector rel L2 {rel:.2e}")
        assert rel <= 1e-4, rel
    finally:
        e.close()

"""Speech-tokenizer encoder of the voice-clone path on the device
(q3t_codec_encoder_*, the reference's Qwen3TtsAudioCodecEncoder::
encode_reference_prefix, codec/network/encoder.rs:121-136) against the
oracle's restatement (oracle.c orc_codec_encode), same seeded weights and
audio:

* frame counts for ragged sample counts (conv.rs:44-64 lengths);
* the hidden the quantizers read (backbone, causal transformer, stride-2
  edge-padded downsample): relative L2 error <= 1e-4 against the f32 oracle
  (the two differ only in summation order and the math library's last bits);
* codes: the residual VQ picks the nearest centroid, so a near-tie can flip
  under that noise and take the rest of its frame's residual path with it;
  every semantic code and >= 98 % of all codes must equal the oracle's;
* causality on the device: a prefix of the audio encodes to the same codes
  except its last frame, bit for bit (the device path sums in the same order
  for every length);
* the reduced and the full-size (Mimi-shaped, 2 s of audio) encoder.
"""
import numpy as np
import pytest

import oracle as O
import q3t
import synthetic as S

pytestmark = pytest.mark.gpu


def _wave(n, seed=1):
    g = np.random.default_rng([seed, 5])
    t = np.arange(n, dtype=np.float32) / 24000.0
    return (0.3 * np.sin(2 * np.pi * 220.0 * t) + 0.05 * g.standard_normal(n)).astype(np.float32)


@pytest.fixture(scope="module")
def small():
    cfg = S.CodecEncoderConfig().small()
    w = S.make_codec_encoder_weights(cfg, seed=0)
    e = q3t.CodecEncoder(cfg, w)
    yield cfg, e, O.OracleCodecEncoder(cfg, w)
    e.close()


def _compare(cfg, e, oe, wave):
    h, oh = e.hidden(wave), oe.hidden(wave)
    assert h.shape == oh.shape == (cfg.hidden, cfg.frames(len(wave)))
    rel = np.linalg.norm(h - oh) / max(np.linalg.norm(oh), 1e-30)
    assert rel <= 1e-4, rel
    c, oc = e.encode(wave), oe.encode(wave)
    assert c.shape == oc.shape == (cfg.n_q, cfg.frames(len(wave)))
    assert c.min() >= 0 and c.max() < cfg.codebook_size
    np.testing.assert_array_equal(c[:cfg.n_semantic], oc[:cfg.n_semantic])
    agree = float((c == oc).mean())
    assert agree >= 0.98, agree
    return rel, agree


@pytest.mark.parametrize("n", [1, 13, 2417, 7000])
def test_small_encoder_matches_oracle(small, n):
    cfg, e, oe = small
    assert e.frames(n) == cfg.frames(n)
    _compare(cfg, e, oe, _wave(n, seed=n))


def test_small_encoder_is_causal_and_prefix_stable(small):
    cfg, e, _ = small
    wave = _wave(3000, seed=2)
    full = e.encode(wave)
    for n1 in (1000, 1210, 2999):
        part = e.encode(wave[:n1])
        T1 = part.shape[1]
        np.testing.assert_array_equal(part[:, :T1 - 1], full[:, :T1 - 1])


def test_small_encoder_valid_prefix_and_errors(small):
    cfg, e, _ = small
    wave = _wave(2417, seed=3)
    full = e.encode(wave)
    np.testing.assert_array_equal(e.encode(wave, n_valid=2), full[:2])
    with pytest.raises(q3t.Q3TError) as err:
        e.encode(wave, n_valid=cfg.n_q + 1)
    assert err.value.status == q3t.INVALID_INPUT


def test_full_size_encoder_matches_oracle():
    cfg = S.CodecEncoderConfig()
    w = S.make_codec_encoder_weights(cfg, seed=0)
    e = q3t.CodecEncoder(cfg, w)
    try:
        rel, agree = _compare(cfg, e, O.OracleCodecEncoder(cfg, w), _wave(48000, seed=9))
        print(f"full-size encoder, 2 s: hidden rel L2 {rel:.2e}, code agreement {agree:.4f}")
    finally:
        e.close()

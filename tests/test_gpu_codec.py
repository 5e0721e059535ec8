"""Speech-tokenizer decoder parity: CUDA path (C ABI) vs the f32 CPU oracle.

Tolerance: waveform SNR >= 40 dB against the oracle's f32 decode of the same
codes; output length and clamping exact; invalid codes rejected.
"""
import numpy as np
import pytest

import oracle as O
import q3t
import synthetic as S

pytestmark = pytest.mark.gpu

SNR_DB = 40.0


def snr_db(got, ref):
    err = np.sum((np.asarray(got, np.float64) - ref) ** 2)
    return 10 * np.log10(np.sum(np.asarray(ref, np.float64) ** 2) / max(err, 1e-30))


@pytest.fixture(scope="module")
def codec():
    cc = S.CodecConfig()
    cw = S.make_codec_weights(cc, seed=0)
    model = q3t.Model(codec_cfg=cc, codec_weights=cw)
    yield cc, model, O.OracleCodec(cc, cw)
    model.close()


def _codes(B, T, seed):
    return np.random.default_rng([seed, 13]).integers(0, 2048, size=(B, 16, T), dtype=np.int64)


@pytest.mark.parametrize("B,T", [(1, 1), (1, 4), (2, 7), (1, 24), (1, 70)])
def test_codec_decode_matches_oracle(codec, B, T):
    cc, model, oc = codec
    codes = _codes(B, T, seed=T)
    wave = model.codec_decode(codes)
    ref = oc.decode(codes)
    assert wave.shape == ref.shape == (B, cc.out_len(T))
    assert np.all(np.abs(wave) <= 1.0)
    for b in range(B):
        s = snr_db(wave[b], ref[b])
        assert s >= SNR_DB, f"item {b}: SNR {s:.1f} dB"


def test_codec_pcm_matches_to_pcm(codec):
    cc, model, oc = codec
    codes = _codes(1, 5, seed=3)
    wave, pcm = model.codec_decode(codes, pcm=True)
    ref = np.zeros(wave.shape[1], np.int16)
    O.lib().orc_to_pcm(O.fp(wave[0]), wave.shape[1], ref.ctypes.data_as(O.C.POINTER(O.C.c_int16)))
    np.testing.assert_array_equal(pcm[0], ref)  # to_pcm of the same f32 samples is bit-exact


def test_codec_batch_items_independent(codec):
    cc, model, oc = codec
    a, b = _codes(1, 6, seed=1), _codes(1, 6, seed=2)
    both = model.codec_decode(np.concatenate([a, b]))
    wa, wb = model.codec_decode(a)[0], model.codec_decode(b)[0]
    assert snr_db(both[0], wa) > 80 and snr_db(both[1], wb) > 80


def test_codec_rejects_bad_codes(codec):
    cc, model, oc = codec
    codes = _codes(1, 3, seed=4)
    codes[0, 5, 1] = 2048
    with pytest.raises(q3t.Q3TError) as e:
        model.codec_decode(codes)
    assert e.value.status == q3t.INVALID_INPUT
    codes[0, 5, 1] = -1
    with pytest.raises(q3t.Q3TError):
        model.codec_decode(codes)


def test_codec_long_sequence_properties(codec):
    """T = 750 frames (60 s), B = 2: the reference's output length
    ((((4T-1)*8-1)*5-1)*4-1)*3 = 1,439,445 samples, finite, clamped; the two
    items with identical codes decode identically."""
    cc, model, oc = codec
    codes = _codes(1, 750, seed=7)
    wave = model.codec_decode(np.concatenate([codes, codes]))
    assert wave.shape == (2, 1_439_445)
    assert np.isfinite(wave).all() and np.abs(wave).max() <= 1.0
    assert snr_db(wave[1], wave[0]) > 80
    assert wave[0].std() > 1e-3


def test_codec_fused_residual_unit_matches_two_launches(codec, monkeypatch):
    """The 96-channel residual units run as one launch (k7 conv, SnakeBeta,
    k1 conv on the tensor cores, intermediate kept in shared memory); the
    two-launch path (Q3T_CODEC_UNFUSED=1) rounds at the same points, so the
    two decodes agree far inside the oracle tolerance."""
    cc, model, oc = codec
    codes = _codes(2, 70, seed=11)
    fused = model.codec_decode(codes)
    monkeypatch.setenv("Q3T_CODEC_UNFUSED", "1")
    split = model.codec_decode(codes)
    for b in range(2):
        assert snr_db(fused[b], split[b]) > 90

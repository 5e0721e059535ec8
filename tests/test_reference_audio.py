"""Voice-clone reference audio in front of the encoders, host code of the C
ABI (no GPU): q3t_wav_read (decode_reference_audio,
execution/reference_audio.rs:17-50, 76-121) and q3t_resample_linear
(resample_linear, :123-156).

* the reference's own tests (reference_audio.rs:159-219, their literals
  extracted into tests/golden/reference_kats.json): resampled lengths,
  empty output for a zero rate, a 48 kHz stereo file mixed down and
  resampled to 24 kHz, the empty-payload error;
* bit-exact against the oracle's restatement for every format the
  reference reads (integer 16 / 24 / 32-bit, 32-bit float, the extensible
  header, extra chunks with odd-size padding) and 1-3 channels, and for
  resampling across the rate pairs reference clips come in;
* 16-bit PCM images written by Python's wave module.
"""
import io
import json
import os
import struct
import wave

import numpy as np
import pytest

import oracle as O
import q3t


def _wav(payload, channels, rate, bits, tag=1, extensible=False, extra_chunk=False):
    """A RIFF/WAVE image of raw interleaved sample bytes."""
    bps = bits // 8
    if extensible:
        fmt = struct.pack("<HHIIHHHHI", 0xFFFE, channels, rate, rate * channels * bps, channels * bps, bits, 22,
                          bits, 0) + struct.pack("<H", tag) + bytes(14)
    else:
        fmt = struct.pack("<HHIIHH", tag, channels, rate, rate * channels * bps, channels * bps, bits)
    body = b"WAVE" + b"fmt " + struct.pack("<I", len(fmt)) + fmt
    if extra_chunk:  # an odd-sized chunk before the data, padded to even
        body += b"LIST" + struct.pack("<I", 3) + b"abc" + b"\0"
    body += b"data" + struct.pack("<I", len(payload)) + payload + (b"\0" if len(payload) & 1 else b"")
    return b"RIFF" + struct.pack("<I", len(body)) + body


def _int_bytes(v, bits):
    v = np.asarray(v, np.int64) & ((1 << bits) - 1)
    return np.stack([(v >> (8 * k)) & 0xFF for k in range(bits // 8)], 1).astype(np.uint8).tobytes()


# ---- the reference's tests (literals extracted by tests/golden/make_golden.py) ----

@pytest.fixture(scope="module")
def kats():
    with open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "reference_kats.json")) as f:
        return json.load(f)


def test_resample_changes_length_for_new_sample_rate(kats):
    k = kats["resample_length"]
    for fn in (q3t.resample_linear, O.resample_linear):
        out = fn(k["input"], k["source_rate"], k["target_rate"])
        assert len(out) == k["expected_len"] and (out > 0).any()


def test_resample_returns_empty_for_invalid_rates(kats):
    for c in kats["resample_invalid_rates"]["cases"]:
        for fn in (q3t.resample_linear, O.resample_linear):
            assert len(fn(c["input"], c["source_rate"], c["target_rate"])) == 0


def test_stereo_mixdown_and_resample(kats):
    k = kats["wav_stereo_prepare"]
    img = _wav(np.array(k["pcm"], np.int16).tobytes(), k["channels"], k["rate"], 16)
    x, rate = q3t.wav_read(img)
    assert rate == k["native_rate"] and len(x) == k["native_len"]
    y = q3t.resample_linear(x, rate, k["target_rate"])
    assert len(y) == k["resampled_len"] and (np.abs(y) < k["max_abs"]).all()


def test_empty_payload_is_rejected(kats):
    with pytest.raises(q3t.Q3TError) as e:
        q3t.wav_read(_wav(b"", 1, 24000, 16))
    assert e.value.status == q3t.INVALID_INPUT
    assert kats["wav_empty_payload"]["message"] in str(e.value)


# ---- against the oracle ----

@pytest.mark.parametrize("channels", [1, 2, 3])
@pytest.mark.parametrize("kind", ["i16", "i24", "i32", "f32", "i16x", "f32x"])
def test_wav_read_matches_oracle(kind, channels):
    g = np.random.default_rng([channels, len(kind)])
    n = 257 * channels + (1 if channels > 1 else 0)  # a trailing partial frame when channels > 1
    if kind.startswith("f32"):
        payload = (g.standard_normal(n) * 0.4).astype("<f4").tobytes()
        img = _wav(payload, channels, 44100, 32, tag=3, extensible=kind.endswith("x"), extra_chunk=True)
    else:
        bits = int(kind[1:3])
        v = g.integers(-(1 << (bits - 1)), 1 << (bits - 1), n)
        v[:3] = [-(1 << (bits - 1)), (1 << (bits - 1)) - 1, 0]  # both extremes
        img = _wav(_int_bytes(v, bits), channels, 22050, bits, extensible=kind.endswith("x"),
                   extra_chunk=channels == 2)
    got, rate = q3t.wav_read(img)
    ref, ref_rate = O.decode_reference_audio(img)
    assert rate == ref_rate and got.shape == ref.shape == (257,)
    np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))
    assert np.abs(got).max() <= 1.0 or kind.startswith("f32")


def test_wav_read_matches_python_wave():
    g = np.random.default_rng(3)
    pcm = g.integers(-32768, 32768, 2 * 1000).astype(np.int16)
    buf = io.BytesIO()
    with wave.open(buf, "wb") as w:
        w.setnchannels(2)
        w.setsampwidth(2)
        w.setframerate(16000)
        w.writeframes(pcm.tobytes())
    got, rate = q3t.wav_read(buf.getvalue())
    lr = pcm.reshape(-1, 2).astype(np.float32) / np.float32(32768)
    assert rate == 16000
    np.testing.assert_array_equal(got, ((np.float32(-0.0) + lr[:, 0]) + lr[:, 1]) / np.float32(2))


@pytest.mark.parametrize("bad", ["not-riff", "zero-channels", "u8", "f64", "align", "truncated", "no-data"])
def test_wav_read_rejects_what_the_reference_rejects(bad):
    pcm = np.arange(8, dtype=np.int16).tobytes()
    img = {
        "not-riff": b"RIFX" + _wav(pcm, 1, 24000, 16)[4:],
        "zero-channels": _wav(pcm, 1, 24000, 16)[:22] + b"\0\0" + _wav(pcm, 1, 24000, 16)[24:],
        "u8": _wav(pcm, 1, 24000, 8),
        "f64": _wav(pcm, 1, 24000, 64, tag=3),
        "align": _wav(pcm, 1, 24000, 16)[:32] + struct.pack("<H", 4) + _wav(pcm, 1, 24000, 16)[34:],
        "truncated": _wav(pcm, 1, 24000, 16)[:-4],
        "no-data": _wav(pcm, 1, 24000, 16)[:36],
    }[bad]
    with pytest.raises(q3t.Q3TError) as e:
        q3t.wav_read(img)
    assert e.value.status == q3t.INVALID_INPUT
    with pytest.raises(ValueError):
        O.decode_reference_audio(img)


@pytest.mark.parametrize("src,dst", [(22050, 24000), (44100, 24000), (48000, 24000), (48000, 16000),
                                     (8000, 24000), (16000, 24000), (24000, 24000), (3, 7)])
@pytest.mark.parametrize("n", [1, 2, 1001])
def test_resample_matches_oracle(src, dst, n):
    x = (np.random.default_rng([src, dst, n]).standard_normal(n) * 0.3).astype(np.float32)
    got, ref = q3t.resample_linear(x, src, dst), O.resample_linear(x, src, dst)
    assert got.shape == ref.shape
    assert len(got) == (n if (src == dst or n == 1) else max((n * dst + src // 2) // src, 1))
    np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_wav_write_then_read_round_trip():
    """q3t_wav_write's image (PcmAudio::write_wav) read back by q3t_wav_read:
    mono samples / 32768, and stereo frames as the mean of their channels."""
    pcm = np.random.default_rng(9).integers(-32768, 32768, 600).astype(np.int16)
    x, rate = q3t.wav_read(q3t.wav_bytes(pcm, 24000, 1))
    assert rate == 24000
    np.testing.assert_array_equal(x, pcm.astype(np.float32) / np.float32(32768))
    y, _ = q3t.wav_read(q3t.wav_bytes(pcm, 48000, 2))
    lr = pcm.reshape(-1, 2).astype(np.float32) / np.float32(32768)
    np.testing.assert_array_equal(y, ((np.float32(-0.0) + lr[:, 0]) + lr[:, 1]) / np.float32(2))


def test_wav_read_differential_on_corrupted_images():
    """Byte flips and truncations of valid images: the library either
    rejects the image (INVALID_INPUT) or decodes exactly what the oracle
    decodes, and rejects exactly what the oracle rejects; it never reads
    outside the image (the parser bounds every chunk by the image size)."""
    g = np.random.default_rng(11)
    bases = [_wav(_int_bytes(g.integers(-2 ** 15, 2 ** 15, 64), 16), 2, 24000, 16, extra_chunk=True),
             _wav(_int_bytes(g.integers(-2 ** 23, 2 ** 23, 48), 24), 3, 16000, 24, extensible=True),
             _wav((g.standard_normal(40) * 0.5).astype("<f4").tobytes(), 1, 44100, 32, tag=3)]
    agree = 0
    for trial in range(600):
        img = bytearray(bases[trial % 3])
        if trial % 4 == 3:
            img = img[:g.integers(0, len(img))]
        else:
            for _ in range(g.integers(1, 4)):
                img[g.integers(0, len(img))] = g.integers(0, 256)
        img = bytes(img)
        try:
            ref = O.decode_reference_audio(img)
        except ValueError:
            ref = None
        try:
            got = q3t.wav_read(img)
        except q3t.Q3TError as e:
            assert e.status == q3t.INVALID_INPUT
            got = None
        assert (got is None) == (ref is None), trial
        if got is not None:
            assert got[1] == ref[1]
            np.testing.assert_array_equal(got[0].view(np.uint32), ref[0].view(np.uint32))
            agree += 1
    assert agree > 100


def test_resample_random_rates_match_oracle():
    """Random rate pairs (1 Hz .. 384 kHz, including ones whose products
    pass 2^32) and lengths: same length and bits as the oracle."""
    g = np.random.default_rng(21)
    for trial in range(300):
        src, dst = (int(v) for v in g.integers(1, 384001, 2))
        if trial % 10 == 0:
            src, dst = 4_000_000_000 - trial, 3_999_999_999  # u32 rates near the top of the range
        n = int(g.integers(1, 400))
        x = (g.standard_normal(n) * 0.5).astype(np.float32)
        got, ref = q3t.resample_linear(x, src, dst), O.resample_linear(x, src, dst)
        assert got.shape == ref.shape, (src, dst, n)
        np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))

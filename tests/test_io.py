"""Host-side IO of the C ABI, no GPU needed: the safetensors reader that
feeds q3t_model_load (checkpoint names, dtypes, shapes, values) and the WAV
writer of PcmAudio::write_wav (tts_infer/src/audio.rs:12-49), checked
byte-for-byte against Python's wave module."""
import ctypes as C
import io
import json
import struct
import wave

import numpy as np
import pytest

import q3t
import synthetic as S
from st_file import write_safetensors


def _values(t):
    n = int(np.prod(t.shape[:t.ndim])) if t.ndim else 1
    if t.dtype == 0:
        return np.ctypeslib.as_array(C.cast(t.data, C.POINTER(C.c_float)), (n,)).copy()
    bits = np.ctypeslib.as_array(C.cast(t.data, C.POINTER(C.c_uint16)), (n,)).astype(np.uint32) << 16
    return bits.view(np.float32)


def test_safetensors_lists_float_tensors(tmp_path):
    g = np.random.default_rng(0)
    a = g.standard_normal((3, 5)).astype(np.float32)
    b = S.bf16_round(g.standard_normal((2, 4, 6)).astype(np.float32))
    c = g.standard_normal((7,)).astype(np.float16)
    p = tmp_path / "w.safetensors"
    write_safetensors(p, {"talker.model.norm.weight": (a, "F32"), "x.y.weight": (b, "BF16"),
                          "half": (c, "F16"), "ids": (np.arange(4), "I64")}, metadata={"format": "pt"})
    ts = q3t.TensorSet(p)
    listed = {n: (d, s) for n, d, s in ts.tensors()}
    assert set(listed) == {"talker.model.norm.weight", "x.y.weight", "half"}, "integer tensors are skipped"
    assert listed["talker.model.norm.weight"] == (0, (3, 5))
    assert listed["x.y.weight"] == (1, (2, 4, 6))
    assert listed["half"] == (0, (7,)), "F16 is widened to f32"
    got = {t.name.decode(): _values(t) for t in ts.raw()}
    assert np.array_equal(got["talker.model.norm.weight"], a.ravel())
    assert np.array_equal(got["x.y.weight"], b.ravel())
    assert np.array_equal(got["half"], c.astype(np.float32))
    ts.close()


def _bad_file(tmp_path, header, data=b""):
    h = json.dumps(header).encode()
    p = tmp_path / "bad.safetensors"
    p.write_bytes(struct.pack("<Q", len(h)) + h + data)
    return p


def test_safetensors_rejects_malformed_files(tmp_path):
    cases = [
        _bad_file(tmp_path, {"w": {"dtype": "F32", "shape": [4], "data_offsets": [0, 16]}}, b"\0" * 8),
        _bad_file(tmp_path, {"w": {"dtype": "F32", "shape": [4], "data_offsets": [0, 12]}}, b"\0" * 16),
        _bad_file(tmp_path, {"w": {"dtype": "F32", "shape": [1, 1, 1, 1, 1], "data_offsets": [0, 4]}}, b"\0" * 4),
    ]
    for p in cases:
        with pytest.raises(q3t.Q3TError) as e:
            q3t.TensorSet(p)
        assert e.value.status == 2  # RUNTIME_LOAD
    trunc = tmp_path / "trunc.safetensors"
    trunc.write_bytes(struct.pack("<Q", 1000) + b"{}")
    with pytest.raises(q3t.Q3TError):
        q3t.TensorSet(trunc)
    with pytest.raises(q3t.Q3TError):
        q3t.TensorSet(tmp_path / "missing.safetensors")


@pytest.mark.parametrize("channels,n", [(1, 0), (1, 4801), (2, 3000)])
def test_wav_matches_python_wave(channels, n):
    pcm = np.random.default_rng(n).integers(-32768, 32768, n).astype(np.int16)
    got = q3t.wav_bytes(pcm, 24000, channels)
    buf = io.BytesIO()
    with wave.open(buf, "wb") as w:
        w.setnchannels(channels)
        w.setsampwidth(2)
        w.setframerate(24000)
        w.writeframes(pcm.tobytes())
    assert got == buf.getvalue()
    assert len(got) == 44 + 2 * n


def test_wav_rejects_partial_frames():
    with pytest.raises(q3t.Q3TError):
        q3t.wav_bytes(np.zeros(3, np.int16), 24000, 2)


def test_safetensors_corrupted_headers_fail_cleanly(tmp_path):
    """Byte flips in the JSON header and truncations of a valid checkpoint:
    the reader either lists tensors whose bytes lie inside the file (each
    read back here) or fails with RUNTIME_LOAD; it never reads past the
    header (numbers are parsed from bounded copies) or past the file."""
    g = np.random.default_rng(2)
    good = tmp_path / "good.safetensors"
    write_safetensors(good, {"a.weight": (g.standard_normal((3, 5)).astype(np.float32), "F32"),
                             "b.weight": (S.bf16_round(g.standard_normal((4, 2)).astype(np.float32)), "BF16"),
                             "c.weight": (g.standard_normal(7).astype(np.float16), "F16"),
                             "ids": (np.arange(3), "I64")})
    blob = good.read_bytes()
    hlen = struct.unpack("<Q", blob[:8])[0]
    ok = 0
    for trial in range(300):
        img = bytearray(blob)
        if trial % 5 == 4:
            img = img[:g.integers(0, len(img))]
        else:
            for _ in range(g.integers(1, 4)):
                img[8 + g.integers(0, hlen)] = g.choice(list(b'0123456789-,:[]{}" e'))
        p = tmp_path / f"c{trial}.safetensors"
        p.write_bytes(bytes(img))
        try:
            ts = q3t.TensorSet(p)
        except q3t.Q3TError as e:
            assert e.status == 2  # RUNTIME_LOAD
            continue
        for t in ts.raw():
            v = _values(t)
            assert v.size == int(np.prod(t.shape[:t.ndim])) if t.ndim else 1
        ts.close()
        ok += 1
    assert ok > 0

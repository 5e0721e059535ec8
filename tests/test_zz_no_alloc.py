"""q3t_codec_decode_static against the allocating q3t_codec_decode, both
called through the C ABI.  The static entry serves callers that must not
allocate device memory while they run: a real-time audio callback, where a
cudaMalloc can stall behind work of the whole device, and host frameworks
whose own allocator owns all device memory.  It uses a file-scope device
array instead.

Both entries launch the same kernels on the same inputs, so the tolerance is
tight: |wave difference| <= 1e-6 and PCM equal to within one LSB.  Two static
calls in a row use different shapes, so the second reuses the scratch that the
first left behind."""
import ctypes as C

import numpy as np
import pytest

import q3t
import synthetic as S

pytestmark = pytest.mark.gpu

WAVE_ATOL = 1e-6
PCM_ATOL = 1


@pytest.fixture(scope="module")
def model():
    cc = S.CodecConfig()
    m = q3t.Model(codec_cfg=cc, codec_weights=S.make_codec_weights(cc, seed=0))
    yield cc, m
    m.close()


def _codes(B, T, seed):
    return np.random.default_rng([seed, 29]).integers(0, 2048, size=(B, 16, T), dtype=np.int64)


def _decode_static(m, codes):
    codes = np.ascontiguousarray(codes, np.int64)
    B, _, T = codes.shape
    n = m.codec_out_len(T)
    wave = np.zeros((B, n), np.float32)
    pcm = np.zeros((B, n), np.int16)
    nn = C.c_int64()
    q3t.check(q3t.lib().q3t_codec_decode_static(
        m.h, codes.ctypes.data_as(C.POINTER(C.c_int64)), B, T,
        wave.ctypes.data_as(C.POINTER(C.c_float)), pcm.ctypes.data_as(C.POINTER(C.c_int16)),
        C.byref(nn), None))
    assert nn.value == n
    return wave, pcm


def test_static_decode_matches_allocating_decode_twice(model):
    cc, m = model
    for B, T, seed in [(1, 24, 1), (2, 7, 2)]:
        codes = _codes(B, T, seed)
        wave, pcm = _decode_static(m, codes)
        ref_wave, ref_pcm = m.codec_decode(codes, pcm=True)
        assert wave.shape == ref_wave.shape == (B, cc.out_len(T))
        np.testing.assert_allclose(wave, ref_wave, rtol=0, atol=WAVE_ATOL)
        assert np.max(np.abs(pcm.astype(np.int32) - ref_pcm)) <= PCM_ATOL


def _device_memory_state():
    """(used and reserved bytes of the device's default stream-ordered pool,
    free device bytes): what any cudaMalloc / cudaMallocAsync, the library's
    or a caching allocator's, would change."""
    from cuda.bindings import runtime as rt
    err, dev = rt.cudaGetDevice()
    assert err == rt.cudaError_t.cudaSuccess
    err, pool = rt.cudaDeviceGetDefaultMemPool(dev)
    assert err == rt.cudaError_t.cudaSuccess
    vals = []
    for attr in (rt.cudaMemPoolAttr.cudaMemPoolAttrUsedMemCurrent,
                 rt.cudaMemPoolAttr.cudaMemPoolAttrReservedMemCurrent):
        err, v = rt.cudaMemPoolGetAttribute(pool, attr)
        assert err == rt.cudaError_t.cudaSuccess
        vals.append(int(v))
    err, free, _ = rt.cudaMemGetInfo()
    assert err == rt.cudaError_t.cudaSuccess
    return tuple(vals) + (int(free),)


def test_static_decode_allocates_nothing(model):
    """The point of the entry: after the library's kernels are loaded (one
    allocating decode of the same shape), two static calls leave the device's
    memory exactly as they found it."""
    _, m = model
    codes = _codes(1, 24, 4)
    m.codec_decode(codes, pcm=True)  # loads every kernel this shape uses
    _decode_static(m, codes)
    before = _device_memory_state()
    w1, _ = _decode_static(m, codes)
    w2, _ = _decode_static(m, codes)
    assert _device_memory_state() == before
    np.testing.assert_array_equal(w1, w2)


def test_static_decode_rejects_oversize(model):
    _, m = model
    with pytest.raises(q3t.Q3TError) as e:
        _decode_static(m, _codes(2, 24, 3))
    assert e.value.status == q3t.INVALID_INPUT
    assert b"static" in q3t.lib().q3t_last_error()

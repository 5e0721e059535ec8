"""Streaming codec (codec_mode 2) inside the continuous batch.

Every chunk_frames frames a request's window of up to left_context +
chunk_frames frames is decoded and the samples of its newest chunk are
emitted (the engine's own mode; the reference decodes whole sequences).
The windows of a step decode on a second stream overlapped with the next
step's frame, so these tests check that what reaches the host is complete
and in order: each request's samples must equal the same windows decoded
directly through q3t_codec_decode (same kernels; batch items are
independent, so > 80 dB), and the per-request / per-step sample counts must
add up.
"""
import numpy as np
import pytest

import q3t
import synthetic as S

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tts():
    cfg = S.TalkerConfig().small(talker_layers=2, predictor_layers=2)
    cc = S.CodecConfig()
    model = q3t.Model(cfg, S.make_talker_weights(cfg, seed=0), cc, S.make_codec_weights(cc, seed=0),
                      kv_pages=2048, max_active=4)
    yield cfg, cc, model
    model.close()


def snr_db(got, ref):
    err = np.sum((np.asarray(got, np.float64) - ref) ** 2)
    return 10 * np.log10(np.sum(np.asarray(ref, np.float64) ** 2) / max(err, 1e-30))


def expected_stream(model, cc, codes_tg, chunk, ctx):
    """The chunk schedule of the streaming mode restated on the host: window
    [f0, e + n) with f0 = max(0, e - ctx); the newest n frames' samples,
    shifted by the samples the both-side trims drop at the window's end."""
    T = codes_tg.shape[0]
    spf = int(np.prod(cc.up_ratios)) * int(np.prod(cc.rates))
    out, e = [], 0
    while e < T:
        n = min(chunk, T - e)
        f0 = max(0, e - ctx)
        Tw = e + n - f0
        nout = cc.out_len(Tw)
        deficit = spf * Tw - nout
        a0 = e - f0
        s0 = min(nout, a0 * spf - deficit) if a0 > 0 else 0
        s1 = min(nout, (a0 + n) * spf - deficit)
        if s1 > s0:
            win = codes_tg[f0:e + n].T[None].copy()  # [1][G][Tw]
            out.append(model.codec_decode(win)[0, s0:s1])
        e += n
    return np.concatenate(out) if out else np.zeros(0, np.float32)


@pytest.mark.parametrize("chunk,ctx", [(4, 2), (3, 0)])
def test_stream_chunks_match_direct_window_decode(tts, chunk, ctx):
    cfg, cc, model = tts
    b = model.batch(max_active=4, codec_mode=2, chunk_frames=chunk, left_context=ctx, keep_output=1)
    specs = [(5, 9, 1), (12, 13, 2), (7, 6, 3), (9, 4, 4), (6, 11, 5)]  # 5 requests, 4 slots: one waits
    ids, codes = [], []
    for S_len, frames, seed in specs:
        prompt, trailing, pad = S.synthetic_talker_inputs(cfg, S_len, seed=seed)
        c = S.teacher_codes(frames, seed=seed)
        ids.append(b.submit(prompt, trailing, pad, frames, forced=c))
        codes.append(c)
    step_samples = 0
    for _ in range(64):
        st = b.step()
        step_samples += st["samples"]
        if st["active"] == 0 and b.pending() == (0, 0):
            break
    total = 0
    for rid, c in zip(ids, codes):
        state, T, ns = b.poll(rid)
        assert state == 2 and T == c.shape[0]
        got_codes, _, wave = b.take(rid, with_wave=True)
        np.testing.assert_array_equal(got_codes, c.T)
        ref = expected_stream(model, cc, c, chunk, ctx)
        assert ns == ref.shape[0] == wave.shape[0]
        assert snr_db(wave, ref) > 80
        total += ns
    assert step_samples == total
    b.close()


def test_stream_without_host_output_counts_samples(tts):
    """keep_output = 0: samples stay on the device, the counts still add up."""
    cfg, cc, model = tts
    b = model.batch(max_active=4, codec_mode=2, chunk_frames=4, left_context=2, keep_output=0)
    frames = [10, 7, 5]
    for i, f in enumerate(frames):
        prompt, trailing, pad = S.synthetic_talker_inputs(cfg, 6 + i, seed=20 + i)
        b.submit(prompt, trailing, pad, f, forced=S.teacher_codes(f, seed=20 + i))
    got = 0
    for _ in range(64):
        st = b.step()
        got += st["samples"]
        if st["active"] == 0 and b.pending() == (0, 0):
            break
    spf = int(np.prod(cc.up_ratios)) * int(np.prod(cc.rates))
    assert got == sum(emitted_samples(cc, f, 4, 2, spf) for f in frames)
    b.close()


def emitted_samples(cc, T, chunk, ctx, spf):
    """Samples the chunk schedule emits for a T-frame request."""
    total, e = 0, 0
    while e < T:
        n = min(chunk, T - e)
        f0 = max(0, e - ctx)
        Tw = e + n - f0
        nout = cc.out_len(Tw)
        deficit = spf * Tw - nout
        a0 = e - f0
        s0 = min(nout, a0 * spf - deficit) if a0 > 0 else 0
        s1 = min(nout, (a0 + n) * spf - deficit)
        total += max(0, s1 - s0)
        e += n
    return total

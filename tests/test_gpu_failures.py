"""Failure paths in the forms that fault no GPU: a bounded device wait that
runs out (a plain global-memory wait for a word nothing sets) and a KV page
pool that runs dry.  Each must come back as a status, leave the device usable
and, for the page pool, fail only the request that ran out."""
import numpy as np
import pytest

import oracle as O
import q3t
import synthetic as S

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def small():
    cfg = S.TalkerConfig().small(talker_layers=2, predictor_layers=5)
    w = S.make_talker_weights(cfg, seed=0)
    yield cfg, w


def _decode_matches_oracle(cfg, w, model, L, seed):
    g = np.random.default_rng([seed, 5])
    c = cfg.talker
    k = S.bf16_round(g.standard_normal((c.n_layers, c.n_kv, L, c.head_dim), dtype=np.float32))
    v = S.bf16_round(g.standard_normal((c.n_layers, c.n_kv, L, c.head_dim), dtype=np.float32))
    prompt, trailing, pad = S.synthetic_talker_inputs(cfg, 1, seed)
    sess = model.session(prompt, trailing, pad, max_new_tokens=4)
    sess.load_kv(S.bf16_bits(k), S.bf16_bits(v), L)
    emb = g.standard_normal(c.hidden).astype(np.float32)
    logits, _ = sess.decode_embeds(emb)
    sess.close()
    ot = O.OracleTalker(cfg, w)
    kvs, mems = ot.make_caches("talker", cap=L + 8)
    for l in range(c.n_layers):
        mems[l][0][:, :L] = k[l]
        mems[l][1][:, :L] = v[l]
        kvs[l].len = L
    ref = ot.codec_head(ot.stack_forward("talker", kvs, emb[None])[0])[0]
    err = np.abs(logits - ref).max()
    assert err <= max(2e-2, 1e-2 * np.abs(ref).max()), err


def test_device_wait_timeout_is_reported_and_the_device_stays_usable(small, monkeypatch):
    """Every CTA of the streamed single-token kernel first waits for a word
    that nothing sets, with a short poll limit: the wait runs out, later waits
    are skipped, the launch ends and the call returns DEVICE_TIMEOUT.  A new
    session on the same model then decodes normally."""
    cfg, w = small
    model = q3t.Model(cfg, w, kv_pages=64, max_active=2)
    monkeypatch.setenv("Q3T_WAIT_POLLS", "4096")
    monkeypatch.setenv("Q3T_TEST_STALL_WAITS", "1")
    prompt, trailing, pad = S.synthetic_talker_inputs(cfg, 3, seed=1)
    sess = model.session(prompt, trailing, pad, max_new_tokens=4)
    emb = np.random.default_rng([1, 9]).standard_normal(cfg.talker.hidden).astype(np.float32)
    with pytest.raises(q3t.Q3TError) as e:
        sess.decode_embeds(emb)
    assert e.value.status == q3t.DEVICE_TIMEOUT
    assert "bounded device wait" in str(e.value)
    sess.close()
    monkeypatch.delenv("Q3T_TEST_STALL_WAITS")
    monkeypatch.delenv("Q3T_WAIT_POLLS")
    _decode_matches_oracle(cfg, w, model, L=40, seed=2)
    model.close()


def test_page_pool_exhaustion_fails_one_request_and_serves_the_rest(small):
    """A 24-page pool (384 tokens): a request whose prompt can never fit
    fails at admission, a long request fails when the pool runs dry, and the
    short ones finish with their teacher-forced codes."""
    cfg, w = small
    model = q3t.Model(cfg, w, kv_pages=24, max_active=4)
    b = model.batch(max_active=4)
    reqs = {}
    for name, S_len, frames, seed in [("short_a", 8, 10, 1), ("long", 40, 400, 2), ("short_b", 9, 12, 3),
                                      ("never_fits", 400, 4, 4)]:
        prompt, trailing, pad = S.synthetic_talker_inputs(cfg, S_len, seed=seed)
        codes = S.teacher_codes(frames, seed=seed)
        reqs[name] = (b.submit(prompt, trailing, pad, frames, forced=codes), codes)
    for _ in range(600):
        b.step()
        if b.pending() == (0, 0):
            break
    assert b.pending() == (0, 0)
    for name in ("short_a", "short_b"):
        rid, codes = reqs[name]
        state, T, _ = b.poll(rid)
        assert state == 2 and T == codes.shape[0], (name, state, T)
        got, _, _ = b.take(rid)
        np.testing.assert_array_equal(got, codes.T)
    rid, _ = reqs["long"]
    state, T, _ = b.poll(rid)
    assert state == 3 and 0 < T < 400
    assert b"KV capacity" in q3t.lib().q3t_last_error()
    rid, _ = reqs["never_fits"]
    state, T, _ = b.poll(rid)
    assert state == 3 and T == 0
    assert b"KV pages" in q3t.lib().q3t_last_error()
    b.close()
    # a session whose prompt cannot fit the pool
    prompt, trailing, pad = S.synthetic_talker_inputs(cfg, 400, seed=5)
    with pytest.raises(q3t.Q3TError) as e:
        model.session(prompt, trailing, pad, max_new_tokens=2)
    assert e.value.status == q3t.OUT_OF_PAGES
    model.close()

"""Pins the CPU oracle to the reference's own known-answer tests (extracted
from the Rust sources into tests/golden/reference_kats.json by
tests/golden/make_golden.py)."""
import math

import numpy as np
import pytest

import oracle as O
import synthetic as S


def test_sample_token_skips_masked_logits(kats):
    k = kats["sample_suppress"]
    lg = np.array(k["logits"], np.float32)
    sup = np.array(k["suppress"], np.int64)
    s = O.sampling()
    tok = O.lib().orc_sample_token(O.fp(lg), len(lg), s, O.ip(sup), len(sup), 0.5)
    assert tok == k["expected"]


@pytest.mark.parametrize("u", [0.0, 0.3, 0.999])
def test_top_k_one_returns_argmax(kats, u):
    k = kats["sample_topk1"]
    lg = np.array(k["logits"], np.float32)
    s = O.sampling(do_sample=k["do_sample"], temperature=k["temperature"], top_k=k["top_k"],
                   top_p=k["top_p"])
    assert O.lib().orc_sample_token(O.fp(lg), len(lg), s, None, 0, u) == k["expected"]


def test_repetition_penalty_enabled(kats):
    for c in kats["repetition_penalty_enabled"]["cases"]:
        p = 0.0 if c["penalty"] is None else float(c["penalty"])
        assert bool(O.lib().orc_repetition_penalty_enabled(p)) == c["enabled"], c


def _kv(cache_dims):
    _, heads, cap, hd = cache_dims
    k = np.zeros((heads, cap, hd), np.float32)
    v = np.zeros_like(k)
    return O.KV(O.fp(k), O.fp(v), 0, cap, heads, hd), (k, v)


def test_kv_reset_preserves_allocation(kats):
    k = kats["kv_reset_len"]
    kv, mem = _kv(k["cache"])
    _, h, s, d = k["input"]
    ones = np.ones((h, s, d), np.float32)
    O.lib().orc_kv_forward(kv, O.fp(ones), O.fp(ones), s, None, None)
    assert kv.len == k["len_after_forward"]
    O.lib().orc_kv_reset_preserve(kv)
    assert kv.len == k["len_after_reset"]


def test_kv_reset_exposes_only_new_values(kats):
    k = kats["kv_reset_values"]
    kv, mem = _kv(k["cache"])
    fk = np.array(k["first_key"], np.float32).reshape(1, -1, 1)
    fv = np.array(k["first_value"], np.float32).reshape(1, -1, 1)
    O.lib().orc_kv_forward(kv, O.fp(fk), O.fp(fv), fk.shape[1], None, None)
    O.lib().orc_kv_reset_preserve(kv)
    nk = np.array(k["next_key"], np.float32).reshape(1, -1, 1)
    nv = np.array(k["next_value"], np.float32).reshape(1, -1, 1)
    ko = np.zeros(4, np.float32)
    vo = np.zeros(4, np.float32)
    n = O.lib().orc_kv_forward(kv, O.fp(nk), O.fp(nv), nk.shape[1], O.fp(ko), O.fp(vo))
    assert n == k["len"] == kv.len
    assert list(ko[:n]) == k["key_out"]
    assert list(vo[:n]) == k["value_out"]


def test_kv_sliding_window_keeps_latest():
    # kv.rs:109-132: a full cache drops the oldest steps
    kv, mem = _kv([1, 1, 4, 1])
    for step in range(6):
        t = np.array([[[float(step)]]], np.float32)
        out = np.zeros(4, np.float32)
        n = O.lib().orc_kv_forward(kv, O.fp(t), O.fp(t), 1, O.fp(out), O.fp(out.copy()))
    assert n == 4 and list(out) == [2.0, 3.0, 4.0, 5.0]


def test_pad_1d(kats):
    for k in kats["pad_1d"]:
        x = np.array(k["input"], np.float32)
        out = np.zeros(len(x) + k["left"] + k["right"], np.float32)
        O.lib().orc_pad_1d(O.fp(x), 1, len(x), k["left"], k["right"],
                           0 if k["mode"] == "constant" else 1, O.fp(out))
        assert list(out) == k["expected"], k["source"]


def test_config_fixture_matches_synthetic_dims(kats):
    c = kats["talker_config"]["config"]
    cfg = S.TalkerConfig()
    t, p = cfg.talker, cfg.predictor
    assert (t.hidden, t.inter, t.n_layers, t.n_heads, t.n_kv, t.head_dim, t.vocab) == (
        c["hidden_size"], c["intermediate_size"], c["num_hidden_layers"],
        c["num_attention_heads"], c["num_key_value_heads"], c["head_dim"], c["vocab_size"])
    pc = c["code_predictor_config"]
    assert (p.hidden, p.inter, p.n_layers, p.n_heads, p.n_kv, p.head_dim, p.vocab) == (
        pc["hidden_size"], pc["intermediate_size"], pc["num_hidden_layers"],
        pc["num_attention_heads"], pc["num_key_value_heads"], pc["head_dim"], pc["vocab_size"])
    assert cfg.n_groups == c["num_code_groups"] == pc["num_code_groups"]
    assert t.eps == c["rms_norm_eps"] and t.theta == c["rope_theta"]
    assert p.theta == pc["rope_theta"]


def test_sdpa_kat_shape_and_masking(kats):
    k = kats["sdpa_shape"]
    q = np.array(k["query"], np.float32).reshape(2, 2, 2)
    kk = np.array(k["key"], np.float32).reshape(2, 2, 2)
    v = np.array(k["value"], np.float32).reshape(2, 2, 2)
    mask = np.array(k["mask"], np.uint8).reshape(2, 2)
    out = np.zeros((2, 2, 2), np.float32)
    scale = 1.0 / math.sqrt(2.0)
    O.lib().orc_sdpa(O.fp(q), O.fp(kk), O.fp(v), mask.ctypes.data_as(O.C.POINTER(O.C.c_uint8)),
                     2, 2, 2, 2, scale, O.fp(out))
    # row 0 attends to key 0 only (mask [0, 1]); row 1 to both
    np.testing.assert_allclose(out[:, 0], v[:, 0], rtol=0, atol=1e-7)
    for h in range(2):
        s = q[h, 1] @ kk[h].T * scale
        p = np.exp(s - s.max()); p /= p.sum()
        np.testing.assert_allclose(out[h, 1], p @ v[h], rtol=1e-6)


def test_suppress_ids():
    out = np.zeros(4096, np.int64)
    n = O.lib().orc_build_suppress_ids(3072, 2150, O.ip(out))
    ids = list(out[:n])
    assert n == 1023 and ids[0] == 2048 and ids[-1] == 3071 and 2150 not in ids


def test_repetition_penalty_accumulates_duplicates():
    lg = np.array([2.0, -1.0, 4.0], np.float32)
    hist = np.array([0, 0, 1], np.int64)
    O.lib().orc_apply_repetition_penalty(O.fp(lg), 3, O.ip(hist), 3, 2.0)
    # delta = logit * (1/p - 1) scatter-added per occurrence, sign ignored
    np.testing.assert_allclose(lg, [2.0 - 1.0 - 1.0, -1.0 + 0.5, 4.0])


def test_codec_output_length():
    assert S.CodecConfig().out_len(750) == 1_439_445
    assert S.CodecConfig().out_len(4) == ((((16 - 1) * 8 - 1) * 5 - 1) * 4 - 1) * 3


def test_to_pcm_rounding():
    x = np.array([0.0, 1.0, -1.0, 2.0, 0.5 / 32768, -1.5 / 32768], np.float32)
    out = np.zeros(len(x), np.int16)
    O.lib().orc_to_pcm(O.fp(x), len(x), out.ctypes.data_as(O.C.POINTER(O.C.c_int16)))
    assert list(out) == [0, 32767, -32768, 32767, 1, -2]


def test_text_projection_oracle_matches_numpy():
    """The oracle's project_text_ids (session_seed.rs:668-679, mlp.rs:36-40)
    against an independent numpy restatement of the same rounding points:
    bf16(silu(fc1 x + b1)), then bf16(fc2 h + b2).  Sums differ only in
    order, so an occasional element rounds to the neighbouring bf16 value
    (and a flipped hidden value moves the smallest outputs by ~1e-6)."""
    cfg = S.TalkerConfig().small(talker_layers=1, predictor_layers=1)
    w = S.make_talker_weights(cfg, seed=0)
    w.update(S.make_text_weights(cfg, seed=0, text_vocab=512, text_hidden=256))
    ot = O.OracleTalker(cfg, w)
    ids = np.array([0, 511, 7, 7, 300], np.int64)
    got = ot.text_project(ids)
    e = w["talker.model.text_embedding.weight"][ids].astype(np.float64)
    a = e @ w["talker.text_projection.linear_fc1.weight"].T.astype(np.float64) + w["talker.text_projection.linear_fc1.bias"]
    h = S.bf16_round((a / (1 + np.exp(-a))).astype(np.float32)).astype(np.float64)
    o = h @ w["talker.text_projection.linear_fc2.weight"].T.astype(np.float64) + w["talker.text_projection.linear_fc2.bias"]
    ref = S.bf16_round(o.astype(np.float32))
    assert got.shape == (5, cfg.talker.hidden)
    assert np.array_equal(got, S.bf16_round(got)), "outputs are bf16 values"
    diff = np.abs(got - ref)
    assert (diff <= np.abs(ref) * 2.0 ** -7 + 1e-3 * np.abs(ref).max()).all()
    assert (diff == 0).mean() > 0.97
    assert np.array_equal(got[2], got[3]), "equal ids give equal rows"


# Control ids of the reference's base-profile compiler fixture with automatic
# language (execution/compiler/tests.rs:87-106): codec prefix
# [nothink, think_bos, think_eos, pad, bos]; pad 2049 and bos 2048 are its
# last two entries (compiler/mod.rs:326).
SEED_CONTROLS = {"tts_bos_token_id": 501, "tts_eos_token_id": 502, "tts_pad_token_id": 503,
                 "codec_prefix_ids": [2051, 2052, 2053, 2049, 2048], "codec_pad_id": 2049, "codec_bos_id": 2048}


def test_session_seed_oracle_layout():
    """build_non_streaming_seed (session_seed.rs:151-215) in the oracle: rows
    = leading + 3 role + (prefix - 1) + body + 2, each row the bf16 sum of the
    projected text row and the codec embedding row the reference pairs it
    with; the pad embedding is P(tts_pad)."""
    cfg = S.TalkerConfig().small(talker_layers=1, predictor_layers=1)
    w = S.make_talker_weights(cfg, seed=0)
    w.update(S.make_text_weights(cfg, seed=0, text_vocab=512, text_hidden=256))
    ot = O.OracleTalker(cfg, w)
    text = np.arange(10, 22, dtype=np.int64)  # role 10..12, body 13..16, 5 trailing ids
    lead = np.array([40, 41], np.int64)
    rows, pad = ot.session_seed(text, SEED_CONTROLS, leading_ids=lead)
    c = SEED_CONTROLS
    assert rows.shape == (2 + 3 + 4 + 4 + 2, cfg.talker.hidden)
    P = lambda ids: ot.text_project(np.asarray(ids, np.int64))
    E = w["talker.model.codec_embedding.weight"].astype(np.float32)
    bos, eos, tpad = P([c["tts_bos_token_id"], c["tts_eos_token_id"], c["tts_pad_token_id"]])
    np.testing.assert_array_equal(pad, tpad)
    np.testing.assert_array_equal(rows[0:2], P(lead))
    np.testing.assert_array_equal(rows[2:5], P(text[:3]))
    for i, cid in enumerate(c["codec_prefix_ids"][:4]):
        t = bos if i == 3 else tpad
        np.testing.assert_array_equal(rows[5 + i], S.bf16_round(t + E[cid]))
    np.testing.assert_array_equal(rows[9:13], S.bf16_round(P(text[3:7]) + E[2049]))
    np.testing.assert_array_equal(rows[13], S.bf16_round(eos + E[2049]))
    np.testing.assert_array_equal(rows[14], S.bf16_round(tpad + E[2048]))
    short, _ = ot.session_seed(text[:8], SEED_CONTROLS)  # empty body, no leading ids
    assert short.shape[0] == 3 + 4 + 0 + 2


def _clone_fixture():
    cfg = S.TalkerConfig().small(talker_layers=1, predictor_layers=1)
    w = S.make_talker_weights(cfg, seed=0)
    w.update(S.make_text_weights(cfg, seed=0, text_vocab=512, text_hidden=256))
    return cfg, w, O.OracleTalker(cfg, w)


def test_voice_clone_seed_oracle_layout():
    """build_voice_clone_seed without reference text (the x-vector recipe,
    session_seed.rs:248-322) in the oracle: 3 role rows, the codec prefix of
    voice_clone_codec_prefix (:538-584: pad + E(tag) for all prefix ids but
    the last two, pad + bf16(x-vector), bos + E(codec_pad)), then P(body[0])
    + E(codec_bos); trailing text P(body[1..]) then P(eos)."""
    cfg, w, ot = _clone_fixture()
    c = SEED_CONTROLS
    H = cfg.talker.hidden
    text = np.arange(10, 22, dtype=np.int64)  # role 10..12, body 13..16, 5 trailing ids
    spk = np.random.default_rng(4).standard_normal(H).astype(np.float32)
    rows, trailing, pad = ot.session_seed_voice_clone(text, c, spk)
    P = lambda ids: ot.text_project(np.asarray(ids, np.int64))
    E = w["talker.model.codec_embedding.weight"].astype(np.float32)
    bos, eos, tpad = P([c["tts_bos_token_id"], c["tts_eos_token_id"], c["tts_pad_token_id"]])
    n = len(c["codec_prefix_ids"])
    assert rows.shape == (3 + n + 1, H)
    np.testing.assert_array_equal(pad, tpad)
    np.testing.assert_array_equal(rows[:3], P(text[:3]))
    for i, cid in enumerate(c["codec_prefix_ids"][:n - 2]):
        np.testing.assert_array_equal(rows[3 + i], S.bf16_round(tpad + E[cid]))
    np.testing.assert_array_equal(rows[3 + n - 2], S.bf16_round(tpad + S.bf16_round(spk)))
    np.testing.assert_array_equal(rows[3 + n - 1], S.bf16_round(bos + E[c["codec_pad_id"]]))
    np.testing.assert_array_equal(rows[3 + n], S.bf16_round(P(text[3:4])[0] + E[c["codec_bos_id"]]))
    np.testing.assert_array_equal(trailing, np.concatenate([P(text[4:7]), eos[None]]))
    short, tr, _ = ot.session_seed_voice_clone(text[:8], c, spk)  # empty body: no bos row, trailing = eos
    assert short.shape[0] == 3 + n and tr.shape[0] == 1
    np.testing.assert_array_equal(tr[0], eos)


@pytest.mark.parametrize("ref_frames", [2, 9])
def test_voice_clone_icl_seed_oracle_layout(ref_frames):
    """build_voice_clone_icl_seed (session_seed.rs:324-396): text = P(ref
    body + target body + eos) against codec = [E(codec_bos), the summed
    reference frames]; with more text than codec rows the excess text is the
    trailing text, otherwise pad rows fill the text side and the trailing
    text is P(pad).  The frame sum (:602-655) adds the 16 group embeddings
    as bf16 tensors in group order."""
    cfg, w, ot = _clone_fixture()
    c = SEED_CONTROLS
    H, G = cfg.talker.hidden, cfg.n_groups
    text = np.arange(30, 42, dtype=np.int64)              # target body 33..36
    ref_text = np.arange(60, 68, dtype=np.int64)          # ref body 63..65 (3 ids, 2 trailing)
    g = np.random.default_rng(ref_frames)
    codes = g.integers(0, 2048, (G, ref_frames))
    spk = g.standard_normal(H).astype(np.float32)
    rows, trailing, pad = ot.session_seed_voice_clone(text, c, spk, ref_text_ids=ref_text, ref_codes=codes)
    n = len(c["codec_prefix_ids"])
    P = lambda ids: ot.text_project(np.asarray(ids, np.int64))
    E = w["talker.model.codec_embedding.weight"].astype(np.float32)
    s = E[codes[0]]
    for j in range(1, G):
        s = S.bf16_round(s + w[f"talker.code_predictor.model.codec_embedding.{j - 1}.weight"][codes[j]])
    codec = np.concatenate([E[c["codec_bos_id"]][None], s])
    all_text = P(np.concatenate([ref_text[3:6], text[3:7], [c["tts_eos_token_id"]]]))  # 8 rows
    assert rows.shape == (3 + n + 1 + ref_frames, H)
    icl = rows[3 + n:]
    if len(all_text) > len(codec):  # 8 text rows against 3 codec rows
        np.testing.assert_array_equal(icl, S.bf16_round(all_text[:len(codec)] + codec))
        np.testing.assert_array_equal(trailing, all_text[len(codec):])
    else:  # 8 text rows + 2 pad rows against 10 codec rows
        filled = np.concatenate([all_text, np.repeat(pad[None], len(codec) - len(all_text), 0)])
        np.testing.assert_array_equal(icl, S.bf16_round(filled + codec))
        np.testing.assert_array_equal(trailing, pad[None])
    with pytest.raises(ValueError):
        ot.session_seed_voice_clone(text, c, spk, ref_text_ids=ref_text)  # no reference codes


def test_voice_clone_icl_seed_equal_lengths():
    """build_voice_clone_icl_seed with as many text rows as codec rows
    (session_seed.rs:366-381, the else branch with no pad rows): every text
    row pairs with a codec row and the trailing text is P(pad)."""
    cfg, w, ot = _clone_fixture()
    c = SEED_CONTROLS
    text = np.arange(30, 40, dtype=np.int64)      # target body 33..34 (2 ids)
    ref_text = np.arange(60, 66, dtype=np.int64)  # ref body 63 (1 id)
    codes = np.random.default_rng(5).integers(0, 2048, (cfg.n_groups, 3))  # 1 + 3 codec rows, 1 + 2 + 1 text rows
    rows, trailing, pad = ot.session_seed_voice_clone(text, c, np.zeros(cfg.talker.hidden, np.float32),
                                                      ref_text_ids=ref_text, ref_codes=codes)
    n = len(c["codec_prefix_ids"])
    assert rows.shape[0] == 3 + n + 4
    np.testing.assert_array_equal(trailing, pad[None])
    all_text = ot.text_project(np.array([63, 33, 34, c["tts_eos_token_id"]], np.int64))
    E = w["talker.model.codec_embedding.weight"].astype(np.float32)
    np.testing.assert_array_equal(rows[3 + n], S.bf16_round(all_text[0] + E[c["codec_bos_id"]]))
    np.testing.assert_array_equal(rows[3 + n + 1:], S.bf16_round(all_text[1:] + ot.ref_codec_sum(codes)))

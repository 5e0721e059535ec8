"""Prompt text projection on the device (q3t_text_project, the reference's
project_text_ids, session_seed.rs:668-679) vs the CPU oracle, and a prompt
built from token ids driving a session (the full-pipeline configuration's
input path: text ids -> text_projection(text_embedding(ids)) -> talker).

Tolerance: the GEMMs round the same tensors to bf16 as the oracle (the SiLU
output and the final rows) with f32 sums in a different order, so an
occasional row element lands on the neighbouring bf16 value:
max |gpu - ref| <= max(2e-2, 1e-2 max |ref|) and relative L2 <= 1e-2, with
>= 95 % of the elements bit-identical.
"""
import numpy as np
import pytest

import oracle as O
import q3t
import synthetic as S

pytestmark = pytest.mark.gpu

TEXT_VOCAB, TEXT_HIDDEN = 4096, 2048


@pytest.fixture(scope="module")
def text_model():
    cfg = S.TalkerConfig().small(talker_layers=2, predictor_layers=1)
    w = S.make_talker_weights(cfg, seed=0)
    w.update(S.make_text_weights(cfg, seed=0, text_vocab=TEXT_VOCAB, text_hidden=TEXT_HIDDEN))
    model = q3t.Model(cfg, w, kv_pages=256, max_active=2)
    yield cfg, w, model, O.OracleTalker(cfg, w)
    model.close()


def _close(gpu, ref, what):
    err = np.abs(gpu - ref)
    bound = max(2e-2, 1e-2 * np.abs(ref).max())
    assert err.max() <= bound, f"{what}: max err {err.max():.3e}"
    rel = np.linalg.norm(gpu - ref) / np.linalg.norm(ref)
    assert rel <= 1e-2, f"{what}: relative L2 {rel:.3e}"


@pytest.mark.parametrize("n", [1, 64, 70])
def test_text_projection_matches_oracle(text_model, n):
    cfg, w, model, ot = text_model
    ids = np.random.default_rng([n, 3]).integers(0, TEXT_VOCAB, n)
    ids[0] = TEXT_VOCAB - 1
    got = model.text_project(ids)
    ref = ot.text_project(ids)
    assert got.shape == (n, cfg.talker.hidden)
    assert np.array_equal(got, S.bf16_round(got)), "rows hold bf16 values"
    _close(got, ref, f"text projection n={n}")
    assert (got == ref).mean() >= 0.95


def test_text_projection_rejects_bad_ids(text_model):
    cfg, w, model, ot = text_model
    for bad in ([TEXT_VOCAB], [-1], [3, TEXT_VOCAB + 7]):
        with pytest.raises(q3t.Q3TError) as e:
            model.text_project(np.array(bad))
        assert e.value.status == 1  # INVALID_INPUT
    assert model.text_project(np.zeros(0, np.int64)).shape == (0, cfg.talker.hidden)


def test_text_projection_absent_is_an_error():
    cfg = S.TalkerConfig().small(talker_layers=1, predictor_layers=1)
    model = q3t.Model(cfg, S.make_talker_weights(cfg, seed=0), kv_pages=64, max_active=1)
    with pytest.raises(q3t.Q3TError):
        model.text_project(np.array([1, 2, 3]))
    model.close()


def test_session_from_text_ids(text_model):
    """64 prompt ids -> device text projection -> prefill + teacher-forced
    frames, against the oracle fed its own projection of the same ids."""
    cfg, w, model, ot = text_model
    ids = np.random.default_rng(0).integers(0, TEXT_VOCAB, 64)
    _, trailing, pad = S.synthetic_talker_inputs(cfg, 1, seed=0)
    prompt_gpu, prompt_ref = model.text_project(ids), ot.text_project(ids)
    codes = S.teacher_codes(4, seed=5)
    sess = model.session(prompt_gpu, trailing, pad, max_new_tokens=4, forced_first=int(codes[0, 0]),
                         first_logits=True)
    og = O.OracleGenerator(ot, prompt_ref, trailing, pad, max_new_tokens=4, forced_first=int(codes[0, 0]))
    _close(sess.first_logits, og.first_logits, "first logits")
    for f in range(3):
        _, tl, pl, _ = sess.step_forced(codes[f])
        _, otl, opl, _ = og.step(forced=codes[f])
        _close(tl, otl, f"talker logits frame {f}")
        _close(pl, opl, f"predictor logits frame {f}")
    sess.close()


# Control ids of the reference's compiler fixture for an explicit language
# (execution/compiler/tests.rs:108-124): [think, think_bos, language,
# think_eos, pad, bos]; text control ids inside the synthetic text vocabulary.
SEED_CONTROLS = {"tts_bos_token_id": TEXT_VOCAB - 3, "tts_eos_token_id": TEXT_VOCAB - 2,
                 "tts_pad_token_id": TEXT_VOCAB - 1,
                 "codec_prefix_ids": [2050, 2052, 3001, 2053, 2049, 2048], "codec_pad_id": 2049, "codec_bos_id": 2048}


@pytest.mark.parametrize("n_text,n_lead", [(8, 0), (40, 0), (90, 12)])
def test_session_seed_matches_oracle(text_model, n_text, n_lead):
    """q3t_session_seed (build_non_streaming_seed, session_seed.rs:151-215) on
    the device vs the oracle's assembly: same rows (text projection tolerance
    above), same row count, the pad embedding = P(tts_pad)."""
    cfg, w, model, ot = text_model
    g = np.random.default_rng([n_text, n_lead])
    text = g.integers(0, TEXT_VOCAB - 3, n_text)
    lead = g.integers(0, TEXT_VOCAB - 3, n_lead) if n_lead else None
    got, pad = model.session_seed(text, SEED_CONTROLS, leading_ids=lead)
    ref, ref_pad = ot.session_seed(text, SEED_CONTROLS, leading_ids=lead)
    assert got.shape == ref.shape == (n_lead + 3 + 5 + (n_text - 8) + 2, cfg.talker.hidden)
    assert np.array_equal(got, S.bf16_round(got)), "rows hold bf16 values"
    _close(got, ref, f"seed rows n_text={n_text}")
    _close(pad, ref_pad, "pad embedding")


def test_session_seed_rejects_bad_input(text_model):
    cfg, w, model, ot = text_model
    text = np.arange(20, dtype=np.int64)
    for bad_text, ctl in ((text[:7], SEED_CONTROLS),
                          (text, dict(SEED_CONTROLS, codec_prefix_ids=[2048])),
                          (text, dict(SEED_CONTROLS, codec_pad_id=cfg.talker.vocab)),
                          (text, dict(SEED_CONTROLS, tts_pad_token_id=TEXT_VOCAB))):
        with pytest.raises(q3t.Q3TError) as e:
            model.session_seed(bad_text, ctl)
        assert e.value.status == 1  # INVALID_INPUT


@pytest.mark.parametrize("recipe,ref_frames", [("xvector", 0), ("icl", 3), ("icl", 40)])
def test_voice_clone_seed_matches_oracle(text_model, recipe, ref_frames):
    """q3t_session_seed_voice_clone (build_voice_clone_seed,
    session_seed.rs:248-322) on the device vs the oracle's assembly, for the
    x-vector recipe and the in-context recipe with fewer reference frames
    than text rows (the excess text trails) and more (pad rows fill the text
    side): same row counts, bf16 rows within the text projection tolerance,
    the rows that hold no projected text (x-vector sum, reference frame
    sums) bit-identical where the oracle's text term is identical too."""
    cfg, w, model, ot = text_model
    g = np.random.default_rng([7, ref_frames])
    H, G = cfg.talker.hidden, cfg.n_groups
    text = g.integers(0, TEXT_VOCAB - 3, 20)
    spk = g.standard_normal(H).astype(np.float32)
    kw = {}
    if recipe == "icl":
        kw = dict(ref_text_ids=g.integers(0, TEXT_VOCAB - 3, 16),
                  ref_codes=np.concatenate([g.integers(0, cfg.talker.vocab, (1, ref_frames)),
                                            g.integers(0, cfg.predictor.vocab, (G - 1, ref_frames))]))
    got, trail, pad = model.session_seed_voice_clone(text, SEED_CONTROLS, spk, **kw)
    ref, ref_trail, ref_pad = ot.session_seed_voice_clone(text, SEED_CONTROLS, spk, **kw)
    assert got.shape == ref.shape and trail.shape == ref_trail.shape
    n = len(SEED_CONTROLS["codec_prefix_ids"])
    if recipe == "xvector":
        assert got.shape[0] == 3 + n + 1 and trail.shape[0] == 12 - 1 + 1
    else:
        assert got.shape[0] == 3 + n + 1 + ref_frames
        text_len = (16 - 5) + 12 + 1
        assert trail.shape[0] == (text_len - 1 - ref_frames if text_len > 1 + ref_frames else 1)
    for a in (got, trail, pad):
        assert np.array_equal(a, S.bf16_round(a)), "rows hold bf16 values"
    _close(got, ref, f"voice-clone seed rows ({recipe}, {ref_frames} frames)")
    _close(trail, ref_trail, "trailing text")
    _close(pad, ref_pad, "pad embedding")
    if recipe == "icl" and ref_frames > 1 + 24 - 1:  # pad rows past the text: P(pad) + frame sum
        pad_rows = slice(3 + n + 24, 3 + n + 1 + ref_frames)
        exact = np.array_equal(pad, ref_pad)
        assert not exact or np.array_equal(got[pad_rows], ref[pad_rows])


def test_voice_clone_seed_rejects_bad_input(text_model):
    cfg, w, model, ot = text_model
    text = np.arange(20, dtype=np.int64)
    spk = np.zeros(cfg.talker.hidden, np.float32)
    G = cfg.n_groups
    codes = np.zeros((G, 4), np.int64)
    bad_codes = codes.copy()
    bad_codes[3, 1] = cfg.predictor.vocab  # a predictor-group code outside its vocabulary
    for args, kw in (((text[:7], SEED_CONTROLS, spk), {}),
                     ((text, dict(SEED_CONTROLS, codec_prefix_ids=[2048]), spk), {}),
                     ((text, SEED_CONTROLS, spk), dict(ref_text_ids=text[:4], ref_codes=codes)),
                     ((text, SEED_CONTROLS, spk), dict(ref_text_ids=text, ref_codes=bad_codes)),
                     ((text, SEED_CONTROLS, spk), dict(ref_text_ids=text))):
        with pytest.raises(q3t.Q3TError) as e:
            model.session_seed_voice_clone(*args, **kw)
        assert e.value.status == 1  # INVALID_INPUT

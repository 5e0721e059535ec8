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

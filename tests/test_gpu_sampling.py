"""Non-greedy device sampling (sample_token, talker/infer/sampling.rs:33-90)
against the oracle: temperature, top-k, top-p and the categorical draw on the
same logits and the same uniform draw u give the same token, and the set of
candidates the device keeps after suppress / top-k / top-p equals an
independent numpy restatement of the reference's filters.  Token ids are
compared exactly (integer work)."""
import numpy as np
import pytest

import oracle as O
import q3t
import synthetic as S

pytestmark = pytest.mark.gpu

CASES = [  # (do_sample, temperature, top_k, top_p)
    (1, 0.9, 50, 0.8),   # the predictor's default recipe shape
    (1, 0.7, 0, 1.0),    # temperature only
    (1, 1.0, 10, 1.0),   # top-k only
    (1, 1.3, 0, 0.6),    # top-p only
    (1, 1.0, 1, 1.0),    # top-k 1 = argmax (the reference's known answer)
    (0, 1.0, 0, 1.0),    # greedy
]
DRAWS = [0.0, 0.013, 0.25, 0.5, 0.777, 0.97, 0.9999]


@pytest.fixture(scope="module")
def model():
    cfg = S.TalkerConfig().small(talker_layers=1, predictor_layers=1)
    m = q3t.Model(cfg, S.make_talker_weights(cfg, seed=0), kv_pages=16, max_active=1)
    yield m
    m.close()


def kept_reference(logits, do_sample, temperature, top_k, top_p, suppress):
    """Candidates left by sampling.rs:51-90 (suppress mask, temperature, top-k
    threshold at the k-th largest value, top-p over the sorted softmax keeping
    a token while the mass before it is below top_p)."""
    lg = logits.astype(np.float32).copy()
    if suppress is not None:
        lg[suppress] = -np.inf
    if not do_sample:
        return np.isfinite(lg)
    lg = lg / np.float32(max(temperature, 1e-5))
    V = lg.shape[0]
    if 0 < top_k < V:
        kth = np.sort(lg)[::-1][top_k - 1]
        lg[lg < kth] = -np.inf
    if 0 < top_p < 1:
        order = np.lexsort((np.arange(V), -lg))  # descending, ties by index
        sv = lg[order]
        e = np.exp(sv - sv[0], dtype=np.float32)
        total = np.float32(0)
        for x in e:  # f32 running sums in sorted order, as the reference's cumsum
            total = np.float32(total + x)
        cum = np.float32(0)
        for i in range(V):
            pi = np.float32(e[i] / total)
            cum = np.float32(cum + pi)
            if not np.float32(cum - pi) < np.float32(top_p):
                lg[order[i]] = -np.inf
    return np.isfinite(lg)


@pytest.mark.parametrize("V", [2048, 3072])
@pytest.mark.parametrize("case", CASES)
def test_device_sampler_matches_oracle(model, V, case):
    do_sample, temp, top_k, top_p = case
    g = np.random.default_rng([V, int(temp * 10), top_k, int(top_p * 10)])
    logits = (g.standard_normal(V) * 3.0).astype(np.float32)
    suppress = np.sort(g.choice(V, size=64, replace=False)).astype(np.int64)
    smp = q3t.sampling(do_sample=do_sample, temperature=temp, top_k=top_k, top_p=top_p)
    osmp = O.sampling(do_sample=do_sample, temperature=temp, top_k=top_k, top_p=top_p)
    ref_kept = kept_reference(logits, do_sample, temp, top_k, top_p, suppress)
    for u in DRAWS:
        u32 = float(np.float32(u))
        tok, kept = model.sample_logits(logits, smp, u32, suppress=suppress)
        ref = O.lib().orc_sample_token(O.fp(logits), V, osmp, O.ip(suppress), len(suppress), u32)
        assert tok == ref, (case, u, tok, ref)
        assert kept[tok] and tok not in set(suppress.tolist())
        np.testing.assert_array_equal(kept, ref_kept)
    if top_k == 1 or not do_sample:
        lg = logits.copy()
        lg[suppress] = -np.inf
        assert tok == int(np.argmax(lg))


def test_categorical_draw_covers_the_distribution(model):
    """Sweeping u over [0, 1) visits the candidates in index order, each for a
    share of u equal to its softmax probability (inverse CDF)."""
    V = 2048
    g = np.random.default_rng(7)
    logits = (g.standard_normal(V) * 2.0).astype(np.float32)
    smp = q3t.sampling(do_sample=1, temperature=1.0, top_k=8)
    kept = kept_reference(logits, 1, 1.0, 8, 1.0, None)
    ids = np.flatnonzero(kept)
    p = np.exp(logits[ids] - logits[ids].max())
    edges = np.cumsum(p / p.sum())
    for i, uid in enumerate(ids):
        lo = 0.0 if i == 0 else edges[i - 1]
        mid = float(np.float32((lo + edges[i]) / 2))
        tok, _ = model.sample_logits(logits, smp, mid)
        assert tok == uid, (i, tok, uid)


def test_sampler_rejects_bad_arguments(model):
    smp = q3t.sampling(do_sample=1)
    with pytest.raises(q3t.Q3TError) as e:
        model.sample_logits(np.zeros(8, np.float32), smp, 1.0)
    assert e.value.status == q3t.INVALID_INPUT
    with pytest.raises(q3t.Q3TError):
        model.sample_logits(np.zeros(5000, np.float32), smp, 0.5)

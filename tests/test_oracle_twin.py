"""The oracle's hot-path restatement against an independent float64 numpy
restatement written from the reference sources (no shared code with
oracle.c): the talker decoder stack (talker/network/layer.rs:23-44,
attention.rs:31-134, mlp.rs:18-23, rope.rs:16-56, model.rs:33-113), the
code-predictor frame (talker/infer/mod.rs:434-578, predictor.rs:33-62) and
the speech-tokenizer decoder (codec/network/decoder.rs, wave.rs, conv.rs,
activation.rs, codebook.rs).

Both sides use the oracle's numerics model: bf16 weights, Linear inputs
rounded to bf16 with wide accumulation, q / k / v rounded to bf16 after the
per-head norm and RoPE (the cache holds the model dtype), residual stream
wide.  The twin accumulates (and computes its RoPE angles) in float64, the
oracle in float32.  Through one layer they agree to float32 rounding plus the
occasional bf16 rounding flip of a q / k / v or Linear input element: a row
agrees to ~1e-7 until a flip, after which it and every row that reads the
flipped cache entry or input sit near 2e-3 relative L2 (measured over
several seeds).  Rows are held to 5e-3; a transcription error (another RoPE
pairing, GQA head map, mask, norm or code order) gives errors of order 1."""
import numpy as np
import pytest

import oracle as O
import synthetic as S

REL = 5e-3
REL_STACK = REL


def rel_err(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


def bf(x):
    return O.bf16_round(np.asarray(x, np.float32)).astype(np.float64)


def rmsnorm(x, g, eps):
    return x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps) * g


def silu(x):
    return x / (1.0 + np.exp(-x))


class TwinStack:
    """Decoder stack of the talker / code predictor in float64 with dense
    per-layer K/V caches [n_kv][len][head_dim]."""

    def __init__(self, w, prefix, c):
        self.c = c
        self.L = []
        for l in range(c.n_layers):
            p = f"{prefix}.layers.{l}"
            g = lambda n: np.asarray(w[f"{p}.{n}.weight"], np.float64)
            self.L.append(dict(inn=g("input_layernorm"), post=g("post_attention_layernorm"),
                               q=g("self_attn.q_proj"), k=g("self_attn.k_proj"), v=g("self_attn.v_proj"),
                               o=g("self_attn.o_proj"), qn=g("self_attn.q_norm"), kn=g("self_attn.k_norm"),
                               gate=g("mlp.gate_proj"), up=g("mlp.up_proj"), down=g("mlp.down_proj")))
        self.norm = np.asarray(w[f"{prefix}.norm.weight"], np.float64)
        self.k = [np.zeros((c.n_kv, 0, c.head_dim)) for _ in range(c.n_layers)]
        self.v = [np.zeros((c.n_kv, 0, c.head_dim)) for _ in range(c.n_layers)]

    def rope(self, x, pos):
        """x [S][heads][hd] -> x * cos + rotate_half(x) * sin, rotate_half(x) =
        cat(-x2, x1); angles pos * theta^(-i / half), duplicated over halves."""
        hd = x.shape[-1]
        half = hd // 2
        inv = np.asarray(self.c.theta, np.float64) ** (-np.arange(half) / half)
        ang = np.asarray(pos, np.float64)[:, None] * inv[None]
        cos = np.cos(np.concatenate([ang, ang], -1))[:, None, :]
        sin = np.sin(np.concatenate([ang, ang], -1))[:, None, :]
        rot = np.concatenate([-x[..., half:], x[..., :half]], -1)
        return x * cos + rot * sin

    def forward(self, x):
        c = self.c
        S_len = x.shape[0]
        nh, nkv, hd = c.n_heads, c.n_kv, c.head_dim
        start = self.k[0].shape[1]
        pos = start + np.arange(S_len)
        x = np.asarray(x, np.float64).copy()
        for l, W in enumerate(self.L):
            h = bf(rmsnorm(x, W["inn"], c.eps))
            q = (h @ W["q"].T).reshape(S_len, nh, hd)
            k = (h @ W["k"].T).reshape(S_len, nkv, hd)
            v = (h @ W["v"].T).reshape(S_len, nkv, hd)
            q = bf(self.rope(rmsnorm(q, W["qn"], c.eps), pos))
            k = bf(self.rope(rmsnorm(k, W["kn"], c.eps), pos))
            v = bf(v)
            self.k[l] = np.concatenate([self.k[l], k.transpose(1, 0, 2)], 1)
            self.v[l] = np.concatenate([self.v[l], v.transpose(1, 0, 2)], 1)
            Lk = self.k[l].shape[1]
            rep = nh // nkv
            out = np.zeros((S_len, nh, hd))
            for hh in range(nh):  # query head hh reads kv head hh // rep (repeat_dim over kv heads)
                sc = q[:, hh, :] @ self.k[l][hh // rep].T / np.sqrt(hd)
                if start == 0 and S_len == Lk and S_len > 1:  # causal mask iff seq_len == key_len
                    sc = np.where(np.triu(np.ones((S_len, Lk), bool), 1), -np.inf, sc)
                p = np.exp(sc - sc.max(-1, keepdims=True))
                p /= p.sum(-1, keepdims=True)
                out[:, hh, :] = p @ self.v[l][hh // rep]
            x = x + bf(out.reshape(S_len, nh * hd)) @ W["o"].T
            h = bf(rmsnorm(x, W["post"], c.eps))
            a = bf(silu(h @ W["gate"].T) * (h @ W["up"].T))
            x = x + a @ W["down"].T
        return rmsnorm(x, self.norm, c.eps)


@pytest.fixture(scope="module")
def talker():
    cfg = S.TalkerConfig().small(talker_layers=1, predictor_layers=1)
    w = S.make_talker_weights(cfg, seed=0)
    return cfg, w, O.OracleTalker(cfg, w)


def test_talker_stack_of_three_layers():
    """Composition: three layers and the final norm, a 5-token prompt."""
    cfg = S.TalkerConfig().small(talker_layers=3, predictor_layers=1)
    w = S.make_talker_weights(cfg, seed=1)
    ot = O.OracleTalker(cfg, w)
    x = (np.random.default_rng(5).standard_normal((5, cfg.talker.hidden)) * 0.5).astype(np.float32)
    kvs, _ = ot.make_caches("talker", cap=16)
    ref = ot.stack_forward("talker", kvs, x)
    got = TwinStack(w, "talker.model", cfg.talker).forward(x)
    assert rel_err(got, ref) <= REL_STACK, rel_err(got, ref)


def test_talker_layer_prefill_and_decode(talker):
    """One decoder layer: a 7-token prompt from an empty cache (causal mask),
    then two single tokens at positions 7 and 8 (no mask), and the codec
    head."""
    cfg, w, ot = talker
    g = np.random.default_rng(3)
    x = (g.standard_normal((7, cfg.talker.hidden)) * 0.5).astype(np.float32)
    twin = TwinStack(w, "talker.model", cfg.talker)
    kvs, _ = ot.make_caches("talker", cap=64)
    ref = ot.stack_forward("talker", kvs, x)
    got = twin.forward(x)
    assert rel_err(got, ref) <= REL, rel_err(got, ref)
    head = np.asarray(w["talker.codec_head.weight"], np.float64)
    for step in range(2):
        e = (g.standard_normal((1, cfg.talker.hidden)) * 0.5).astype(np.float32)
        ref = ot.stack_forward("talker", kvs, e)
        got = twin.forward(e)
        assert rel_err(got, ref) <= REL, (step, rel_err(got, ref))
        lg_ref = ot.codec_head(ref)[0]
        lg = bf(got) @ head.T
        assert rel_err(lg[0], lg_ref) <= REL


def test_predictor_frame(talker):
    """generate_code_predictor_groups with teacher-forced codes: the prefill
    pair [talker hidden, talker codec embedding of code 0] (causal), lm_head 0
    on its last position, then 14 one-token passes of the previous code's
    predictor embedding, each followed by its lm_head."""
    cfg, w, ot = talker
    G = cfg.n_groups
    g = np.random.default_rng(4)
    hidden = (g.standard_normal(cfg.talker.hidden) * 0.7).astype(np.float32)
    forced = g.integers(0, cfg.predictor.vocab, size=G).astype(np.int64)
    codes, ref = ot.predict_frame(hidden, int(forced[0]), forced=forced)
    np.testing.assert_array_equal(codes, forced)
    twin = TwinStack(w, "talker.code_predictor.model", cfg.predictor)
    emb0 = np.asarray(w["talker.model.codec_embedding.weight"], np.float64)
    x2 = np.stack([np.asarray(hidden, np.float64), emb0[forced[0]]])
    out = twin.forward(x2)[1:]
    heads = [np.asarray(w[f"talker.code_predictor.lm_head.{j}.weight"], np.float64) for j in range(G - 1)]
    got = [bf(out) @ heads[0].T]
    for j in range(1, G - 1):
        e = np.asarray(w[f"talker.code_predictor.model.codec_embedding.{j - 1}.weight"], np.float64)[forced[j]]
        out = twin.forward(e[None])
        got.append(bf(out) @ heads[j].T)
    got = np.concatenate(got)
    assert got.shape == ref.shape == (G - 1, cfg.predictor.vocab)
    for j in range(G - 1):
        assert rel_err(got[j], ref[j]) <= REL, (j, rel_err(got[j], ref[j]))


def test_twin_detects_another_rope_pairing(talker):
    """The tolerance discriminates: the same layer with RoPE on adjacent pairs
    (x[2i], x[2i+1]) instead of rotate-half misses by orders of magnitude."""
    cfg, w, ot = talker

    class Interleaved(TwinStack):
        def rope(self, x, pos):
            half = x.shape[-1] // 2
            inv = np.asarray(self.c.theta, np.float64) ** (-np.arange(half) / half)
            ang = np.asarray(pos, np.float64)[:, None, None] * inv[None, None]
            x0, x1 = x[..., 0::2], x[..., 1::2]
            out = np.empty_like(x)
            out[..., 0::2] = x0 * np.cos(ang) - x1 * np.sin(ang)
            out[..., 1::2] = x1 * np.cos(ang) + x0 * np.sin(ang)
            return out

    x = (np.random.default_rng(9).standard_normal((6, cfg.talker.hidden)) * 0.5).astype(np.float32)
    kvs, _ = ot.make_caches("talker", cap=16)
    ref = ot.stack_forward("talker", kvs, x)
    assert rel_err(Interleaved(w, "talker.model", cfg.talker).forward(x), ref) > 20 * REL


# ---------------------------------------------------------------------------
# speech-tokenizer decoder (no bf16 rounding points: the oracle's codec runs
# in f32 throughout, the twin in float64, so they agree to float32 rounding)
# ---------------------------------------------------------------------------
REL_CODEC = 1e-4


def causal_conv(x, w, b, dilation=1, groups=1):
    """AudioCodecCausalConv1d (conv.rs:33-83) with stride 1: constant-zero left
    pad of (k - 1) * dilation (conv1d_padding gives no extra right pad at
    stride 1), then Conv1d; x [Cin][L], w [Cout][Cin / groups][k]."""
    co, cig, k = w.shape
    L = x.shape[1]
    pad = (k - 1) * dilation
    xp = np.concatenate([np.zeros((x.shape[0], pad)), x], 1)
    out = np.zeros((co, L))
    if groups == 1:
        for j in range(k):
            out += w[:, :, j] @ xp[:, j * dilation:j * dilation + L]
    else:  # depthwise (groups == channels)
        for j in range(k):
            out += w[:, 0, j][:, None] * xp[:, j * dilation:j * dilation + L]
    return out + b[:, None]


def conv_transpose(x, w, b, stride):
    """AudioCodecCausalTransConv1d (conv.rs:19-31): ConvTranspose1d (weight
    [Cin][Cout][k], output (L - 1) * stride + k), then trim k - stride steps
    from both ends."""
    ci, co, k = w.shape
    L = x.shape[1]
    out = np.zeros((co, (L - 1) * stride + k))
    for j in range(k):
        out[:, j:j + (L - 1) * stride + 1:stride] += w[:, :, j].T @ x
    out += b[:, None]
    trim = max(k - stride, 0)
    return out[:, trim:out.shape[1] - trim] if trim else out


def snake_beta(x, alpha, beta):
    """activation.rs:16-37: x + sin^2(exp(alpha) x) / (exp(beta) + 1e-9)."""
    a = np.exp(alpha)[:, None]
    return x + np.sin(a * x) ** 2 / (np.exp(beta)[:, None] + 1e-9)


def rope_adjacent_pairs(x, theta):
    """burn::nn::RotaryEncoding at offset 0 on x [T][heads][d]: rotates the
    adjacent pairs (x[2i], x[2i + 1]) by t * theta^(-2i / d)."""
    T, _, d = x.shape
    inv = np.asarray(theta, np.float64) ** (-(2.0 * np.arange(d // 2)) / d)
    ang = np.arange(T, dtype=np.float64)[:, None, None] * inv[None, None]
    x0, x1 = x[..., 0::2], x[..., 1::2]
    out = np.empty_like(x)
    out[..., 0::2] = x0 * np.cos(ang) - x1 * np.sin(ang)
    out[..., 1::2] = x0 * np.sin(ang) + x1 * np.cos(ang)
    return out


def twin_codec_decode(c, w, codes):
    """Qwen3TtsAudioCodecDecoder::forward (decoder.rs:250-278) for one item,
    codes [n_q][T] -> samples [n]."""
    f = lambda n: np.asarray(w[n], np.float64)
    T = codes.shape[1]

    def centroids(grp, i):  # codebook.rs:4-11
        p = f"decoder.quantizer.{grp}.vq.layers.{i}._codebook"
        return f(p + ".embedding_sum") / np.maximum(f(p + ".cluster_usage"), 1e-6)[:, None]

    # quantizer (decoder.rs:205-247): gather-sum per group, 1x1 output_proj each, summed
    sem = sum(centroids("rvq_first", i)[codes[i]] for i in range(c.n_semantic))
    ac = sum(centroids("rvq_rest", i)[codes[c.n_semantic + i]] for i in range(c.n_q - c.n_semantic))
    x = f("decoder.quantizer.rvq_first.output_proj.weight")[:, :, 0] @ sem.T
    x = x + f("decoder.quantizer.rvq_rest.output_proj.weight")[:, :, 0] @ ac.T
    x = causal_conv(x, f("decoder.pre_conv.conv.weight"), f("decoder.pre_conv.conv.bias"))
    # pre-transformer (decoder.rs:173-194), on [T][latent]
    pt = "decoder.pre_transformer"
    h = x.T @ f(f"{pt}.input_proj.weight").T + f(f"{pt}.input_proj.bias")
    nh, nkv, hd = c.n_heads, c.n_kv, c.head_dim
    for l in range(c.n_layers):
        p = f"{pt}.layers.{l}"
        n = rmsnorm(h, f(f"{p}.input_layernorm.weight"), c.eps)
        q = rope_adjacent_pairs((n @ f(f"{p}.self_attn.q_proj.weight").T).reshape(T, nh, hd), c.theta)
        k = rope_adjacent_pairs((n @ f(f"{p}.self_attn.k_proj.weight").T).reshape(T, nkv, hd), c.theta)
        v = (n @ f(f"{p}.self_attn.v_proj.weight").T).reshape(T, nkv, hd)
        att = np.zeros((T, nh, hd))
        for hh in range(nh):  # no mask: every frame sees every frame
            kv = hh // (nh // nkv)
            sc = q[:, hh] @ k[:, kv].T / np.sqrt(hd)
            pr = np.exp(sc - sc.max(-1, keepdims=True))
            att[:, hh] = (pr / pr.sum(-1, keepdims=True)) @ v[:, kv]
        h = h + (att.reshape(T, nh * hd) @ f(f"{p}.self_attn.o_proj.weight").T) * f(f"{p}.self_attn_layer_scale.scale")
        n = rmsnorm(h, f(f"{p}.post_attention_layernorm.weight"), c.eps)
        m = silu(n @ f(f"{p}.mlp.gate_proj.weight").T) * (n @ f(f"{p}.mlp.up_proj.weight").T)
        h = h + (m @ f(f"{p}.mlp.down_proj.weight").T) * f(f"{p}.mlp_layer_scale.scale")
    h = rmsnorm(h, f(f"{pt}.norm.weight"), c.eps) @ f(f"{pt}.output_proj.weight").T + f(f"{pt}.output_proj.bias")
    x = h.T
    # upsampling: transposed conv (k = stride = ratio) + ConvNeXt block (wave.rs:96-108)
    from math import erf
    gelu = np.vectorize(lambda v: 0.5 * v * (1.0 + erf(v / np.sqrt(2.0))))
    for u, r in enumerate(c.up_ratios):
        p = f"decoder.upsample.{u}"
        x = conv_transpose(x, f(f"{p}.0.conv.weight"), f(f"{p}.0.conv.bias"), r)
        d = causal_conv(x, f(f"{p}.1.dwconv.conv.weight"), f(f"{p}.1.dwconv.conv.bias"), groups=x.shape[0]).T
        mu = d.mean(-1, keepdims=True)
        var = ((d - mu) ** 2).mean(-1, keepdims=True)
        d = (d - mu) / np.sqrt(var + 1e-6) * f(f"{p}.1.norm.weight") + f(f"{p}.1.norm.bias")
        d = gelu(d @ f(f"{p}.1.pwconv1.weight").T + f(f"{p}.1.pwconv1.bias"))
        d = d @ f(f"{p}.1.pwconv2.weight").T + f(f"{p}.1.pwconv2.bias")
        x = x + (d * f(f"{p}.1.gamma")).T
    # wave decoder (wave.rs:12-94, config.rs:350-377, 539-585)
    x = causal_conv(x, f("decoder.decoder.0.conv.weight"), f("decoder.decoder.0.conv.bias"))
    for i, r in enumerate(c.rates):
        p = f"decoder.decoder.{i + 1}.block"
        x = snake_beta(x, f(f"{p}.0.alpha"), f(f"{p}.0.beta"))
        x = conv_transpose(x, f(f"{p}.1.conv.weight"), f(f"{p}.1.conv.bias"), r)
        for ru, dil in zip(range(3), (1, 3, 9)):
            q = f"{p}.{ru + 2}"
            y = snake_beta(x, f(f"{q}.act1.alpha"), f(f"{q}.act1.beta"))
            y = causal_conv(y, f(f"{q}.conv1.conv.weight"), f(f"{q}.conv1.conv.bias"), dilation=dil)
            y = snake_beta(y, f(f"{q}.act2.alpha"), f(f"{q}.act2.beta"))
            x = x + causal_conv(y, f(f"{q}.conv2.conv.weight"), f(f"{q}.conv2.conv.bias"))
    n = len(c.rates)
    x = snake_beta(x, f(f"decoder.decoder.{n + 1}.alpha"), f(f"decoder.decoder.{n + 1}.beta"))
    x = causal_conv(x, f(f"decoder.decoder.{n + 2}.conv.weight"), f(f"decoder.decoder.{n + 2}.conv.bias"))
    return np.clip(x[0], -1.0, 1.0)


@pytest.mark.parametrize("T", [1, 5])
def test_codec_decoder(T):
    """Full-size decoder config at small T against the oracle's f32 decode."""
    c = S.CodecConfig()
    w = S.make_codec_weights(c, seed=0)
    codes = np.random.default_rng([T, 17]).integers(0, c.codebook_size, size=(c.n_q, T), dtype=np.int64)
    ref = O.OracleCodec(c, w).decode(codes[None])[0]
    got = twin_codec_decode(c, w, codes)
    assert got.shape == ref.shape == (c.out_len(T),)
    assert rel_err(got, ref) <= REL_CODEC, rel_err(got, ref)


@pytest.mark.slow
def test_argmax_noise_floor():
    """How well two correct implementations of the full-depth path can agree
    on the argmax of seed-0 random-init logits: the oracle against itself
    built with double accumulation (liboracle_wide.so: the same math and bf16
    rounding points, another summation precision).  Their logits differ by
    ~4e-3 RMS through cascading bf16 rounding flips, and the random-init
    logits have many top-2 gaps below that, so raw argmax agreement sits near
    99 % (99.05 % over 1158 rows measured when this test was written), under
    the 99.5 % the path's tolerance names.  The GPU parity tests hold the GPU
    to this floor; here both builds must agree on every row whose top-2
    margin exceeds 2e-2."""
    cfg = S.TalkerConfig()
    w = S.make_talker_weights(cfg, seed=0)
    ot = O.OracleTalker(cfg, w)

    def run(variant, seed, frames=8):
        prev = O.use_library(variant)
        try:
            prompt, trailing, pad = S.synthetic_talker_inputs(cfg, 64, seed=seed)
            codes = S.teacher_codes(frames + 1, seed=seed)
            og = O.OracleGenerator(ot, prompt, trailing, pad, max_new_tokens=frames + 1,
                                   forced_first=int(codes[0, 0]))
            rows = [og.first_logits[None]]
            for f in range(frames):
                _, tl, pl, _ = og.step(forced=codes[f])
                rows += [pl, tl[None]]
            return rows
        finally:
            O.use_library(prev)

    agree = total = 0
    for seed in range(3):
        a, b = run("liboracle.so", seed), run("liboracle_wide.so", seed)
        for ra, rb in zip(a, b):
            same = ra.argmax(-1) == rb.argmax(-1)
            top2 = np.sort(ra, -1)[:, -2:]
            assert same[(top2[:, 1] - top2[:, 0]) > 2e-2].all()
            agree += int(same.sum())
            total += len(same)
    floor = agree / total
    print(f"\noracle vs wide-accumulation oracle: argmax agreement {floor:.4f} over {total} rows")
    assert floor >= 0.98

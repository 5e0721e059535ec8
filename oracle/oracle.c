/*
 * CPU oracle for the Qwen3-TTS synthesis hot path — TEST INFRASTRUCTURE ONLY
 * (checker and timed CPU baseline; never part of the product).  See oracle.h
 * for the parity status and the precision model.  Every function cites the
 * reference file:line (paths inside onenewcode/tts-rs, crate tts_qwen3_tts
 * unless stated) whose behaviour it restates.
 */
#include "oracle.h"

#include <math.h>
#include <omp.h>
#include <stdlib.h>
#include <string.h>

#define MAXF(a, b) ((a) > (b) ? (a) : (b))

void orc_set_threads(int n) {
  if (n > 0) omp_set_num_threads(n);
}
int orc_get_threads(void) { return omp_get_max_threads(); }

/* round-to-nearest-even f32 -> bf16 -> f32 (load-time dtype cast,
 * loading/load_adapter.rs:18-46) */
float orc_bf16_round(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  if ((u & 0x7f800000u) == 0x7f800000u) {
    if (u & 0x7fffffu) u |= 0x400000u;
    u &= 0xffff0000u;
  } else {
    u += 0x7fffu + ((u >> 16) & 1u);
    u &= 0xffff0000u;
  }
  memcpy(&x, &u, 4);
  return x;
}

void orc_bf16_round_array(float *x, int64_t n) {
  for (int64_t i = 0; i < n; i++) x[i] = orc_bf16_round(x[i]);
}

/* 8-lane dot product: keeps the loop vectorisable without -ffast-math.
 * Built with -DORC_WIDE_ACC (liboracle_wide.so) it accumulates in double
 * instead: the same math in another summation precision, which measures how
 * far two correct implementations of this path drift apart through bf16
 * rounding flips alone (the argmax noise floor on random-init weights). */
#ifdef ORC_WIDE_ACC
static float dot8(const float *a, const float *b, int n) {
  double s = 0.0;
  for (int k = 0; k < n; k++) s += (double)a[k] * (double)b[k];
  return (float)s;
}
#else
static float dot8(const float *a, const float *b, int n) {
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  int k = 0;
  for (; k + 8 <= n; k += 8)
    for (int j = 0; j < 8; j++) acc[j] += a[k + j] * b[k + j];
  float s = 0.f;
  for (; k < n; k++) s += a[k] * b[k];
  for (int j = 0; j < 8; j++) s += acc[j];
  return s;
}
#endif

/* burn::nn::Linear on rows (weights in PyTorch [out][in] layout); the
 * reference runs Linear in the runtime dtype, restated as bf16 inputs with
 * f32 accumulation when round_in is set. */
static void linear_rows(const float *W, const float *bias, const float *x,
                        int S, int K, int N, float *y, int round_in) {
  const float *xr = x;
  float *tmp = NULL;
  if (round_in) {
    tmp = (float *)malloc((size_t)S * K * sizeof(float));
    for (int64_t i = 0; i < (int64_t)S * K; i++) tmp[i] = orc_bf16_round(x[i]);
    xr = tmp;
  }
#pragma omp parallel for schedule(static)
  for (int n = 0; n < N; n++) {
    const float *w = W + (size_t)n * K;
    for (int s = 0; s < S; s++)
      y[(size_t)s * N + n] = dot8(w, xr + (size_t)s * K, K) + (bias ? bias[n] : 0.f);
  }
  free(tmp);
}

void orc_linear(const float *W, const float *bias, const float *x, int S,
                int K, int N, float *y) {
  linear_rows(W, bias, x, S, K, N, y, 1);
}

/* burn::nn::RmsNorm: x / sqrt(mean(x^2) + eps) * gamma (used at
 * talker/network/layer.rs:34,41, attention.rs:49-56, model.rs:112) */
static void rmsnorm(const float *x, const float *g, int n, float eps,
                    float *out) {
  float ss = 0.f;
  for (int i = 0; i < n; i++) ss += x[i] * x[i];
  float rms = sqrtf(ss / (float)n + eps);
  for (int i = 0; i < n; i++) out[i] = (x[i] / rms) * g[i];
}

static float silu(float x) { return x / (1.f + expf(-x)); }

/* project_text_ids (execution/compiler/session_seed.rs:668-679):
 * Qwen3TtsTalkerResizeMlp (talker/network/mlp.rs:36-40) over the text
 * embedding.  emb [vocab][Ht], w1 [Ht][Ht] + b1, w2 [H][Ht] + b2 (bf16 values
 * held as f32).  Rounding points: silu(fc1 + b1) and fc2 + b2 are rounded to
 * bf16 (the model dtype); sums run in f32. */
void orc_text_project(const float *emb, const float *w1, const float *b1, const float *w2,
                      const float *b2, int Ht, int H, const int64_t *ids, int n, float *out) {
  float *x = (float *)malloc((size_t)Ht * sizeof(float));
  float *h = (float *)malloc((size_t)Ht * sizeof(float));
  for (int i = 0; i < n; i++) {
    memcpy(x, emb + (size_t)ids[i] * Ht, (size_t)Ht * sizeof(float));
    orc_linear(w1, b1, x, 1, Ht, Ht, h);
    for (int j = 0; j < Ht; j++) h[j] = orc_bf16_round(silu(h[j]));
    orc_linear(w2, b2, h, 1, Ht, H, out + (size_t)i * H);
    for (int j = 0; j < H; j++) out[(size_t)i * H + j] = orc_bf16_round(out[(size_t)i * H + j]);
  }
  free(x);
  free(h);
}

/* ------------------------------------------------------------------------ */
/* KV cache: talker/network/kv.rs:56-161                                     */
/* ------------------------------------------------------------------------ */
static void kv_copy_steps(orc_kv *c, int dst, const float *src, int src_steps,
                          int src_from, int n, float *base) {
  /* base[h][dst + i] = src[h][src_from + i], i < n, src laid out [n_kv][src_steps][hd] */
  for (int h = 0; h < c->n_kv; h++)
    memmove(base + ((size_t)h * c->cap + dst) * c->head_dim,
            src + ((size_t)h * src_steps + src_from) * c->head_dim,
            (size_t)n * c->head_dim * sizeof(float));
}

static void kv_forward_one(orc_kv *c, float *base, const float *t, int S,
                           float *out, int *ret_len) {
  int hd = c->head_dim;
  if (S >= c->cap) { /* kv.rs:86-107: keep the latest window only */
    int keep_from = S - c->cap;
    kv_copy_steps(c, 0, t, S, keep_from, c->cap, base);
    *ret_len = c->cap;
    if (out)
      for (int h = 0; h < c->n_kv; h++)
        memcpy(out + (size_t)h * c->cap * hd, t + ((size_t)h * S + keep_from) * hd,
               (size_t)c->cap * hd * sizeof(float));
    return;
  }
  int cur = c->len;
  int new_len = c->len + S;
  if (new_len > c->cap) { /* kv.rs:109-132: slide the window */
    cur = c->cap - S;
    for (int h = 0; h < c->n_kv; h++)
      memmove(base + (size_t)h * c->cap * hd, base + ((size_t)h * c->cap + S) * hd,
              (size_t)cur * hd * sizeof(float));
    new_len = c->cap;
  }
  kv_copy_steps(c, cur, t, S, 0, S, base);
  *ret_len = new_len;
  if (out)
    for (int h = 0; h < c->n_kv; h++)
      memcpy(out + (size_t)h * new_len * hd, base + (size_t)h * c->cap * hd,
             (size_t)new_len * hd * sizeof(float));
}

int orc_kv_forward(orc_kv *c, const float *k_new, const float *v_new, int S,
                   float *k_out, float *v_out) {
  int lk, lv;
  kv_forward_one(c, c->k, k_new, S, k_out, &lk);
  kv_forward_one(c, c->v, v_new, S, v_out, &lv);
  c->len = lk;
  return lk;
}

void orc_kv_reset_preserve(orc_kv *c) { c->len = 0; }

/* ------------------------------------------------------------------------ */
/* SDPA: model/nn/attention.rs:5-27 (f32; mask fill -inf; softmax; .V)       */
/* ------------------------------------------------------------------------ */
void orc_sdpa(const float *q, const float *k, const float *v,
              const uint8_t *mask, int H, int S, int L, int D, float scale,
              float *out) {
#pragma omp parallel for collapse(2) schedule(static)
  for (int h = 0; h < H; h++)
    for (int s = 0; s < S; s++) {
      float *sc = (float *)malloc((size_t)L * sizeof(float));
      const float *qs = q + ((size_t)h * S + s) * D;
      float mx = -INFINITY;
      for (int j = 0; j < L; j++) {
        float d = dot8(qs, k + ((size_t)h * L + j) * D, D) * scale;
        if (mask && mask[(size_t)s * L + j]) d = -INFINITY;
        sc[j] = d;
        mx = d > mx ? d : mx;
      }
      float sum = 0.f;
      for (int j = 0; j < L; j++) {
        sc[j] = expf(sc[j] - mx);
        sum += sc[j];
      }
      float *o = out + ((size_t)h * S + s) * D;
      for (int d = 0; d < D; d++) o[d] = 0.f;
      for (int j = 0; j < L; j++) {
        float p = sc[j] / sum;
        const float *vj = v + ((size_t)h * L + j) * D;
        for (int d = 0; d < D; d++) o[d] += p * vj[d];
      }
      free(sc);
    }
}

/* ------------------------------------------------------------------------ */
/* Decoder layer: talker/network/layer.rs:23-44, attention.rs:31-134,       */
/* mlp.rs:18-23; RoPE rope.rs:16-56 (MRoPE with equal rows, rope.rs:86-131) */
/* ------------------------------------------------------------------------ */
static void layer_forward(const orc_lm_cfg *c, const orc_layer *L, orc_kv *kv,
                          float *x, int S) {
  const int H = c->hidden, nh = c->n_heads, nkv = c->n_kv, hd = c->head_dim;
  const int qd = nh * hd, kd = nkv * hd, half = hd / 2;
  const int start = kv->len;
  const int empty = kv->len == 0;
  float *h = (float *)malloc((size_t)S * H * sizeof(float));
  float *q = (float *)malloc((size_t)S * qd * sizeof(float));
  float *k = (float *)malloc((size_t)S * kd * sizeof(float));
  float *v = (float *)malloc((size_t)S * kd * sizeof(float));
  for (int s = 0; s < S; s++) rmsnorm(x + (size_t)s * H, L->in_norm, H, c->eps, h + (size_t)s * H);
  linear_rows(L->wq, NULL, h, S, H, qd, q, 1);
  linear_rows(L->wk, NULL, h, S, H, kd, k, 1);
  linear_rows(L->wv, NULL, h, S, H, kd, v, 1);
  /* q_norm / k_norm over head_dim before RoPE (attention.rs:49-59) */
  float *tmp = (float *)malloc((size_t)hd * sizeof(float));
  for (int s = 0; s < S; s++) {
    for (int hh = 0; hh < nh; hh++) {
      float *p = q + (size_t)s * qd + hh * hd;
      rmsnorm(p, L->q_norm, hd, c->eps, tmp);
      memcpy(p, tmp, hd * sizeof(float));
    }
    for (int hh = 0; hh < nkv; hh++) {
      float *p = k + (size_t)s * kd + hh * hd;
      rmsnorm(p, L->k_norm, hd, c->eps, tmp);
      memcpy(p, tmp, hd * sizeof(float));
    }
  }
  free(tmp);
  /* rotate-half RoPE: x*cos + cat(-x2, x1)*sin (attention.rs:60-69,126-134);
   * inv_freq = 1/theta^(i/half) (rope.rs:21-24), position = cache.len + s */
  for (int s = 0; s < S; s++) {
    float pos = (float)(start + s);
    for (int i = 0; i < half; i++) {
      float inv = 1.0f / powf(c->theta, (float)i / (float)half);
      float f = pos * inv;
      float cs = cosf(f), sn = sinf(f);
      for (int hh = 0; hh < nh + nkv; hh++) {
        float *p = hh < nh ? q + (size_t)s * qd + hh * hd
                           : k + (size_t)s * kd + (hh - nh) * hd;
        float x1 = p[i], x2 = p[i + half];
        p[i] = x1 * cs - x2 * sn;
        p[i + half] = x2 * cs + x1 * sn;
      }
    }
  }
  /* runtime dtype bf16 for q, k, v (the cache holds bf16) */
  orc_bf16_round_array(q, (int64_t)S * qd);
  orc_bf16_round_array(k, (int64_t)S * kd);
  orc_bf16_round_array(v, (int64_t)S * kd);
  /* [S][nkv][hd] -> [nkv][S][hd] for the cache */
  float *kt = (float *)malloc((size_t)S * kd * sizeof(float));
  float *vt = (float *)malloc((size_t)S * kd * sizeof(float));
  for (int s = 0; s < S; s++)
    for (int hh = 0; hh < nkv; hh++) {
      memcpy(kt + ((size_t)hh * S + s) * hd, k + (size_t)s * kd + hh * hd, hd * sizeof(float));
      memcpy(vt + ((size_t)hh * S + s) * hd, v + (size_t)s * kd + hh * hd, hd * sizeof(float));
    }
  int cap_out = kv->len + S > kv->cap ? kv->cap : kv->len + S;
  if (S >= kv->cap) cap_out = kv->cap;
  float *kc = (float *)malloc((size_t)nkv * cap_out * hd * sizeof(float));
  float *vc = (float *)malloc((size_t)nkv * cap_out * hd * sizeof(float));
  int Lk = orc_kv_forward(kv, kt, vt, S, kc, vc);
  /* GQA: head hh reads kv head hh / n_rep (attention.rs:101-115) */
  int n_rep = nh / nkv;
  float *qh = (float *)malloc((size_t)nh * S * hd * sizeof(float));
  float *ke = (float *)malloc((size_t)nh * Lk * hd * sizeof(float));
  float *ve = (float *)malloc((size_t)nh * Lk * hd * sizeof(float));
  for (int hh = 0; hh < nh; hh++) {
    for (int s = 0; s < S; s++)
      memcpy(qh + ((size_t)hh * S + s) * hd, q + (size_t)s * qd + hh * hd, hd * sizeof(float));
    memcpy(ke + (size_t)hh * Lk * hd, kc + (size_t)(hh / n_rep) * Lk * hd, (size_t)Lk * hd * sizeof(float));
    memcpy(ve + (size_t)hh * Lk * hd, vc + (size_t)(hh / n_rep) * Lk * hd, (size_t)Lk * hd * sizeof(float));
  }
  uint8_t *mask = NULL;
  if (empty && S == Lk && S > 1) { /* model.rs:44-48: causal iff seq_len == key_len */
    mask = (uint8_t *)calloc((size_t)S * Lk, 1);
    for (int s = 0; s < S; s++)
      for (int j = s + 1; j < Lk; j++) mask[(size_t)s * Lk + j] = 1;
  }
  float *ao = (float *)malloc((size_t)nh * S * hd * sizeof(float));
  orc_sdpa(qh, ke, ve, mask, nh, S, Lk, hd, 1.0f / sqrtf((float)hd), ao);
  /* [nh][S][hd] -> [S][nh*hd] (attention.rs:119-121) */
  float *ar = (float *)malloc((size_t)S * qd * sizeof(float));
  for (int hh = 0; hh < nh; hh++)
    for (int s = 0; s < S; s++)
      memcpy(ar + (size_t)s * qd + hh * hd, ao + ((size_t)hh * S + s) * hd, hd * sizeof(float));
  float *o = (float *)malloc((size_t)S * H * sizeof(float));
  linear_rows(L->wo, NULL, ar, S, qd, H, o, 1);
  for (int64_t i = 0; i < (int64_t)S * H; i++) x[i] += o[i];
  /* MLP: down(silu(gate(x)) * up(x)) (mlp.rs:18-23) */
  for (int s = 0; s < S; s++) rmsnorm(x + (size_t)s * H, L->post_norm, H, c->eps, h + (size_t)s * H);
  float *g = (float *)malloc((size_t)S * c->inter * sizeof(float));
  float *u = (float *)malloc((size_t)S * c->inter * sizeof(float));
  linear_rows(L->w_gate, NULL, h, S, H, c->inter, g, 1);
  linear_rows(L->w_up, NULL, h, S, H, c->inter, u, 1);
  for (int64_t i = 0; i < (int64_t)S * c->inter; i++) g[i] = silu(g[i]) * u[i];
  linear_rows(L->w_down, NULL, g, S, c->inter, H, o, 1);
  for (int64_t i = 0; i < (int64_t)S * H; i++) x[i] += o[i];
  free(h); free(q); free(k); free(v); free(kt); free(vt); free(kc); free(vc);
  free(qh); free(ke); free(ve); free(mask); free(ao); free(ar); free(o); free(g);
  free(u);
}

/* model.rs:94-113 (talker decode) and predictor.rs:33-62 */
void orc_stack_forward(const orc_stack *st, orc_kv *caches, const float *x,
                       int S, float *out) {
  const int H = st->cfg.hidden;
  float *cur = (float *)malloc((size_t)S * H * sizeof(float));
  memcpy(cur, x, (size_t)S * H * sizeof(float));
  for (int l = 0; l < st->cfg.n_layers; l++)
    layer_forward(&st->cfg, &st->layers[l], &caches[l], cur, S);
  for (int s = 0; s < S; s++)
    rmsnorm(cur + (size_t)s * H, st->final_norm, H, st->cfg.eps, out + (size_t)s * H);
  free(cur);
}

/* ------------------------------------------------------------------------ */
/* Sampling: talker/infer/sampling.rs                                        */
/* ------------------------------------------------------------------------ */
int orc_repetition_penalty_enabled(float p) { /* sampling.rs:152-156 */
  return isfinite(p) && p > 0.f && fabsf(p - 1.f) > 1.1920929e-7f;
}

void orc_apply_repetition_penalty(float *logits, int V, const int64_t *hist,
                                  int n_hist, float penalty) {
  /* sampling.rs:128-150: gather original logits at the history ids, scale by
   * (1/p - 1) and scatter-ADD, so repeated ids accumulate and sign is ignored */
  if (!orc_repetition_penalty_enabled(penalty) || n_hist == 0) return;
  float scale = 1.0f / penalty - 1.0f;
  float *delta = (float *)malloc((size_t)n_hist * sizeof(float));
  for (int i = 0; i < n_hist; i++) delta[i] = logits[hist[i]] * scale;
  for (int i = 0; i < n_hist; i++) logits[hist[i]] += delta[i];
  free(delta);
  (void)V;
}

static int cmp_desc(const void *a, const void *b) {
  float x = *(const float *)a, y = *(const float *)b;
  return (x < y) - (x > y);
}

typedef struct { float v; int i; } vi_t;
static int cmp_vi_desc(const void *a, const void *b) {
  const vi_t *x = (const vi_t *)a, *y = (const vi_t *)b;
  if (x->v > y->v) return -1;
  if (x->v < y->v) return 1;
  return (x->i > y->i) - (x->i < y->i);
}

int64_t orc_sample_token(const float *logits_in, int V, const orc_sampling *s,
                         const int64_t *suppress, int n_suppress, float u) {
  float *lg = (float *)malloc((size_t)V * sizeof(float));
  memcpy(lg, logits_in, (size_t)V * sizeof(float));
  /* suppress mask (sampling.rs:101-126): ids >= vocab are dropped */
  for (int i = 0; i < n_suppress; i++)
    if (suppress[i] >= 0 && suppress[i] < V) lg[suppress[i]] = -INFINITY;
  int64_t tok = 0;
  if (!s->do_sample) { /* argmax, first index on ties (sampling.rs:60-62) */
    float best = lg[0];
    for (int i = 1; i < V; i++)
      if (lg[i] > best) { best = lg[i]; tok = i; }
    free(lg);
    return tok;
  }
  float t = s->temperature > 1e-5f ? s->temperature : 1e-5f;
  for (int i = 0; i < V; i++) lg[i] /= t;
  if (s->top_k > 0 && s->top_k < V) { /* threshold at the k-th value (:69-76) */
    float *srt = (float *)malloc((size_t)V * sizeof(float));
    memcpy(srt, lg, (size_t)V * sizeof(float));
    qsort(srt, V, sizeof(float), cmp_desc);
    float kth = srt[s->top_k - 1];
    for (int i = 0; i < V; i++)
      if (lg[i] < kth) lg[i] = -INFINITY;
    free(srt);
  }
  if (isfinite(s->top_p) && s->top_p > 0.f && s->top_p < 1.f) { /* :78-86 */
    vi_t *a = (vi_t *)malloc((size_t)V * sizeof(vi_t));
    for (int i = 0; i < V; i++) { a[i].v = lg[i]; a[i].i = i; }
    qsort(a, V, sizeof(vi_t), cmp_vi_desc);
    float mx = a[0].v, sum = 0.f;
    for (int i = 0; i < V; i++) sum += expf(a[i].v - mx);
    float cum = 0.f;
    for (int i = 0; i < V; i++) {
      float p = expf(a[i].v - mx) / sum;
      cum += p;
      if (!((cum - p) < s->top_p)) lg[a[i].i] = -INFINITY;
    }
    free(a);
  }
  /* softmax + categorical by inverse CDF over index order with draw u */
  float mx = -INFINITY;
  for (int i = 0; i < V; i++) mx = MAXF(mx, lg[i]);
  double sum = 0.0;
  for (int i = 0; i < V; i++) sum += expf(lg[i] - mx);
  double target = (double)u * sum, cum = 0.0;
  tok = V - 1;
  for (int i = 0; i < V; i++) {
    double p = expf(lg[i] - mx);
    if (p <= 0.0) continue;
    cum += p;
    if (cum > target) { tok = i; break; }
  }
  free(lg);
  return tok;
}

int orc_build_suppress_ids(int vocab, int64_t eos, int64_t *out) {
  int n = 0;
  for (int id = vocab > 1024 ? vocab - 1024 : 0; id < vocab; id++)
    if (id != eos) out[n++] = id;
  return n;
}

/* ------------------------------------------------------------------------ */
/* Talker generator: talker/infer/mod.rs                                     */
/* ------------------------------------------------------------------------ */
struct orc_gen {
  const orc_talker *m;
  orc_kv *kv, *pkv;
  float *kv_mem, *pkv_mem;
  float *hidden;
  int64_t selected;
  int eos_seen, finished, step_idx, max_new;
  int64_t eos;
  int64_t *hist;
  int hist_on;
  int64_t *codes; /* [max_new][n_groups] */
  const float *trailing;
  int trailing_len;
  const float *pad;
  orc_sampling ts, cs;
};

static orc_kv *alloc_caches(const orc_lm_cfg *c, int cap, float **mem) {
  orc_kv *kv = (orc_kv *)calloc(c->n_layers, sizeof(orc_kv));
  size_t per = (size_t)c->n_kv * cap * c->head_dim;
  *mem = (float *)calloc(per * 2 * c->n_layers, sizeof(float));
  for (int l = 0; l < c->n_layers; l++) {
    kv[l].k = *mem + per * 2 * l;
    kv[l].v = kv[l].k + per;
    kv[l].cap = cap;
    kv[l].len = 0;
    kv[l].n_kv = c->n_kv;
    kv[l].head_dim = c->head_dim;
  }
  return kv;
}

void orc_codec_group_embedding(const orc_talker *m, const int64_t *codes,
                               const float *extra, float *out) {
  /* infer/mod.rs:361-383 + add_trailing_text_embed :343-359 */
  const int H = m->talker.cfg.hidden;
  const float *e0 = m->talker_codec_emb + (size_t)codes[0] * H;
  for (int i = 0; i < H; i++) out[i] = e0[i];
  for (int g = 1; g < m->n_groups; g++) {
    const float *e = m->cp_codec_emb[g - 1] + (size_t)codes[g] * H;
    for (int i = 0; i < H; i++) out[i] += e[i];
  }
  if (extra)
    for (int i = 0; i < H; i++) out[i] += extra[i];
}

static void predict_frame_with(const orc_talker *m, orc_kv *pkv,
                               const float *hidden, int64_t code0,
                               const orc_sampling *s, const int64_t *forced,
                               const float *u, int64_t *codes, float *logits) {
  /* infer/mod.rs:434-535 */
  const orc_lm_cfg *pc = &m->predictor.cfg;
  const int H = m->talker.cfg.hidden, PH = pc->hidden, V = m->cp_vocab;
  const int G = m->n_groups;
  for (int l = 0; l < pc->n_layers; l++) orc_kv_reset_preserve(&pkv[l]);
  float *x2 = (float *)malloc((size_t)2 * H * sizeof(float));
  float *o2 = (float *)malloc((size_t)2 * PH * sizeof(float));
  float *lg = (float *)malloc((size_t)V * sizeof(float));
  int64_t *hist = (int64_t *)calloc(G, sizeof(int64_t));
  int hist_on = orc_repetition_penalty_enabled(s->repetition_penalty);
  memcpy(x2, hidden, H * sizeof(float));
  memcpy(x2 + H, m->talker_codec_emb + (size_t)code0 * H, H * sizeof(float));
  orc_stack_forward(&m->predictor, pkv, x2, 2, o2);
  orc_linear(m->lm_heads[0], NULL, o2 + PH, 1, PH, V, lg);
  if (logits) memcpy(logits, lg, V * sizeof(float));
  int64_t tok = orc_sample_token(lg, V, s, NULL, 0, u ? u[1] : 0.5f);
  if (forced) tok = forced[1];
  codes[0] = code0;
  codes[1] = tok;
  hist[0] = tok;
  for (int j = 1; j < G - 1; j++) {
    const float *e = m->cp_codec_emb[j - 1] + (size_t)codes[j] * H;
    orc_stack_forward(&m->predictor, pkv, e, 1, o2);
    orc_linear(m->lm_heads[j], NULL, o2, 1, PH, V, lg);
    if (hist_on) orc_apply_repetition_penalty(lg, V, hist, j, s->repetition_penalty);
    if (logits) memcpy(logits + (size_t)j * V, lg, V * sizeof(float));
    tok = orc_sample_token(lg, V, s, NULL, 0, u ? u[j + 1] : 0.5f);
    if (forced) tok = forced[j + 1];
    codes[j + 1] = tok;
    hist[j] = tok;
  }
  free(x2); free(o2); free(lg); free(hist);
}

void orc_predict_frame(const orc_talker *m, const float *hidden, int64_t code0,
                       const orc_sampling *s, const int64_t *forced,
                       const float *u, int64_t *codes, float *logits) {
  float *mem;
  orc_kv *pkv = alloc_caches(&m->predictor.cfg, m->n_groups + 1, &mem);
  predict_frame_with(m, pkv, hidden, code0, s, forced, u, codes, logits);
  free(pkv);
  free(mem);
}

orc_gen *orc_gen_start(const orc_talker *m, const float *inputs, int S,
                       const float *trailing, int trailing_len,
                       const float *pad, const orc_sampling *talker_s,
                       const orc_sampling *cp_s, int max_new_tokens,
                       int64_t eos, const int64_t *suppress, int n_suppress,
                       int64_t forced_first, float *first_logits, int *status) {
  /* infer/mod.rs:69-188 */
  if (max_new_tokens <= 0 || trailing_len <= 0 || S <= 0) {
    *status = -1;
    return NULL;
  }
  const int H = m->talker.cfg.hidden, V = m->vocab;
  orc_gen *g = (orc_gen *)calloc(1, sizeof(orc_gen));
  g->m = m;
  g->kv = alloc_caches(&m->talker.cfg, 4096, &g->kv_mem);
  g->pkv = alloc_caches(&m->predictor.cfg, m->n_groups + 1, &g->pkv_mem);
  g->hidden = (float *)malloc((size_t)H * sizeof(float));
  float *out = (float *)malloc((size_t)S * H * sizeof(float));
  orc_stack_forward(&m->talker, g->kv, inputs, S, out);
  memcpy(g->hidden, out + (size_t)(S - 1) * H, H * sizeof(float));
  free(out);
  float *lg = (float *)malloc((size_t)V * sizeof(float));
  orc_linear(m->codec_head, NULL, g->hidden, 1, H, V, lg);
  if (first_logits) memcpy(first_logits, lg, V * sizeof(float));
  int64_t tok = orc_sample_token(lg, V, talker_s, suppress, n_suppress, 0.5f);
  free(lg);
  if (forced_first >= 0) tok = forced_first;
  g->selected = tok;
  g->eos = eos;
  g->eos_seen = eos >= 0 && tok == eos;
  g->hist_on = orc_repetition_penalty_enabled(talker_s->repetition_penalty);
  g->hist = (int64_t *)calloc((size_t)max_new_tokens + 1, sizeof(int64_t));
  g->hist[0] = tok;
  g->codes = (int64_t *)calloc((size_t)max_new_tokens * m->n_groups, sizeof(int64_t));
  g->max_new = max_new_tokens;
  g->trailing = trailing;
  g->trailing_len = trailing_len;
  g->pad = pad;
  g->ts = *talker_s;
  g->cs = *cp_s;
  *status = 0;
  return g;
}

int orc_gen_step(orc_gen *g, const int64_t *forced, const float *u,
                 float *talker_logits, float *cp_logits, float *hidden_out) {
  /* infer/mod.rs:190-299 */
  const orc_talker *m = g->m;
  const int H = m->talker.cfg.hidden, V = m->vocab, G = m->n_groups;
  if (g->finished) return 0;
  if (g->eos_seen) {
    if (g->step_idx == 0) return -2; /* "EOS before any audio codec token" */
    g->finished = 1;
    return 0;
  }
  int64_t code0 = g->selected;
  if (forced) { /* teacher forcing replaces the token where it was sampled */
    code0 = forced[0];
    g->hist[g->step_idx] = code0;
  }
  int64_t *codes = g->codes + (size_t)g->step_idx * G;
  predict_frame_with(m, g->pkv, g->hidden, code0, &g->cs, forced, u, codes, cp_logits);
  float *emb = (float *)malloc((size_t)H * sizeof(float));
  const float *extra = g->step_idx < g->trailing_len
                           ? g->trailing + (size_t)g->step_idx * H
                           : g->pad;
  orc_codec_group_embedding(m, codes, extra, emb);
  g->step_idx++;
  if (g->step_idx >= g->max_new) {
    g->finished = 1;
    free(emb);
    return 2;
  }
  float *out = (float *)malloc((size_t)H * sizeof(float));
  orc_stack_forward(&m->talker, g->kv, emb, 1, out);
  float *lg = (float *)malloc((size_t)V * sizeof(float));
  orc_linear(m->codec_head, NULL, out, 1, H, V, lg);
  if (g->hist_on)
    orc_apply_repetition_penalty(lg, V, g->hist, g->step_idx, g->ts.repetition_penalty);
  if (talker_logits) memcpy(talker_logits, lg, V * sizeof(float));
  int64_t tok = orc_sample_token(lg, V, &g->ts, NULL, 0, u ? u[0] : 0.5f);
  g->selected = tok;
  if (g->eos >= 0 && tok == g->eos) g->eos_seen = 1;
  g->hist[g->step_idx] = tok;
  memcpy(g->hidden, out, H * sizeof(float));
  if (hidden_out) memcpy(hidden_out, out, H * sizeof(float));
  free(emb); free(out); free(lg);
  if (g->eos_seen) g->finished = 1;
  return g->finished ? 2 : 1;
}

int orc_gen_num_frames(const orc_gen *g) { return g->step_idx; }

void orc_gen_codes(const orc_gen *g, int64_t *out) {
  /* finalize: cat of [1,16,1] steps along time (infer/mod.rs:301-311) */
  const int G = g->m->n_groups, T = g->step_idx;
  for (int t = 0; t < T; t++)
    for (int q = 0; q < G; q++) out[(size_t)q * T + t] = g->codes[(size_t)t * G + q];
}

void orc_gen_free(orc_gen *g) {
  if (!g) return;
  free(g->kv); free(g->pkv); free(g->kv_mem); free(g->pkv_mem);
  free(g->hidden); free(g->hist); free(g->codes); free(g);
}

/* ------------------------------------------------------------------------ */
/* Codec decoder: codec/network/{decoder,wave,conv,activation,codebook}.rs  */
/* ------------------------------------------------------------------------ */
void orc_conv1d_padding(int L, int k, int dil, int stride, int *pad_total,
                        int *extra) {
  /* conv.rs:44-64 */
  int eff = (k - 1) * dil + 1;
  int pt = eff > stride ? eff - stride : 0;
  int padded = L + pt;
  int missing = eff > padded ? eff - padded : 0;
  *pad_total = pt;
  *extra = missing > 0 ? missing : (stride - (padded - eff) % stride) % stride;
}

void orc_pad_1d(const float *x, int C, int L, int left, int right, int mode,
                float *out) {
  /* conv.rs:71-83 (Burn pad: constant or edge replicate) */
  int Lo = L + left + right;
  for (int c = 0; c < C; c++) {
    const float *xi = x + (size_t)c * L;
    float *o = out + (size_t)c * Lo;
    for (int t = 0; t < Lo; t++) {
      int s = t - left;
      if (s >= 0 && s < L) o[t] = xi[s];
      else if (mode == 1) o[t] = xi[s < 0 ? 0 : L - 1];
      else o[t] = 0.f;
    }
  }
}

/* causal Conv1d with constant-0 left pad (conv.rs:33-42): x [Ci][L] ->
 * y [Co][L]; groups = 1 or Ci (depthwise) */
static void conv1d_causal(const float *x, int Ci, int L, const float *w,
                          const float *b, int Co, int k, int dil, int groups,
                          float *y) {
  int pt, ex;
  orc_conv1d_padding(L, k, dil, 1, &pt, &ex);
  int Lp = L + pt + ex;
  float *xp = (float *)malloc((size_t)Ci * Lp * sizeof(float));
  orc_pad_1d(x, Ci, L, pt, ex, 0, xp);
  int Lo = Lp - ((k - 1) * dil + 1) + 1;
  int cig = Ci / groups, cog = Co / groups;
#pragma omp parallel for schedule(static)
  for (int o = 0; o < Co; o++) {
    float *yo = y + (size_t)o * Lo;
    for (int t = 0; t < Lo; t++) yo[t] = b ? b[o] : 0.f;
    int gi = o / cog;
    for (int ii = 0; ii < cig; ii++) {
      int i = gi * cig + ii;
      const float *xi = xp + (size_t)i * Lp;
      for (int j = 0; j < k; j++) {
        float wv = w[((size_t)o * cig + ii) * k + j];
        const float *xs = xi + j * dil;
        for (int t = 0; t < Lo; t++) yo[t] += wv * xs[t];
      }
    }
  }
  free(xp);
}

/* ConvTranspose1d (burn, weight [Ci][Co][k], no padding) followed by the
 * causal trim of k - stride from both ends (conv.rs:19-31): returns Lo */
static int convtr1d_trim(const float *x, int Ci, int L, const float *w,
                         const float *b, int Co, int k, int stride, float *y) {
  int Lfull = (L - 1) * stride + k;
  int trim = k > stride ? k - stride : 0;
  int Lo = Lfull - 2 * trim;
  if (Lo < 0) Lo = 0;
#pragma omp parallel for schedule(static)
  for (int o = 0; o < Co; o++) {
    float *full = (float *)malloc((size_t)Lfull * sizeof(float));
    for (int t = 0; t < Lfull; t++) full[t] = b ? b[o] : 0.f;
    for (int i = 0; i < Ci; i++) {
      const float *xi = x + (size_t)i * L;
      for (int j = 0; j < k; j++) {
        float wv = w[((size_t)i * Co + o) * k + j];
        for (int s = 0; s < L; s++) full[s * stride + j] += wv * xi[s];
      }
    }
    memcpy(y + (size_t)o * Lo, full + trim, (size_t)Lo * sizeof(float));
    free(full);
  }
  return Lo;
}

/* SnakeBeta: x + sin^2(e^alpha x) / (e^beta + 1e-9) (activation.rs:16-37) */
static void snake(float *x, int C, int L, const float *alpha,
                  const float *beta, float *out) {
#pragma omp parallel for schedule(static)
  for (int c = 0; c < C; c++) {
    float a = expf(alpha[c]), bb = expf(beta[c]) + 1e-9f;
    for (int t = 0; t < L; t++) {
      float v = x[(size_t)c * L + t];
      float s = sinf(v * a);
      out[(size_t)c * L + t] = v + (s * s) / bb;
    }
  }
}

static void transpose(const float *x, int R, int C, float *y) {
  for (int r = 0; r < R; r++)
    for (int c = 0; c < C; c++) y[(size_t)c * R + r] = x[(size_t)r * C + c];
}

/* burn::nn::RotaryEncoding (adjacent pairs, theta_i = theta^(-2i/d)) used
 * by the codec pre-transformer with offset 0 (decoder.rs:126-128) */
static void rope_pairs(float *x, int T, int nh, int hd, float theta) {
  for (int t = 0; t < T; t++)
    for (int i = 0; i < hd / 2; i++) {
      float th = expf((float)(2 * i) / (float)hd * logf(theta));
      th = 1.0f / th;
      float f = (float)t * th;
      float cs = cosf(f), sn = sinf(f);
      for (int h = 0; h < nh; h++) {
        float *p = x + ((size_t)t * nh + h) * hd + 2 * i;
        float x0 = p[0], x1 = p[1];
        p[0] = x0 * cs - x1 * sn;
        p[1] = x1 * cs + x0 * sn;
      }
    }
}

/* one pre-transformer layer on h [T][H] (decoder.rs:98-173) */
static void codec_layer(const orc_codec *c, const orc_codec_layer *L, float *h,
                        int T) {
  const int H = c->hidden, nh = c->n_heads, nkv = c->n_kv, hd = c->head_dim;
  const int qd = nh * hd, kd = nkv * hd;
  float *n = (float *)malloc((size_t)T * H * sizeof(float));
  float *q = (float *)malloc((size_t)T * qd * sizeof(float));
  float *k = (float *)malloc((size_t)T * kd * sizeof(float));
  float *v = (float *)malloc((size_t)T * kd * sizeof(float));
  for (int t = 0; t < T; t++) rmsnorm(h + (size_t)t * H, L->in_norm, H, c->eps, n + (size_t)t * H);
  linear_rows(L->wq, NULL, n, T, H, qd, q, 0);
  linear_rows(L->wk, NULL, n, T, H, kd, k, 0);
  linear_rows(L->wv, NULL, n, T, H, kd, v, 0);
  rope_pairs(q, T, nh, hd, c->theta);
  rope_pairs(k, T, nkv, hd, c->theta);
  int n_rep = nh / nkv;
  float *qh = (float *)malloc((size_t)nh * T * hd * sizeof(float));
  float *ke = (float *)malloc((size_t)nh * T * hd * sizeof(float));
  float *ve = (float *)malloc((size_t)nh * T * hd * sizeof(float));
  for (int hh = 0; hh < nh; hh++)
    for (int t = 0; t < T; t++) {
      memcpy(qh + ((size_t)hh * T + t) * hd, q + (size_t)t * qd + hh * hd, hd * sizeof(float));
      memcpy(ke + ((size_t)hh * T + t) * hd, k + (size_t)t * kd + (hh / n_rep) * hd, hd * sizeof(float));
      memcpy(ve + ((size_t)hh * T + t) * hd, v + (size_t)t * kd + (hh / n_rep) * hd, hd * sizeof(float));
    }
  float *ao = (float *)malloc((size_t)nh * T * hd * sizeof(float));
  orc_sdpa(qh, ke, ve, NULL, nh, T, T, hd, 1.0f / sqrtf((float)hd), ao);
  float *ar = (float *)malloc((size_t)T * qd * sizeof(float));
  for (int hh = 0; hh < nh; hh++)
    for (int t = 0; t < T; t++)
      memcpy(ar + (size_t)t * qd + hh * hd, ao + ((size_t)hh * T + t) * hd, hd * sizeof(float));
  float *o = (float *)malloc((size_t)T * H * sizeof(float));
  linear_rows(L->wo, NULL, ar, T, qd, H, o, 0);
  for (int t = 0; t < T; t++)
    for (int i = 0; i < H; i++) h[(size_t)t * H + i] += o[(size_t)t * H + i] * L->attn_scale[i];
  for (int t = 0; t < T; t++) rmsnorm(h + (size_t)t * H, L->post_norm, H, c->eps, n + (size_t)t * H);
  float *g = (float *)malloc((size_t)T * c->inter * sizeof(float));
  float *u = (float *)malloc((size_t)T * c->inter * sizeof(float));
  linear_rows(L->w_gate, NULL, n, T, H, c->inter, g, 0);
  linear_rows(L->w_up, NULL, n, T, H, c->inter, u, 0);
  for (int64_t i = 0; i < (int64_t)T * c->inter; i++) g[i] = silu(g[i]) * u[i];
  linear_rows(L->w_down, NULL, g, T, c->inter, H, o, 0);
  for (int t = 0; t < T; t++)
    for (int i = 0; i < H; i++) h[(size_t)t * H + i] += o[(size_t)t * H + i] * L->mlp_scale[i];
  free(n); free(q); free(k); free(v); free(qh); free(ke); free(ve); free(ao);
  free(ar); free(o); free(g); free(u);
}

static float gelu_erf(float x) { return 0.5f * x * (1.f + erff(x * 0.70710678118654752f)); }

/* ConvNeXt block (wave.rs:96-108) on x [C][L] in place */
static void convnext(const orc_convnext *b, float *x, int C, int L) {
  float *d = (float *)malloc((size_t)C * L * sizeof(float));
  conv1d_causal(x, C, L, b->dw_w, b->dw_b, C, 7, 1, C, d);
  float *t = (float *)malloc((size_t)L * C * sizeof(float));
  transpose(d, C, L, t); /* [L][C] */
  for (int s = 0; s < L; s++) { /* LayerNorm eps 1e-6, biased variance */
    float *r = t + (size_t)s * C;
    float mean = 0.f;
    for (int i = 0; i < C; i++) mean += r[i];
    mean /= (float)C;
    float var = 0.f;
    for (int i = 0; i < C; i++) var += (r[i] - mean) * (r[i] - mean);
    var /= (float)C;
    float den = sqrtf(var + 1e-6f);
    for (int i = 0; i < C; i++) r[i] = (r[i] - mean) / den * b->ln_w[i] + b->ln_b[i];
  }
  float *p1 = (float *)malloc((size_t)L * 4 * C * sizeof(float));
  linear_rows(b->pw1_w, b->pw1_b, t, L, C, 4 * C, p1, 0);
  for (int64_t i = 0; i < (int64_t)L * 4 * C; i++) p1[i] = gelu_erf(p1[i]);
  linear_rows(b->pw2_w, b->pw2_b, p1, L, 4 * C, C, t, 0);
  for (int c = 0; c < C; c++)
    for (int s = 0; s < L; s++) x[(size_t)c * L + s] += t[(size_t)s * C + c] * b->gamma[c];
  free(d); free(t); free(p1);
}

int64_t orc_codec_out_len(const orc_codec *c, int T) {
  int64_t L = T;
  for (int i = 0; i < c->n_up; i++) L *= c->up_ratio[i];
  for (int i = 0; i < c->n_stage; i++) L = L > 0 ? (L - 1) * c->rates[i] : 0;
  return L;
}

static int64_t codec_one(const orc_codec *c, const int64_t *codes, int T,
                         int tap, float *out) {
  const int half = c->codebook_dim / 2, D = c->codebook_dim;
  for (int q = 0; q < c->n_q; q++)
    for (int t = 0; t < T; t++)
      if (codes[(size_t)q * T + t] < 0 || codes[(size_t)q * T + t] >= c->codebook_size) return -1;
  /* quantizer (decoder.rs:196-247, codebook.rs:4-41) */
  float *sem = (float *)calloc((size_t)half * T, sizeof(float));
  float *aco = (float *)calloc((size_t)half * T, sizeof(float));
  for (int q = 0; q < c->n_q; q++) {
    float *acc = q < c->n_semantic ? sem : aco;
    for (int t = 0; t < T; t++) {
      int64_t id = codes[(size_t)q * T + t];
      float us = c->usage[q][id];
      us = us < 1e-6f ? 1e-6f : us;
      const float *e = c->emb_sum[q] + (size_t)id * half;
      for (int i = 0; i < half; i++) acc[(size_t)i * T + t] += e[i] / us;
    }
  }
  float *qo = (float *)malloc((size_t)D * T * sizeof(float));
  float *tmp = (float *)malloc((size_t)D * T * sizeof(float));
  conv1d_causal(sem, half, T, c->first_out_proj, NULL, D, 1, 1, 1, qo);
  if (c->n_q > c->n_semantic) {
    conv1d_causal(aco, half, T, c->rest_out_proj, NULL, D, 1, 1, 1, tmp);
    for (int64_t i = 0; i < (int64_t)D * T; i++) qo[i] += tmp[i];
  }
  free(sem); free(aco); free(tmp);
  if (tap == 0) { if (out) memcpy(out, qo, (size_t)D * T * sizeof(float)); free(qo); return (int64_t)D * T; }
  /* pre_conv k3 (decoder.rs:261) */
  const int LAT = c->latent, H = c->hidden;
  float *x = (float *)malloc((size_t)LAT * T * sizeof(float));
  conv1d_causal(qo, D, T, c->pre_conv_w, c->pre_conv_b, LAT, 3, 1, 1, x);
  free(qo);
  if (tap == 1) { if (out) memcpy(out, x, (size_t)LAT * T * sizeof(float)); free(x); return (int64_t)LAT * T; }
  /* pre_transformer (decoder.rs:175-194, 262-266) */
  float *xt = (float *)malloc((size_t)T * LAT * sizeof(float));
  transpose(x, LAT, T, xt);
  float *h = (float *)malloc((size_t)T * H * sizeof(float));
  linear_rows(c->in_proj_w, c->in_proj_b, xt, T, LAT, H, h, 0);
  for (int l = 0; l < c->n_layers; l++) codec_layer(c, &c->layers[l], h, T);
  float *hn = (float *)malloc((size_t)T * H * sizeof(float));
  for (int t = 0; t < T; t++) rmsnorm(h + (size_t)t * H, c->final_norm, H, c->eps, hn + (size_t)t * H);
  linear_rows(c->out_proj_w, c->out_proj_b, hn, T, H, LAT, xt, 0);
  transpose(xt, T, LAT, x);
  free(xt); free(h); free(hn);
  if (tap == 2) { if (out) memcpy(out, x, (size_t)LAT * T * sizeof(float)); free(x); return (int64_t)LAT * T; }
  /* upsample: ConvT(k=r, s=r) + ConvNeXt (decoder.rs:268-271) */
  int L = T;
  for (int u = 0; u < c->n_up; u++) {
    int r = c->up_ratio[u];
    float *y = (float *)malloc((size_t)LAT * L * r * sizeof(float));
    L = convtr1d_trim(x, LAT, L, c->up[u].wt, c->up[u].bt, LAT, r, r, y);
    free(x);
    x = y;
    convnext(&c->up[u], x, LAT, L);
  }
  if (tap == 3) { if (out) memcpy(out, x, (size_t)LAT * L * sizeof(float)); free(x); return (int64_t)LAT * L; }
  /* wave decoder (wave.rs:12-94, decoder.rs:273-276) */
  int C = c->decoder_dim;
  float *w = (float *)malloc((size_t)C * L * sizeof(float));
  conv1d_causal(x, LAT, L, c->in_conv_w, c->in_conv_b, C, 7, 1, 1, w);
  free(x);
  if (tap == 4) { if (out) memcpy(out, w, (size_t)C * L * sizeof(float)); free(w); return (int64_t)C * L; }
  for (int s = 0; s < c->n_stage; s++) {
    const orc_wave_stage *st = &c->stages[s];
    int r = c->rates[s], Co = C / 2;
    float *a = (float *)malloc((size_t)C * L * sizeof(float));
    snake(w, C, L, st->snake_alpha, st->snake_beta, a);
    int Lo = (L - 1) * r;
    float *y = (float *)malloc((size_t)Co * (Lo > 0 ? Lo : 1) * sizeof(float));
    Lo = convtr1d_trim(a, C, L, st->wt, st->bt, Co, 2 * r, r, y);
    free(a);
    free(w);
    w = y;
    C = Co;
    L = Lo;
    float *t1 = (float *)malloc((size_t)C * L * sizeof(float));
    float *t2 = (float *)malloc((size_t)C * L * sizeof(float));
    static const int dil[3] = {1, 3, 9};
    for (int ru = 0; ru < 3; ru++) { /* residual unit (wave.rs:57-66) */
      const orc_resunit *R = &st->ru[ru];
      snake(w, C, L, R->a1_alpha, R->a1_beta, t1);
      conv1d_causal(t1, C, L, R->w1, R->b1, C, 7, dil[ru], 1, t2);
      snake(t2, C, L, R->a2_alpha, R->a2_beta, t1);
      conv1d_causal(t1, C, L, R->w2, R->b2, C, 1, 1, 1, t2);
      for (int64_t i = 0; i < (int64_t)C * L; i++) w[i] += t2[i];
    }
    free(t1); free(t2);
    if (tap == 5 + s) { if (out) memcpy(out, w, (size_t)C * L * sizeof(float)); free(w); return (int64_t)C * L; }
  }
  float *a = (float *)malloc((size_t)C * L * sizeof(float));
  snake(w, C, L, c->out_alpha, c->out_beta, a);
  float *y = (float *)malloc((size_t)L * sizeof(float));
  conv1d_causal(a, C, L, c->out_conv_w, c->out_conv_b, 1, 7, 1, 1, y);
  for (int t = 0; t < L; t++) y[t] = y[t] < -1.f ? -1.f : (y[t] > 1.f ? 1.f : y[t]);
  if (out) memcpy(out, y, (size_t)L * sizeof(float));
  free(a); free(w); free(y);
  return L;
}

int64_t orc_codec_decode_tap(const orc_codec *c, const int64_t *codes, int T,
                             int tap, float *out) {
  return codec_one(c, codes, T, tap, out);
}

int orc_codec_decode(const orc_codec *c, const int64_t *codes, int B, int T,
                     float *wave) {
  int64_t n = orc_codec_out_len(c, T);
  for (int b = 0; b < B; b++) {
    int64_t r = codec_one(c, codes + (size_t)b * c->n_q * T, T, 99, wave + (size_t)b * n);
    if (r < 0) return -1;
  }
  return 0;
}

void orc_to_pcm(const float *x, int64_t n, int16_t *out) {
  /* codec/infer/mod.rs:80-90 */
  for (int64_t i = 0; i < n; i++) {
    float s = x[i] < -1.f ? -1.f : (x[i] > 1.f ? 1.f : x[i]);
    int v = (int)roundf(s * 32768.0f);
    v = v < -32768 ? -32768 : (v > 32767 ? 32767 : v);
    out[i] = (int16_t)v;
  }
}

/* ------------------------------------------------------------------------ */
/* Codec encoder: codec/network/encoder.rs, init in codec/config.rs:136-346  */
/* ------------------------------------------------------------------------ */
/* Conv1d behind conv1d_padding + pad_1d (encoder.rs:155-161, conv.rs:33-83):
 * left pad = effective kernel - stride, right pad = the extra that completes
 * the last stride window; mode 0 = constant 0, 1 = edge.  x [ci][L] ->
 * y [co][Lo]; returns Lo. */
static int enc_conv(const orc_conv *c, const float *x, int L, int mode, float *y) {
  int pt, ex;
  orc_conv1d_padding(L, c->k, 1, c->stride, &pt, &ex);
  const int Lp = L + pt + ex;
  float *xp = (float *)malloc((size_t)c->ci * Lp * sizeof(float));
  orc_pad_1d(x, c->ci, L, pt, ex, mode, xp);
  const int Lo = (Lp - c->k) / c->stride + 1;
#pragma omp parallel for schedule(static)
  for (int o = 0; o < c->co; o++) {
    float *yo = y + (size_t)o * Lo;
    for (int t = 0; t < Lo; t++) yo[t] = c->b ? c->b[o] : 0.f;
    for (int i = 0; i < c->ci; i++) {
      const float *xi = xp + (size_t)i * Lp;
      for (int j = 0; j < c->k; j++) {
        const float wv = c->w[((size_t)o * c->ci + i) * c->k + j];
        for (int t = 0; t < Lo; t++) yo[t] += wv * xi[t * c->stride + j];
      }
    }
  }
  free(xp);
  return Lo;
}

/* output length of enc_conv for input length L */
static int enc_conv_len(const orc_conv *c, int L) {
  int pt, ex;
  orc_conv1d_padding(L, c->k, 1, c->stride, &pt, &ex);
  return (L + pt + ex - c->k) / c->stride + 1;
}

static void elu_inplace(float *x, int64_t n) { /* burn elu, alpha 1 (encoder.rs:163-167) */
  for (int64_t i = 0; i < n; i++) x[i] = x[i] > 0.f ? x[i] : expf(x[i]) - 1.f;
}

/* burn LayerNorm with bias, biased variance */
static void layer_norm(const float *x, const float *w, const float *b, int n, float eps, float *y) {
  float mean = 0.f, var = 0.f;
  for (int i = 0; i < n; i++) mean += x[i];
  mean /= (float)n;
  for (int i = 0; i < n; i++) var += (x[i] - mean) * (x[i] - mean);
  var /= (float)n;
  const float inv = 1.f / sqrtf(var + eps);
  for (int i = 0; i < n; i++) y[i] = (x[i] - mean) * inv * w[i] + b[i];
}

/* one encoder transformer layer on h [T][H] (encoder.rs:202-288): causal
 * (autoregressive mask) GQA attention with burn RotaryEncoding at offset 0,
 * GELU MLP, LayerScale on both branches */
static void enc_layer(const orc_codec_encoder *e, const orc_enc_layer *L, float *h, int T) {
  const int H = e->hidden, nh = e->n_heads, nkv = e->n_kv, hd = e->head_dim;
  const int qd = nh * hd, kd = nkv * hd, I = e->inter;
  float *n = (float *)malloc((size_t)T * H * sizeof(float));
  float *q = (float *)malloc((size_t)T * qd * sizeof(float));
  float *k = (float *)malloc((size_t)T * kd * sizeof(float));
  float *v = (float *)malloc((size_t)T * kd * sizeof(float));
  for (int t = 0; t < T; t++) layer_norm(h + (size_t)t * H, L->ln1_w, L->ln1_b, H, e->norm_eps, n + (size_t)t * H);
  linear_rows(L->wq, L->bq, n, T, H, qd, q, 0);
  linear_rows(L->wk, L->bk, n, T, H, kd, k, 0);
  linear_rows(L->wv, L->bv, n, T, H, kd, v, 0);
  rope_pairs(q, T, nh, hd, e->theta);
  rope_pairs(k, T, nkv, hd, e->theta);
  const int rep = nh / nkv;
  float *qh = (float *)malloc((size_t)nh * T * hd * sizeof(float));
  float *ke = (float *)malloc((size_t)nh * T * hd * sizeof(float));
  float *ve = (float *)malloc((size_t)nh * T * hd * sizeof(float));
  for (int hh = 0; hh < nh; hh++)
    for (int t = 0; t < T; t++) {
      memcpy(qh + ((size_t)hh * T + t) * hd, q + (size_t)t * qd + hh * hd, hd * sizeof(float));
      memcpy(ke + ((size_t)hh * T + t) * hd, k + (size_t)t * kd + (hh / rep) * hd, hd * sizeof(float));
      memcpy(ve + ((size_t)hh * T + t) * hd, v + (size_t)t * kd + (hh / rep) * hd, hd * sizeof(float));
    }
  uint8_t *mask = (uint8_t *)malloc((size_t)T * T);
  for (int s = 0; s < T; s++)
    for (int j = 0; j < T; j++) mask[(size_t)s * T + j] = j > s; /* generate_autoregressive_mask */
  float *ao = (float *)malloc((size_t)nh * T * hd * sizeof(float));
  orc_sdpa(qh, ke, ve, mask, nh, T, T, hd, 1.0f / sqrtf((float)hd), ao);
  float *ar = (float *)malloc((size_t)T * qd * sizeof(float));
  for (int hh = 0; hh < nh; hh++)
    for (int t = 0; t < T; t++)
      memcpy(ar + (size_t)t * qd + hh * hd, ao + ((size_t)hh * T + t) * hd, hd * sizeof(float));
  float *o = (float *)malloc((size_t)T * H * sizeof(float));
  linear_rows(L->wo, L->bo, ar, T, qd, H, o, 0);
  for (int64_t i = 0; i < (int64_t)T * H; i++) h[i] += o[i] * L->attn_scale[i % H];
  for (int t = 0; t < T; t++) layer_norm(h + (size_t)t * H, L->ln2_w, L->ln2_b, H, e->norm_eps, n + (size_t)t * H);
  float *f = (float *)malloc((size_t)T * I * sizeof(float));
  linear_rows(L->fc1, NULL, n, T, H, I, f, 0);
  for (int64_t i = 0; i < (int64_t)T * I; i++) f[i] = gelu_erf(f[i]);
  linear_rows(L->fc2, NULL, f, T, I, H, o, 0);
  for (int64_t i = 0; i < (int64_t)T * H; i++) h[i] += o[i] * L->mlp_scale[i % H];
  free(n); free(q); free(k); free(v); free(qh); free(ke); free(ve); free(mask); free(ao); free(ar); free(o); free(f);
}

void orc_rvq_encode(const float *const *embed_sum, const float *const *usage, int n_layers, int codebook_size,
                    int vq, float *x, int T, int64_t *codes) {
  /* encoder.rs:319-368, codebook.rs:4-41: centroids = embed_sum /
   * clamp_min(usage, 1e-6); id = argmin_j sum_d (x_d - c_jd)^2 (first index
   * on ties); the residual loses the chosen centroid */
  float *cent = (float *)malloc((size_t)codebook_size * vq * sizeof(float));
  for (int l = 0; l < n_layers; l++) {
    for (int j = 0; j < codebook_size; j++) {
      const float u = usage[l][j] < 1e-6f ? 1e-6f : usage[l][j];
      for (int d = 0; d < vq; d++) cent[(size_t)j * vq + d] = embed_sum[l][(size_t)j * vq + d] / u;
    }
#pragma omp parallel for schedule(static)
    for (int t = 0; t < T; t++) {
      int best = 0;
      float bd = INFINITY;
      for (int j = 0; j < codebook_size; j++) {
        float s = 0.f;
        for (int d = 0; d < vq; d++) {
          const float df = x[(size_t)d * T + t] - cent[(size_t)j * vq + d];
          s += df * df;
        }
        if (s < bd) {
          bd = s;
          best = j;
        }
      }
      codes[(size_t)l * T + t] = best;
      for (int d = 0; d < vq; d++) x[(size_t)d * T + t] -= cent[(size_t)best * vq + d];
    }
  }
  free(cent);
}

/* encoder.rs:128-130: backbone, transformer and downsample; returns the
 * hidden [H][T] (malloc'd, caller frees) and T, or NULL */
static float *encoder_hidden(const orc_codec_encoder *e, const float *wave, int n, int *T_out) {
  /* backbone (encoder.rs:138-175; layers as config.rs:174-236 builds them) */
  int L = n, C = 1;
  float *x = (float *)malloc((size_t)n * sizeof(float));
  memcpy(x, wave, (size_t)n * sizeof(float));
  {
    const int Lo = enc_conv_len(&e->in_conv, L);
    float *y = (float *)malloc((size_t)e->in_conv.co * Lo * sizeof(float));
    enc_conv(&e->in_conv, x, L, 0, y);
    free(x); x = y; L = Lo; C = e->in_conv.co;
  }
  for (int s = 0; s < e->n_stages; s++) {
    /* resnet: x + conv_out(elu(conv_in(elu(x)))) */
    float *h = (float *)malloc((size_t)C * L * sizeof(float));
    memcpy(h, x, (size_t)C * L * sizeof(float));
    elu_inplace(h, (int64_t)C * L);
    float *m = (float *)malloc((size_t)e->res_in[s].co * L * sizeof(float));
    enc_conv(&e->res_in[s], h, L, 0, m);
    elu_inplace(m, (int64_t)e->res_in[s].co * L);
    enc_conv(&e->res_out[s], m, L, 0, h);
    for (int64_t i = 0; i < (int64_t)C * L; i++) x[i] += h[i];
    free(m); free(h);
    elu_inplace(x, (int64_t)C * L);
    const int Lo = enc_conv_len(&e->down[s], L);
    float *y = (float *)malloc((size_t)e->down[s].co * Lo * sizeof(float));
    enc_conv(&e->down[s], x, L, 0, y);
    free(x); x = y; L = Lo; C = e->down[s].co;
  }
  elu_inplace(x, (int64_t)C * L);
  {
    const int Lo = enc_conv_len(&e->out_conv, L);
    float *y = (float *)malloc((size_t)e->out_conv.co * Lo * sizeof(float));
    enc_conv(&e->out_conv, x, L, 0, y);
    free(x); x = y; L = Lo; C = e->out_conv.co;
  }
  /* transformer on [T][H] (encoder.rs:179-200) */
  const int H = e->hidden;
  if (C != H) { free(x); return NULL; }
  float *h = (float *)malloc((size_t)L * H * sizeof(float));
  transpose(x, H, L, h);
  for (int l = 0; l < e->n_layers; l++) enc_layer(e, &e->layers[l], h, L);
  transpose(h, L, H, x);
  free(h);
  /* downsample: stride 2, edge padding (config.rs:155-166) */
  const int T = enc_conv_len(&e->downsample, L);
  float *z = (float *)malloc((size_t)H * T * sizeof(float));
  enc_conv(&e->downsample, x, L, 1, z);
  free(x);
  *T_out = T;
  return z;
}

int orc_codec_encoder_hidden(const orc_codec_encoder *e, const float *wave, int n, float *out, int max_frames) {
  if (!e || !wave || n <= 0) return -1;
  int T = 0;
  float *z = encoder_hidden(e, wave, n, &T);
  if (!z) return -1;
  if (T > max_frames) { free(z); return -1; }
  memcpy(out, z, (size_t)e->hidden * T * sizeof(float));
  free(z);
  return T;
}

int orc_codec_encode(const orc_codec_encoder *e, const float *wave, int n, int n_valid, int64_t *codes,
                     int max_frames) {
  if (!e || !wave || n <= 0 || e->semantic.n_layers <= 0 || n_valid < e->semantic.n_layers) return -1;
  int T = 0;
  float *z = encoder_hidden(e, wave, n, &T);
  if (!z) return -1;
  const int H = e->hidden;
  if (T > max_frames || T <= 0) { free(z); return -1; }
  /* quantizers on the same hidden (encoder.rs:290-317) */
  const int vq = e->vq_dim;
  const orc_enc_rvq *q[2] = {&e->semantic, &e->acoustic};
  int want[2] = {e->semantic.n_layers, n_valid - e->semantic.n_layers};
  if (want[1] > e->acoustic.n_layers) want[1] = e->acoustic.n_layers;
  int row = 0;
  for (int g = 0; g < 2; g++) {
    if (want[g] <= 0) continue;
    float *r = (float *)malloc((size_t)vq * T * sizeof(float)); /* input_proj, Conv1d k1 without bias */
#pragma omp parallel for schedule(static)
    for (int d = 0; d < vq; d++)
      for (int t = 0; t < T; t++) {
        float s = 0.f;
        for (int c = 0; c < H; c++) s += q[g]->in_proj[(size_t)d * H + c] * z[(size_t)c * T + t];
        r[(size_t)d * T + t] = s;
      }
    orc_rvq_encode(q[g]->embed_sum, q[g]->usage, want[g], e->codebook_size, vq, r, T, codes + (size_t)row * T);
    row += want[g];
    free(r);
  }
  free(z);
  return T;
}

/* ------------------------------------------------------------------------ */
/* Speaker encoder: model/speaker/infer/feature.rs, model/speaker/network    */
/* ------------------------------------------------------------------------ */
/* in-place iterative radix-2 DFT (the transform rustfft computes; forward,
 * unnormalised), n a power of two */
static void fft_pow2(double *re, double *im, int n) {
  for (int i = 1, j = 0; i < n; i++) {
    int bit = n >> 1;
    for (; j & bit; bit >>= 1) j ^= bit;
    j ^= bit;
    if (i < j) {
      double t = re[i]; re[i] = re[j]; re[j] = t;
      t = im[i]; im[i] = im[j]; im[j] = t;
    }
  }
  for (int len = 2; len <= n; len <<= 1) {
    const double ang = -2.0 * M_PI / len;
    for (int i = 0; i < n; i += len)
      for (int k = 0; k < len / 2; k++) {
        const double wr = cos(ang * k), wi = sin(ang * k);
        const double ur = re[i + k], ui = im[i + k];
        const double vr = re[i + k + len / 2] * wr - im[i + k + len / 2] * wi;
        const double vi = re[i + k + len / 2] * wi + im[i + k + len / 2] * wr;
        re[i + k] = ur + vr; im[i + k] = ui + vi;
        re[i + k + len / 2] = ur - vr; im[i + k + len / 2] = ui - vi;
      }
  }
}

static float hz_to_mel(float hz) { return 2595.0f * log10f(1.0f + hz / 700.0f); }
static float mel_to_hz(float m) { return 700.0f * (powf(10.0f, m / 2595.0f) - 1.0f); }

int orc_speaker_mel(const float *x, int n, int sr, int n_mels, float *out, int max_frames) {
  /* feature.rs:32-150 (n_fft 1024, hop 256, win 1024, fmin 0, fmax sr / 2) */
  const int n_fft = 1024, hop = 256, pad = (n_fft - hop) / 2, nf = n_fft / 2 + 1;
  if (!x || n < n_fft - 2 * pad || n_mels <= 0) return -1;
  const int plen = n + 2 * pad, frames = (plen - n_fft) / hop + 1;
  if (frames > max_frames) return -1;
  float *p = (float *)malloc((size_t)plen * sizeof(float));
  for (int i = 0; i < pad; i++) { /* left: samples[pad], ..., samples[1] (feature.rs:100-102) */
    int idx = pad - i;
    p[i] = x[idx < n - 1 ? idx : n - 1];
  }
  memcpy(p + pad, x, (size_t)n * sizeof(float));
  for (int i = 0; i < pad; i++) { /* right: samples[n - 2 - i], saturating (feature.rs:104-109) */
    int idx = n - 2 - i;
    if (idx < 0) idx = 0;
    if (idx > n - 1) idx = n - 1;
    p[pad + n + i] = x[idx];
  }
  float win[1024];
  for (int i = 0; i < n_fft; i++) { /* periodic Hann (feature.rs:135-142), f32 */
    const float ph = 2.0f * (float)M_PI * (float)i / (float)n_fft;
    win[i] = 0.5f - 0.5f * cosf(ph);
  }
  /* mel filterbank (feature.rs:156-194), f32 */
  float *fb = (float *)calloc((size_t)n_mels * nf, sizeof(float));
  float *hz = (float *)malloc((size_t)(n_mels + 2) * sizeof(float));
  const float mn = hz_to_mel(0.0f), mx = hz_to_mel((float)sr / 2.0f);
  for (int i = 0; i <= n_mels + 1; i++) hz[i] = mel_to_hz(mn + (mx - mn) * (float)i / (float)(n_mels + 1));
  for (int m = 0; m < n_mels; m++) {
    const float l = hz[m], c = hz[m + 1], r = hz[m + 2];
    for (int f = 0; f < nf; f++) {
      const float fq = (float)f * (float)sr / (float)n_fft;
      float v = 0.f;
      if (fq >= l && fq <= c && c > l) v = (fq - l) / (c - l);
      else if (fq > c && fq <= r && r > c) v = (r - fq) / (r - c);
      fb[(size_t)m * nf + f] = v;
    }
    const float bw = hz[m + 2] - hz[m];
    if (bw > 0.f)
      for (int f = 0; f < nf; f++) fb[(size_t)m * nf + f] *= 2.0f / bw;
  }
#pragma omp parallel for schedule(static)
  for (int t = 0; t < frames; t++) {
    double re[1024], im[1024];
    float mag[513];
    for (int i = 0; i < n_fft; i++) {
      re[i] = (double)(p[t * hop + i] * win[i]);
      im[i] = 0.0;
    }
    fft_pow2(re, im, n_fft);
    for (int f = 0; f < nf; f++) {
      const float a = (float)re[f], b = (float)im[f];
      mag[f] = sqrtf(a * a + b * b + 1e-9f);
    }
    for (int m = 0; m < n_mels; m++) {
      float sum = 0.f;
      for (int f = 0; f < nf; f++) sum += fb[(size_t)m * nf + f] * mag[f];
      out[(size_t)m * frames + t] = logf(sum > 1e-5f ? sum : 1e-5f);
    }
  }
  free(p); free(fb); free(hz);
  return frames;
}

/* TimeDelayNetBlock (tdnn.rs:16-82): reflect pad (total / 2 left, the rest
 * right), dilated valid conv with bias, ReLU; x [ci][T] -> y [co][T] */
static int tdnn_forward(const orc_tdnn *b, const float *x, int T, float *y) {
  const int total = b->dil * (b->k - 1), pl = total / 2, pr = total - pl;
  if ((pl > 0 && T < pl + 1) || (pr > 0 && T < pr + 1)) return -1; /* the reference's slices need these */
  const int Tp = T + total;
  float *xp = (float *)malloc((size_t)b->ci * Tp * sizeof(float));
  for (int c = 0; c < b->ci; c++) {
    const float *xi = x + (size_t)c * T;
    float *o = xp + (size_t)c * Tp;
    for (int i = 0; i < pl; i++) o[i] = xi[pl - i];           /* x[pl], ..., x[1] */
    memcpy(o + pl, xi, (size_t)T * sizeof(float));
    for (int i = 0; i < pr; i++) o[pl + T + i] = xi[T - 2 - i]; /* x[T-2], ..., x[T-1-pr] */
  }
#pragma omp parallel for schedule(static)
  for (int o = 0; o < b->co; o++) {
    float *yo = y + (size_t)o * T;
    for (int t = 0; t < T; t++) yo[t] = b->b[o];
    for (int i = 0; i < b->ci; i++) {
      const float *xi = xp + (size_t)i * Tp;
      for (int j = 0; j < b->k; j++) {
        const float wv = b->w[((size_t)o * b->ci + i) * b->k + j];
        for (int t = 0; t < T; t++) yo[t] += wv * xi[t + j * b->dil];
      }
    }
    for (int t = 0; t < T; t++) yo[t] = yo[t] > 0.f ? yo[t] : 0.f;
  }
  free(xp);
  return 0;
}

/* SqueezeExcitationRes2NetBlock (res2net.rs:96-119) on x [C][T] in place */
static int se_block_forward(const orc_se_block *b, float *x, int C, int T) {
  float *h = (float *)malloc((size_t)C * T * sizeof(float));
  float *g = (float *)malloc((size_t)C * T * sizeof(float));
  int rc = tdnn_forward(&b->tdnn1, x, T, h);
  /* Res2Net (res2net.rs:37-58): out = [c0, y1, ..., y_{s-1}], y1 = B1(c1),
   * y_i = B_i(c_i + y_{i-1}) */
  const int cs = C / b->scale;
  memcpy(g, h, (size_t)cs * T * sizeof(float));
  float *in = (float *)malloc((size_t)cs * T * sizeof(float));
  for (int i = 1; i < b->scale && rc == 0; i++) {
    const float *ci = h + (size_t)i * cs * T;
    for (int64_t e = 0; e < (int64_t)cs * T; e++) in[e] = ci[e] + (i > 1 ? g[(size_t)(i - 1) * cs * T + e] : 0.f);
    rc = tdnn_forward(&b->res[i - 1], in, T, g + (size_t)i * cs * T);
  }
  free(in);
  if (rc == 0) rc = tdnn_forward(&b->tdnn2, g, T, h);
  if (rc == 0) { /* squeeze-excitation (res2net.rs:62-90) */
    float *m = (float *)malloc((size_t)C * sizeof(float));
    float *z = (float *)malloc((size_t)b->se_ch * sizeof(float));
    for (int c = 0; c < C; c++) {
      float s = 0.f;
      for (int t = 0; t < T; t++) s += h[(size_t)c * T + t];
      m[c] = s / (float)T;
    }
    for (int j = 0; j < b->se_ch; j++) {
      float s = b->se_b1[j];
      for (int c = 0; c < C; c++) s += b->se_w1[(size_t)j * C + c] * m[c];
      z[j] = s > 0.f ? s : 0.f;
    }
    for (int c = 0; c < C; c++) {
      float s = b->se_b2[c];
      for (int j = 0; j < b->se_ch; j++) s += b->se_w2[(size_t)c * b->se_ch + j] * z[j];
      const float sc = 1.f / (1.f + expf(-s));
      for (int t = 0; t < T; t++) x[(size_t)c * T + t] += h[(size_t)c * T + t] * sc;
    }
    free(m); free(z);
  }
  free(h); free(g);
  return rc;
}

int orc_speaker_forward(const orc_speaker *s, const float *mel, int T, float *emb) {
  if (!s || !mel || T <= 0) return -1;
  const int C = s->channels[1], C4 = s->channels[4];
  float *x = (float *)malloc((size_t)C * T * sizeof(float));
  float *cat = (float *)malloc((size_t)3 * C * T * sizeof(float));
  int rc = tdnn_forward(&s->block0, mel, T, x);
  for (int i = 0; i < 3 && rc == 0; i++) { /* network/mod.rs:75-92 */
    rc = se_block_forward(&s->se[i], x, C, T);
    memcpy(cat + (size_t)i * C * T, x, (size_t)C * T * sizeof(float));
  }
  float *h = (float *)malloc((size_t)C4 * T * sizeof(float));
  if (rc == 0) rc = tdnn_forward(&s->mfa, cat, T, h);
  if (rc == 0) { /* AttentiveStatisticsPooling (pooling.rs:25-72) */
    float *ain = (float *)malloc((size_t)3 * C4 * T * sizeof(float));
    float *mean = (float *)malloc((size_t)C4 * sizeof(float)), *sd = (float *)malloc((size_t)C4 * sizeof(float));
    for (int c = 0; c < C4; c++) {
      float s1 = 0.f, s2 = 0.f;
      for (int t = 0; t < T; t++) {
        const float v = h[(size_t)c * T + t];
        s1 += v;
        s2 += v * v;
      }
      const float mu = s1 / (float)T, var = s2 / (float)T - mu * mu;
      mean[c] = mu;
      sd[c] = sqrtf((var > 0.f ? var : 0.f) + 1e-5f);
      for (int t = 0; t < T; t++) {
        ain[(size_t)c * T + t] = h[(size_t)c * T + t];
        ain[(size_t)(C4 + c) * T + t] = mu;
        ain[(size_t)(2 * C4 + c) * T + t] = sd[c];
      }
    }
    const int A = s->asp_tdnn.co;
    float *a = (float *)malloc((size_t)A * T * sizeof(float));
    rc = tdnn_forward(&s->asp_tdnn, ain, T, a);
    for (int64_t e = 0; e < (int64_t)A * T; e++) a[e] = tanhf(a[e]);
    float *pooled = (float *)malloc((size_t)2 * C4 * sizeof(float));
#pragma omp parallel for schedule(static)
    for (int c = 0; c < C4; c++) {
      float *sc = (float *)malloc((size_t)T * sizeof(float));
      float mx = -INFINITY;
      for (int t = 0; t < T; t++) {
        float v = s->asp_b[c];
        for (int j = 0; j < A; j++) v += s->asp_w[(size_t)c * A + j] * a[(size_t)j * T + t];
        sc[t] = v;
        mx = v > mx ? v : mx;
      }
      float z = 0.f;
      for (int t = 0; t < T; t++) {
        sc[t] = expf(sc[t] - mx);
        z += sc[t];
      }
      float wm = 0.f, w2 = 0.f;
      for (int t = 0; t < T; t++) {
        const float p = sc[t] / z, v = h[(size_t)c * T + t];
        wm += v * p;
        w2 += v * v * p;
      }
      const float wv = w2 - wm * wm;
      pooled[c] = wm;
      pooled[C4 + c] = sqrtf((wv > 0.f ? wv : 0.f) + 1e-5f);
      free(sc);
    }
    for (int o = 0; o < s->enc_dim; o++) { /* fc: Conv1d k1 (network/mod.rs:59-61) */
      float v = s->fc_b[o];
      for (int c = 0; c < 2 * C4; c++) v += s->fc_w[(size_t)o * 2 * C4 + c] * pooled[c];
      emb[o] = v;
    }
    free(ain); free(mean); free(sd); free(a); free(pooled);
  }
  free(x); free(cat); free(h);
  return rc;
}

int orc_speaker_embed(const orc_speaker *s, const float *samples, int n, float *emb) {
  if (!s || !samples || n < 256) return -1;
  const int frames = (n + 768 - 1024) / 256 + 1;
  float *mel = (float *)malloc((size_t)s->mel_dim * frames * sizeof(float));
  int T = orc_speaker_mel(samples, n, s->sample_rate, s->mel_dim, mel, frames);
  int rc = T < 0 ? -1 : orc_speaker_forward(s, mel, T, emb);
  free(mel);
  return rc;
}

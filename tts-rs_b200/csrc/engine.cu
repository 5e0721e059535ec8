// Host runtime of the B200 Qwen3-TTS hot path: model load (bf16 cast +
// fragment packing), paged KV pools, the ragged batch engine (admission,
// prefill, one CUDA-graph-replayed decode frame per step, retirement) and
// the C ABI of include/q3t.h.
//
// The per-request state machine mirrors TalkerGenerator
// (tts_qwen3_tts/src/model/talker/infer/mod.rs:69-311): start = prefill +
// first sample with the suppress list; step = code predictor (15 codebooks)
// -> codec-group embedding (+ trailing text / pad) -> push codes -> stop at
// max_new_tokens -> talker decode -> codec_head -> repetition penalty ->
// sample -> EOS check; finalize = codes [G][T].
#include <cmath>
#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <deque>
#include <memory>
#include <mutex>

#include "codec.cuh"
#include "engine.h"
#include "lm_kernels.cuh"

namespace q3t {

thread_local std::string g_err;
thread_local int64_t g_thread_launch_base = 0;

void set_error(const char *fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
}

template <class F>
static q3t_status guard(F &&f) {
  try {
    f();
    return Q3T_OK;
  } catch (const Status &s) {
    return s.code;
  } catch (const CudaFail &c) {
    set_error("CUDA error %s (%s) in %s", cudaGetErrorName(c.err), cudaGetErrorString(c.err),
              c.what.c_str());
    return Q3T_CUDA_ERROR;
  } catch (const std::bad_alloc &) {
    set_error("host allocation failed");
    return Q3T_CUDA_ERROR;
  }
}

// ----------------------------------------------------------------------------
// Weight upload
// ----------------------------------------------------------------------------
struct Tensors {
  std::map<std::string, const q3t_tensor *> m;
  explicit Tensors(const q3t_model_desc *d) {
    for (int i = 0; i < d->num_tensors; i++)
      if (d->tensors[i].name) m[d->tensors[i].name] = &d->tensors[i];
  }
  const q3t_tensor *find(const std::string &name) const {
    auto it = m.find(name);
    if (it == m.end()) {
      const std::string alt = checkpoint_alias(name);
      if (!alt.empty()) it = m.find(alt);
    }
    return it == m.end() ? nullptr : it->second;
  }
  const q3t_tensor *get(const std::string &name, std::vector<int64_t> shape) const {
    auto it = m.find(name);
    if (it == m.end()) {
      const std::string alt = checkpoint_alias(name);
      if (!alt.empty()) it = m.find(alt);
    }
    if (it == m.end()) FAIL(Q3T_RUNTIME_LOAD, "missing tensor %s", name.c_str());
    const q3t_tensor *t = it->second;
    int64_t n1 = 1, n2 = 1;
    for (int i = 0; i < t->ndim; i++) n1 *= t->shape[i];
    for (auto s : shape) n2 *= s;
    bool ok = n1 == n2 && t->data && (t->dtype == Q3T_F32 || t->dtype == Q3T_BF16);
    if (ok && t->ndim == (int)shape.size())
      for (int i = 0; i < t->ndim; i++) ok = ok && t->shape[i] == shape[i];
    if (!ok) FAIL(Q3T_RUNTIME_LOAD, "tensor %s has an unexpected shape, dtype or no data", name.c_str());
    return t;
  }
};

static int64_t numel(const q3t_tensor *t) {
  int64_t n = 1;
  for (int i = 0; i < t->ndim; i++) n *= t->shape[i];
  return n;
}

// host tensor -> device bf16 row-major (temporary unless arena given)
static uint16_t *to_dev_bf16(const q3t_tensor *t, DevArena *ar, cudaStream_t st) {
  const int64_t n = numel(t);
  uint16_t *d;
  if (ar)
    d = ar->alloc<uint16_t>(n);
  else
    CK(cudaMalloc(&d, n * 2));
  if (t->dtype == Q3T_BF16) {
    CK(cudaMemcpyAsync(d, t->data, n * 2, cudaMemcpyHostToDevice, st));
    CK(cudaStreamSynchronize(st));
  } else {
    float *tmp;
    CK(cudaMalloc(&tmp, n * 4));
    CK(cudaMemcpyAsync(tmp, t->data, n * 4, cudaMemcpyHostToDevice, st));
    f32_to_bf16(tmp, d, n, st);
    CK(cudaStreamSynchronize(st));
    CK(cudaFree(tmp));
  }
  return d;
}

float *upload_f32(const q3t_tensor *t, DevArena &ar, cudaStream_t st) {
  const int64_t n = numel(t);
  float *d = ar.alloc<float>(n);
  if (t->dtype == Q3T_F32) {
    CK(cudaMemcpyAsync(d, t->data, n * 4, cudaMemcpyHostToDevice, st));
    CK(cudaStreamSynchronize(st));
  } else {
    std::vector<float> h(n);
    const uint16_t *s = reinterpret_cast<const uint16_t *>(t->data);
    for (int64_t i = 0; i < n; i++) {
      uint32_t u = (uint32_t)s[i] << 16;
      memcpy(&h[i], &u, 4);
    }
    CK(cudaMemcpyAsync(d, h.data(), n * 4, cudaMemcpyHostToDevice, st));
    CK(cudaStreamSynchronize(st));
  }
  return d;
}

uint16_t *upload_bf16(const q3t_tensor *t, DevArena &ar, cudaStream_t st) {
  return to_dev_bf16(t, &ar, st);
}

// host tensor -> dst (bf16, n elements) on the device
static void upload_into(const q3t_tensor *t, uint16_t *dst, cudaStream_t st) {
  uint16_t *tmp = to_dev_bf16(t, nullptr, st);
  CK(cudaMemcpyAsync(dst, tmp, (size_t)numel(t) * 2, cudaMemcpyDeviceToDevice, st));
  CK(cudaStreamSynchronize(st));
  CK(cudaFree(tmp));
}

// a [N][K] bf16 weight at w with its TMA descriptor
static Linear make_linear(const uint16_t *w, int N, int K, const char *name) {
  if (N % 128 || K % 128) FAIL(Q3T_RUNTIME_LOAD, "linear %s: dims %d x %d not multiples of 128", name, N, K);
  Linear L;
  L.w = w;
  L.N = N;
  L.K = K;
  if (!make_tmap_bf16(&L.tm, w, (uint64_t)K, (uint64_t)N, (uint64_t)K * 2, 64, 128))
    FAIL(Q3T_RUNTIME_LOAD, "linear %s: TMA descriptor encoding failed", name);
  return L;
}

static Linear load_linear(const q3t_tensor *t, int N, int K, DevArena &ar, cudaStream_t st) {
  uint16_t *w = ar.alloc<uint16_t>((size_t)N * K);
  upload_into(t, w, st);
  return make_linear(w, N, K, t->name);
}

// gate [I][H] and up [I][H] -> one [2I][H] matrix whose 128-row blocks are
// [gate rows 64r..64r+63 | up rows 64r..64r+63] (the GE_SILU epilogue pairs them)
static Linear load_gate_up(const q3t_tensor *gate, const q3t_tensor *up, int I, int H, DevArena &ar,
                           cudaStream_t st) {
  if (I % 64) FAIL(Q3T_RUNTIME_LOAD, "gate/up: intermediate %d not a multiple of 64", I);
  uint16_t *g = to_dev_bf16(gate, nullptr, st), *u = to_dev_bf16(up, nullptr, st);
  uint16_t *gu = ar.alloc<uint16_t>((size_t)2 * I * H);
  const size_t blk = (size_t)64 * H * 2;  // bytes of 64 rows
  CK(cudaMemcpy2DAsync(gu, 2 * blk, g, blk, blk, I / 64, cudaMemcpyDeviceToDevice, st));
  CK(cudaMemcpy2DAsync(reinterpret_cast<char *>(gu) + blk, 2 * blk, u, blk, blk, I / 64, cudaMemcpyDeviceToDevice, st));
  CK(cudaStreamSynchronize(st));
  CK(cudaFree(g));
  CK(cudaFree(u));
  return make_linear(gu, 2 * I, H, gate->name);
}

static void load_stack(q3t_model *m, LMStack &S, const q3t_lm_config &c, const std::string &prefix,
                       const Tensors &T, cudaStream_t st) {
  S.cfg = c;
  const int H = c.hidden_size, I = c.intermediate_size, nh = c.num_attention_heads,
            nkv = c.num_key_value_heads, hd = c.head_dim;
  if (hd != 128) FAIL(Q3T_INVALID_INPUT, "%s: head_dim %d unsupported (kernels are built for 128)", prefix.c_str(), hd);
  if (H % 256 || I % 256) FAIL(Q3T_INVALID_INPUT, "%s: hidden/intermediate must be multiples of 256", prefix.c_str());
  if (nh != 2 * nkv) FAIL(Q3T_INVALID_INPUT, "%s: kernels are built for 2 query heads per kv head", prefix.c_str());
  auto &ar = m->arena;
  for (int l = 0; l < c.num_hidden_layers; l++) {
    const std::string p = prefix + ".layers." + std::to_string(l);
    S.in_norm.push_back(upload_f32(T.get(p + ".input_layernorm.weight", {H}), ar, st));
    S.post_norm.push_back(upload_f32(T.get(p + ".post_attention_layernorm.weight", {H}), ar, st));
    S.q_norm.push_back(upload_f32(T.get(p + ".self_attn.q_norm.weight", {hd}), ar, st));
    S.k_norm.push_back(upload_f32(T.get(p + ".self_attn.k_norm.weight", {hd}), ar, st));
    const int Nq = nh * hd, Nk = nkv * hd;
    uint16_t *qkv = ar.alloc<uint16_t>((size_t)(Nq + 2 * Nk) * H);
    upload_into(T.get(p + ".self_attn.q_proj.weight", {Nq, H}), qkv, st);
    upload_into(T.get(p + ".self_attn.k_proj.weight", {Nk, H}), qkv + (size_t)Nq * H, st);
    upload_into(T.get(p + ".self_attn.v_proj.weight", {Nk, H}), qkv + (size_t)(Nq + Nk) * H, st);
    S.qkv.push_back(make_linear(qkv, Nq + 2 * Nk, H, "qkv_proj"));
    S.o.push_back(load_linear(T.get(p + ".self_attn.o_proj.weight", {H, Nq}), H, Nq, ar, st));
    S.gu.push_back(
        load_gate_up(T.get(p + ".mlp.gate_proj.weight", {I, H}), T.get(p + ".mlp.up_proj.weight", {I, H}), I, H, ar, st));
    S.down.push_back(load_linear(T.get(p + ".mlp.down_proj.weight", {H, I}), H, I, ar, st));
  }
  S.final_norm = upload_f32(T.get(prefix + ".norm.weight", {H}), ar, st);
  // rope.rs:21-24: inv_freq[i] = 1 / theta^(i / half), computed in f32 on the host
  std::vector<float> inv(hd / 2);
  for (int i = 0; i < hd / 2; i++) inv[i] = 1.0f / powf(c.rope_theta, (float)i / (float)(hd / 2));
  S.inv_freq = ar.alloc<float>(hd / 2);
  CK(cudaMemcpyAsync(S.inv_freq, inv.data(), inv.size() * 4, cudaMemcpyHostToDevice, st));
  CK(cudaStreamSynchronize(st));
}

}  // namespace q3t

using namespace q3t;

extern "C" q3t_status q3t_model_load(const q3t_model_desc *desc, q3t_model **out) {
  if (!desc || !out) {
    set_error("q3t_model_load: null argument");
    return Q3T_INVALID_INPUT;
  }
  *out = nullptr;
  auto *m = new q3t_model();
  q3t_status rc = guard([&] {
    CK(cudaSetDevice(desc->device));
    m->device = desc->device;
    m->tc = desc->talker;
    m->cc = desc->codec;
    m->has_talker = desc->has_talker != 0;
    m->has_codec = desc->has_codec != 0;
    m->kv_pages = desc->kv_pages > 0 ? desc->kv_pages : 8192;
    m->max_active = desc->max_active > 0 ? desc->max_active : 64;
    if (m->max_active > 64) FAIL(Q3T_INVALID_INPUT, "max_active %d > 64", m->max_active);
    init_kernel_attributes();
    mk_init_attributes();
    {  // keep stream-ordered allocations (codec workspaces) cached between calls
      cudaMemPool_t pool;
      CK(cudaDeviceGetDefaultMemPool(&pool, desc->device));
      uint64_t thr = UINT64_MAX;
      CK(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr));
    }
    cudaStream_t st;
    CK(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    Tensors T(desc);
    if (m->has_talker) {
      const auto &tc = m->tc;
      const int G = tc.num_code_groups;
      if (G < 2 || G > 32) FAIL(Q3T_INVALID_INPUT, "num_code_groups %d unsupported", G);
      if (tc.predictor.hidden_size != tc.talker.hidden_size)
        FAIL(Q3T_INVALID_INPUT, "code predictor hidden %d != talker hidden %d (small_to_mtp_projection unsupported)",
             tc.predictor.hidden_size, tc.talker.hidden_size);
      if (tc.talker.vocab_size > 4096 || tc.predictor.vocab_size > 4096 || tc.talker.vocab_size % 128 ||
          tc.predictor.vocab_size % 128)
        FAIL(Q3T_INVALID_INPUT, "vocab sizes must be multiples of 128 and <= 4096");
      load_stack(m, m->talker, tc.talker, "talker.model", T, st);
      load_stack(m, m->pred, tc.predictor, "talker.code_predictor.model", T, st);
      const int H = tc.talker.hidden_size, V = tc.talker.vocab_size, PV = tc.predictor.vocab_size;
      m->codec_head = load_linear(T.get("talker.codec_head.weight", {V, H}), V, H, m->arena, st);
      m->talker_emb = upload_bf16(T.get("talker.model.codec_embedding.weight", {V, H}), m->arena, st);
      for (int j = 0; j < G - 1; j++) {
        m->cp_emb.push_back(upload_bf16(
            T.get("talker.code_predictor.model.codec_embedding." + std::to_string(j) + ".weight", {PV, H}),
            m->arena, st));
        m->lm_heads.push_back(load_linear(
            T.get("talker.code_predictor.lm_head." + std::to_string(j) + ".weight", {PV, H}), PV, H, m->arena, st));
      }
      m->cp_emb_dev = m->arena.alloc<uint16_t *>(G - 1);
      CK(cudaMemcpyAsync(m->cp_emb_dev, m->cp_emb.data(), (G - 1) * sizeof(uint16_t *), cudaMemcpyHostToDevice,
                         st));
    }
    if (m->has_talker && T.find("talker.model.text_embedding.weight")) {
      // text projection (talker/network/model.rs:22, 76; config.rs:200-209)
      const q3t_tensor *e = T.find("talker.model.text_embedding.weight");
      if (e->ndim != 2) FAIL(Q3T_RUNTIME_LOAD, "talker.model.text_embedding.weight must be 2-D");
      const int Vt = (int)e->shape[0], Ht = (int)e->shape[1], H = m->tc.talker.hidden_size;
      if (Ht % 256 || Ht > 8192) FAIL(Q3T_RUNTIME_LOAD, "text hidden size %d unsupported (multiple of 256)", Ht);
      m->text_vocab = Vt;
      m->text_hidden = Ht;
      m->text_emb = upload_bf16(T.get("talker.model.text_embedding.weight", {Vt, Ht}), m->arena, st);
      m->tp_fc1 = load_linear(T.get("talker.text_projection.linear_fc1.weight", {Ht, Ht}), Ht, Ht, m->arena, st);
      m->tp_b1 = upload_f32(T.get("talker.text_projection.linear_fc1.bias", {Ht}), m->arena, st);
      m->tp_fc2 = load_linear(T.get("talker.text_projection.linear_fc2.weight", {H, Ht}), H, Ht, m->arena, st);
      m->tp_b2 = upload_f32(T.get("talker.text_projection.linear_fc2.bias", {H}), m->arena, st);
    }
    if (m->has_codec) m->codec = codec_load(m, desc, st);
    CK(cudaStreamSynchronize(st));
    CK(cudaStreamDestroy(st));
    // zero-fills (cudaMemset) run on the legacy stream: finish them before any
    // non-blocking library stream touches the buffers
    CK(cudaDeviceSynchronize());
  });
  if (rc != Q3T_OK) {
    q3t_model_free(m);
    return rc;
  }
  *out = m;
  return Q3T_OK;
}

extern "C" void q3t_model_free(q3t_model *m) {
  if (!m) return;
  cudaSetDevice(m->device);
  if (m->tp_st) cudaStreamDestroy(m->tp_st);
  if (m->codec) codec_free(m->codec);
  delete m;
}

// ----------------------------------------------------------------------------
// Batch engine
// ----------------------------------------------------------------------------
namespace q3t {

}  // namespace q3t

namespace q3t {

static int bucket_tok(int B) {
  if (B <= 1) return 1;
  int n = 8;
  while (n < B) n <<= 1;
  return n;
}

static void batch_init(q3t_batch *b, q3t_model *m, const q3t_batch_desc &d) {
  b->m = m;
  b->desc = d;
  const auto &tc = m->tc;
  b->A = d.max_active;
  b->G = tc.num_code_groups;
  b->H = tc.talker.hidden_size;
  b->V = tc.talker.vocab_size;
  b->PV = tc.predictor.vocab_size;
  b->NQKV = (tc.talker.num_attention_heads + 2 * tc.talker.num_key_value_heads) * 128;
  b->NQKVP = (tc.predictor.num_attention_heads + 2 * tc.predictor.num_key_value_heads) * 128;
  b->I2 = 2 * std::max(tc.talker.intermediate_size, tc.predictor.intermediate_size);
  const char *g = getenv("Q3T_GRAPHS");
  b->use_graphs = !(g && g[0] == '0');
  {  // highest priority: the streaming codec's windows fill in behind the frame kernels
    int least = 0, greatest = 0;
    CK(cudaDeviceGetStreamPriorityRange(&least, &greatest));
    CK(cudaStreamCreateWithPriority(&b->st, cudaStreamNonBlocking, greatest));
  }
  CK(cudaEventCreate(&b->ev0));
  CK(cudaEventCreate(&b->ev1));
  for (auto &e : b->evf) CK(cudaEventCreate(&e));
  auto &ar = b->ar;
  const int A = b->A;
  // talker KV pool
  const int nkv = tc.talker.num_key_value_heads, L = tc.talker.num_hidden_layers;
  b->n_pages = (int)std::min<int64_t>(m->kv_pages, (int64_t)A * kPtStride);
  b->t_layer_stride = (int64_t)b->n_pages * nkv * kPage * 128;
  b->tk = ar.alloc<uint16_t>((size_t)b->t_layer_stride * L);
  b->tv = ar.alloc<uint16_t>((size_t)b->t_layer_stride * L);
  for (int p = b->n_pages - 1; p >= 0; p--) b->free_pages.push_back(p);
  CK(cudaMallocHost(&b->h_pt, (size_t)A * kPtStride * sizeof(int)));
  memset(b->h_pt, 0, (size_t)A * kPtStride * sizeof(int));
  b->d_pt = ar.zalloc<int>((size_t)A * kPtStride);
  {  // request inputs come from a stream-ordered pool that keeps its memory
    cudaMemPoolProps pp{};
    pp.allocType = cudaMemAllocationTypePinned;
    pp.location.type = cudaMemLocationTypeDevice;
    pp.location.id = m->device;
    CK(cudaMemPoolCreate(&b->pool, &pp));
    uint64_t keep = UINT64_MAX;
    CK(cudaMemPoolSetAttribute(b->pool, cudaMemPoolAttrReleaseThreshold, &keep));
  }
  CK(cudaMallocHost(&b->h_init, (size_t)A * sizeof(SlotInit)));
  b->d_first_eos = ar.zalloc<int>(A);
  CK(cudaMallocHost(&b->h_first_eos, (size_t)A * sizeof(int)));
  b->d_zero = ar.zalloc<int>(1);
  // predictor pool: slot s owns pages 2s, 2s+1 (capacity 32 >= num_code_groups + 1)
  const int pnkv = tc.predictor.num_key_value_heads, PL = tc.predictor.num_hidden_layers;
  b->p_layer_stride = (int64_t)2 * A * pnkv * kPage * 128;
  b->pk = ar.alloc<uint16_t>((size_t)b->p_layer_stride * PL);
  b->pv = ar.alloc<uint16_t>((size_t)b->p_layer_stride * PL);
  {
    std::vector<int> ppt((size_t)A * 2);
    for (int s = 0; s < A; s++) ppt[2 * s] = 2 * s, ppt[2 * s + 1] = 2 * s + 1;
    b->d_ppt = ar.alloc<int>(ppt.size());
    CK(cudaMemcpyAsync(b->d_ppt, ppt.data(), ppt.size() * 4, cudaMemcpyHostToDevice, b->st));
  }
  // slot state
  b->maxF = kMaxSeq;
  b->hist_cap = kMaxSeq + 1;
  const int G = b->G, H = b->H;
  b->d_codes = ar.zalloc<int64_t>((size_t)A * G);
  b->d_hist_codes = ar.zalloc<int64_t>((size_t)A * b->maxF * G);
  b->d_forced = ar.zalloc<int64_t>((size_t)A * b->maxF * G);
  b->d_forced_count = ar.zalloc<int>(A);
  b->d_raw = ar.zalloc<int32_t>((size_t)A * b->maxF * G);
  b->d_eos = ar.zalloc<int64_t>(A);
  b->d_suppress = ar.zalloc<int64_t>((size_t)A * b->n_suppress_cap);
  b->d_nsup = ar.zalloc<int>(A);
  b->d_hidden = ar.zalloc<float>((size_t)A * H);
  b->d_thist = ar.zalloc<int32_t>((size_t)A * b->hist_cap);
  b->d_thist_len = ar.zalloc<int>(A);
  b->d_sup_on = ar.zalloc<int>(A);
  b->d_params = ar.zalloc<SampleParams>((size_t)A * 2);
  // activation rows: the predictor's pass 0 (two rows per decode token) or a
  // talker pass (decode tokens + prompt-chunk tokens), each rounded up to the
  // token bucket the frame graphs run at, so every GEMM token tile of a
  // bucket lies inside the buffers
  b->Tmax = std::max(2 * bucket_tok(A), kTalkerTok);
  const int T = b->Tmax;
  b->x = ar.zalloc<float>((size_t)T * H);
  b->xn = ar.zalloc<uint16_t>((size_t)T * H);
  b->xg = ar.zalloc<uint16_t>((size_t)T * H);
  b->ss = ar.zalloc<float>((size_t)(std::max(tc.talker.hidden_size, tc.predictor.hidden_size) / 128) * T);
  b->hlog = ar.zalloc<float>((size_t)T * std::max(b->V, b->PV));
  b->q = ar.zalloc<uint16_t>((size_t)T * 128 * std::max(tc.talker.num_attention_heads, tc.predictor.num_attention_heads));
  b->attn = ar.zalloc<uint16_t>((size_t)T * 128 * std::max(tc.talker.num_attention_heads, tc.predictor.num_attention_heads));
  b->act = ar.zalloc<uint16_t>((size_t)T * b->I2 / 2);
  b->tlog = ar.zalloc<float>((size_t)T * b->V);
  b->plog = ar.zalloc<float>((size_t)(G - 1) * A * b->PV);
  b->d_err = ar.zalloc<int>(1);
  CK(cudaMallocHost(&b->h_err, sizeof(int)));
  *b->h_err = 0;
  const int mkv = std::max(nkv, pnkv);
  b->ws.part = ar.zalloc<float>((size_t)T * mkv * kAttnMaxUnits * 2 * 132);
  b->ws.counters = ar.zalloc<int>((size_t)T * mkv);
  // streamed small-batch kernel: on unless Q3T_MK=0 or the device cannot host it
  {
    const char *e = getenv("Q3T_MK");
    b->mk_grid = mk_grid(m->device);
    b->use_mk = !(e && e[0] == '0') && b->mk_grid > 0;
    if (!(e && e[0] == '0') && b->mk_grid <= 0)
      fprintf(stderr, "q3t: the streamed small-batch kernel cannot be resident on device %d; "
                      "single-token steps use the per-layer kernels\n", m->device);
    const int Hm = std::max(tc.talker.hidden_size, tc.predictor.hidden_size);
    b->mk_x = ar.zalloc<uint2>((size_t)2 * kMkMaxTok * Hm);
    b->mk_qkv = ar.zalloc<uint2>((size_t)kMkMaxTok * std::max(b->NQKV, b->NQKVP));
    b->mk_act = ar.zalloc<uint2>((size_t)kMkMaxTok * b->I2 / 2);
    b->mk_attn = ar.zalloc<uint2>((size_t)kMkMaxTok * 128 *
                                  std::max(tc.talker.num_attention_heads, tc.predictor.num_attention_heads));
    b->mk_part = ar.zalloc<uint2>((size_t)kMkMaxTok * mkv * kAttnMaxUnits * 2 * kMkPartLd);
    b->mk_ctr = ar.zalloc<unsigned>(4);
    // bounded-wait tests: Q3T_WAIT_POLLS sets the poll limit of the tagged
    // waits, Q3T_TEST_STALL_WAITS=1 makes every CTA wait on a word nothing
    // sets, so the wait runs out and the call returns Q3T_DEVICE_TIMEOUT
    if (const char *e = getenv("Q3T_WAIT_POLLS")) b->wait_polls = std::max(0, atoi(e));
    if (const char *e = getenv("Q3T_TEST_STALL_WAITS")) b->stall_waits = e[0] == '1';
    const unsigned epoch1 = 1u;  // tags of epoch 0 would match the zero-filled buffers
    CK(cudaMemcpy(b->mk_ctr, &epoch1, sizeof epoch1, cudaMemcpyHostToDevice));
  }
  // persistent frame kernel for the predictor loop: off unless
  // Q3T_FRAME_KERNEL=1 (correct, but measured slower than the per-phase
  // kernels under programmatic dependent launch; see frame.cu)
  {
    const char *e = getenv("Q3T_FRAME_KERNEL");
    if (e && e[0] == '1' && frame_init(m->device, &b->frame_grid, &b->frame_hc)) {
      b->use_frame = true;
      b->frame_bar = ar.zalloc<unsigned>(1);
    }
  }
  // metadata
  b->meta_n = M_HDR + 8 * A + 5 * b->TT();
  b->d_meta = ar.zalloc<int>(b->meta_n);
  CK(cudaMallocHost(&b->h_meta, b->meta_n * sizeof(int)));
  memset(b->h_meta, 0, b->meta_n * sizeof(int));
  b->d_extra = ar.zalloc<const float *>(A);
  CK(cudaMallocHost(&b->h_extra, A * sizeof(float *)));
  const int nchunks = kMaxSeq / kPrefillTok;
  // one block per prefill chunk of every admission of a step (admissions do
  // not synchronise, so a block is rewritten only after the step's sync)
  b->pmeta_blocks = nchunks * A;
  b->d_pmeta = ar.zalloc<int>((size_t)b->pmeta_blocks * b->pmeta_stride());
  CK(cudaMallocHost(&b->h_pmeta, (size_t)b->pmeta_blocks * b->pmeta_stride() * sizeof(int)));
  b->d_eosflag = ar.zalloc<int>(T);
  CK(cudaMallocHost(&b->h_eosflag, T * sizeof(int)));
  CK(cudaMallocHost(&b->h_codes, (size_t)A * G * sizeof(int64_t)));
  b->slots.assign(A, nullptr);
  CK(cudaStreamSynchronize(b->st));
  CK(cudaDeviceSynchronize());  // the arena's cudaMemset zero-fills run on the legacy stream
}

static void batch_destroy(q3t_batch *b) {
  for (auto &kv : b->graphs) cudaGraphExecDestroy(kv.second.exec);
  b->graphs.clear();
  b->programs.clear();
  b->xmaps.clear();
  if (b->h_err) cudaFreeHost(b->h_err);
  for (auto &r : b->reqs)
    for (void *p : {(void *)r.second->d_trailing, (void *)r.second->d_pad, (void *)r.second->d_prompt,
                    (void *)r.second->d_forced, (void *)r.second->d_suppress})
      if (p) cudaFreeAsync(p, b->st);
  if (b->st) cudaStreamSynchronize(b->st);
  if (b->pool) cudaMemPoolDestroy(b->pool);
  if (b->h_pt) cudaFreeHost(b->h_pt);
  if (b->h_init) cudaFreeHost(b->h_init);
  if (b->h_first_eos) cudaFreeHost(b->h_first_eos);
  if (b->h_meta) cudaFreeHost(b->h_meta);
  if (b->h_extra) cudaFreeHost(b->h_extra);
  if (b->h_pmeta) cudaFreeHost(b->h_pmeta);
  if (b->h_eosflag) cudaFreeHost(b->h_eosflag);
  if (b->h_codes) cudaFreeHost(b->h_codes);
  if (b->ev0) cudaEventDestroy(b->ev0);
  if (b->ev1) cudaEventDestroy(b->ev1);
  for (auto &e : b->evf)
    if (e) cudaEventDestroy(e);
  if (b->st) cudaStreamDestroy(b->st);
  b->ar.release();
}

static void check_launches() {
  const char *k = "";
  cudaError_t e = take_launch_error(&k);
  if (e != cudaSuccess) throw CudaFail{e, k};
}

template <class F>
static void run_graph(q3t_batch *b, std::tuple<int, int, int> key, F &&body) {
  if (!b->use_graphs) {
    body();
    check_launches();
    return;
  }
  auto it = b->graphs.find(key);
  if (it == b->graphs.end()) {
    const int64_t l0 = g_launches;
    CK(cudaStreamBeginCapture(b->st, cudaStreamCaptureModeThreadLocal));
    body();
    cudaGraph_t graph = nullptr;
    cudaError_t e = cudaStreamEndCapture(b->st, &graph);
    const char *kname = "";
    cudaError_t le = take_launch_error(&kname);
    if (e != cudaSuccess || le != cudaSuccess) {
      fprintf(stderr, "q3t: graph capture failed (%s / %s in %s); running without graphs\n",
              cudaGetErrorString(e), cudaGetErrorString(le), kname);
      if (graph) cudaGraphDestroy(graph);
      cudaGetLastError();
      b->use_graphs = false;
      g_launches = l0;
      body();
      check_launches();
      return;
    }
    GraphEntry ge;
    ge.nodes = g_launches - l0;
    g_launches = l0;
    CK(cudaGraphInstantiate(&ge.exec, graph, 0));
    cudaGraphDestroy(graph);
    it = b->graphs.emplace(key, ge).first;
  }
  CK(cudaGraphLaunch(it->second.exec, b->st));
  g_launches += it->second.nodes;
}

// minimum pages per attention work unit: larger with more tokens in the
// batch, so that the units stay a few waves deep at every batch size
static int attn_pw(int max_tok) { return max_tok >= 32 ? 8 : max_tok >= 8 ? 2 : 1; }
// attention units per (token, head) for kv length L, rounded up to a power of
// two (it keys the CUDA graphs); the device uses the same page split
static int bucket_units(int L, int pw) {
  const int pages = (L + 15) / 16, per = std::max(pw, (pages + kAttnMaxUnits - 1) / kAttnMaxUnits);
  int s = (pages + per - 1) / per, n = 1;
  while (n < s) n <<= 1;
  return n;
}

static KVView talker_kv(q3t_batch *b) {
  return KVView{b->tk, b->tv, b->t_layer_stride, b->d_pt, kPtStride,
                b->m->tc.talker.num_key_value_heads};
}
static KVView pred_kv(q3t_batch *b) {
  return KVView{b->pk, b->pv, b->p_layer_stride, b->d_ppt, 2, b->m->tc.predictor.num_key_value_heads};
}


// ---------------------------------------------------------------------------
// X = bf16 rows of a batch buffer, row t at x + t * ldx, `width` columns
// (default ldx) and `rows` rows (default Tmax), loaded by TMA (descriptor per
// buffer, row pitch and token-tile height, made on first use); GEMM timeouts
// go to d_err.
static GemmArgs gemm_bf16_x(q3t_batch *b, GemmArgs g, const uint16_t *x, int ldx, int width = 0, int rows = 0) {
  g.xmode = GX_BF16;
  g.xb = x;
  g.ldx = ldx;
  g.err = b->d_err;
  const auto key = std::make_tuple((const void *)x, ldx, g.nt);
  auto it = b->xmaps.find(key);
  if (it == b->xmaps.end()) {
    CUtensorMap m;
    if (!make_tmap_bf16(&m, x, (uint64_t)(width ? width : ldx), (uint64_t)(rows ? rows : b->Tmax), (uint64_t)ldx * 2,
                        64, (uint32_t)(8 * g.nt)))
      FAIL(Q3T_CUDA_ERROR, "TMA descriptor encoding failed for an activation buffer");
    it = b->xmaps.emplace(key, m).first;
  }
  g.tx = it->second;
  return g;
}

// ---------------------------------------------------------------------------
// Phase emitter: the decode frame is built once per (token bucket mt,
// attention unit bucket ms) as a phase list and captured into a CUDA graph;
// the per-step inputs (active slots, positions, frames, trailing-text rows,
// step counter) live in the device metadata the phases point at.  With
// direct = true (prefill, sessions) each phase launches as it is emitted.
// ---------------------------------------------------------------------------
struct ProgBuilder {
  q3t_batch *b;
  bool direct;
  std::vector<Phase> ph;
  static Phase phase(int type, int max_tok) {
    Phase p;
    memset(&p, 0, sizeof(Phase));
    p.type = type;
    p.max_tok = max_tok;
    return p;
  }
  void push(const Phase &p) {
    if (direct)
      run_phases(&p, 1, b->st);
    else
      ph.push_back(p);
  }
  void norm(const RmsArgs &a, int max_tok) {
    Phase p = phase(PH_NORM, max_tok);
    p.norm = a;
    push(p);
  }
  void gemm(const GemmArgs &g, int max_tok) {
    Phase p = phase(PH_GEMM, max_tok);
    p.gemm = g;
    push(p);
  }
  void sample(const SampleArgs &a, int max_tok, const RmsArgs *tail) {
    Phase p = phase(PH_SAMPLE, max_tok);
    p.smp = a;
    if (tail) {
      p.has_tail = 1;
      p.tail = *tail;
    }
    push(p);
  }
  // X = bf16 rows [Tmax][ldx] of a batch buffer, loaded by TMA
  GemmArgs bf16_x(GemmArgs g, const uint16_t *x, int ldx) const { return gemm_bf16_x(b, g, x, ldx); }
  // X = RMSNorm(x rows t * row_mul + row_add) from the residual stream and
  // the sum-of-squares partials its last GE_RESID epilogue wrote
  GemmArgs norm_x(GemmArgs g, const float *gamma, float eps, int row_mul = 1, int row_add = 0) const {
    g.xmode = GX_NORM;
    g.x = b->x;
    g.ldx = g.K;
    g.xrow_mul = row_mul;
    g.xrow_add = row_add;
    g.ss = b->ss;
    g.nss = g.K / 128;
    g.ss_ld = b->Tmax;
    g.gamma = gamma;
    g.eps = eps;
    g.err = b->d_err;
    return g;
  }
  // X = RMSNorm(x rows t * row_mul + row_add) as GX_SCALED: the bf16 rows of
  // x * gamma the residual epilogue that wrote x left in xg, and the scale
  // from its sum-of-squares partials.  The persistent frame kernel takes
  // GX_NORM instead.
  GemmArgs scaled_x(GemmArgs g, const float *gamma, float eps, int row_mul = 1, int row_add = 0) const {
    if (b->use_frame) return norm_x(g, gamma, eps, row_mul, row_add);
    const int H = g.K;
    g = row_mul == 1 ? gemm_bf16_x(b, g, b->xg, H)
                     : gemm_bf16_x(b, g, b->xg + (size_t)row_add * H, row_mul * H, H,
                                   (b->Tmax - 1 - row_add) / row_mul + 1);
    g.xmode = GX_SCALED;
    g.xrow_mul = row_mul;
    g.xrow_add = row_add;
    g.ss = b->ss;
    g.nss = g.K / 128;
    g.ss_ld = b->Tmax;
    g.eps = eps;
    return g;
  }
  // residual epilogue; next_gamma (nullable): the gamma of the RMSNorm that
  // reads the new rows through scaled_x
  GemmArgs resid(GemmArgs g, const float *next_gamma) const {
    g.epi = GE_RESID;
    g.y = b->x;
    g.ldy = g.N;
    g.ss_out = b->ss;
    g.ss_ld = b->Tmax;
    if (!b->use_frame && next_gamma) {
      g.xg_out = b->xg;
      g.xg_gamma = next_gamma;
    }
    return g;
  }
  // One decoder stack (layer.rs:23-44) over the tokens of tv; the caller has
  // built the input rows x and their normalised bf16 copy xn.  Afterwards x
  // holds the output residual rows and ss their sum-of-squares partials,
  // and with out_gamma xg holds bf16(x * out_gamma) for a scaled_x reader.
  void stack(const LMStack &S, KVView kv, TokView tv, int max_tok, int max_units, int pw,
             const float *out_gamma = nullptr) {
    const auto &c = S.cfg;
    const int H = c.hidden_size, I = c.intermediate_size, nh = c.num_attention_heads, nkv = c.num_key_value_heads;
    const int QD = nh * 128;
    const float eps = c.rms_norm_eps;
    for (int l = 0; l < c.num_hidden_layers; l++) {
      GemmArgs q = gemm_args(S.qkv[l], tv.ntok, max_tok);
      q = l == 0 ? bf16_x(q, b->xn, H) : scaled_x(q, S.in_norm[l], eps);
      q.epi = GE_QKV;
      q.q_norm = S.q_norm[l];
      q.k_norm = S.k_norm[l];
      q.inv_freq = S.inv_freq;
      q.nh = nh;
      q.nkv = nkv;
      q.tv = tv;
      q.q = b->q;
      q.kv = kv;
      q.layer = l;
      gemm(q, max_tok);
      Phase at = phase(PH_ATTN, max_tok);
      AttnArgs &aa = at.attn;
      aa.q = b->q;
      aa.kv = kv;
      aa.layer = l;
      aa.tv = tv;
      aa.nh = nh;
      aa.pw = pw;
      aa.max_units = max_units;
      aa.scale = 1.0f / sqrtf(128.0f);
      aa.ws = b->ws;
      aa.out = b->attn;
      push(at);
      gemm(resid(bf16_x(gemm_args(S.o[l], tv.ntok, max_tok), b->attn, QD), S.post_norm[l]), max_tok);
      GemmArgs gu = scaled_x(gemm_args(S.gu[l], tv.ntok, max_tok), S.post_norm[l], eps);
      gu.epi = GE_SILU;
      gu.h = b->act;
      gu.ldh = I;
      gemm(gu, max_tok);
      gemm(resid(bf16_x(gemm_args(S.down[l], tv.ntok, max_tok), b->act, I),
                 l + 1 < c.num_hidden_layers ? S.in_norm[l + 1] : out_gamma),
           max_tok);
    }
  }
};

// ---------------------------------------------------------------------------
// Programs of the streamed small-batch kernel (mk.cu): the same decoder
// stack as ProgBuilder::stack, as GEMV and attention stages over the batch
// buffers; token rows 0..ntok-1 of x / act / attn.
// ---------------------------------------------------------------------------
static MkStage mk_gemv(const Linear &W) {
  MkStage s;
  memset(&s, 0, sizeof s);
  s.op = MK_GEMV;
  s.g.w = W.w;
  s.g.N = W.N;
  s.g.K = W.K;
  return s;
}

// One decoder stack over input rows x; returns the stack's output rows.
// The residual stream alternates between the two tagged x buffers.
static MkIn mk_stack(q3t_batch *b, const LMStack &S, KVView kv, MkIn x, std::vector<MkStage> &out) {
  const auto &c = S.cfg;
  const int H = c.hidden_size, I = c.intermediate_size, nh = c.num_attention_heads, nkv = c.num_key_value_heads;
  const int NQ = (nh + 2 * nkv) * 128;
  const float eps = c.rms_norm_eps;
  int buf = 0;
  auto xbuf = [&](int stage) {
    MkIn r{nullptr, b->mk_x + (size_t)buf * kMkMaxTok * H, stage, H};
    buf ^= 1;
    return r;
  };
  for (int l = 0; l < c.num_hidden_layers; l++) {
    const int s_qkv = (int)out.size();
    MkStage q = mk_gemv(S.qkv[l]);
    q.g.xsrc = MKX_NORM;
    q.g.x = x;
    q.g.gamma = S.in_norm[l];
    q.g.eps = eps;
    q.g.epi = MKE_TAG;
    q.g.yt = b->mk_qkv;
    q.g.ldy = NQ;
    out.push_back(q);
    const int s_at = (int)out.size();
    MkStage at;
    memset(&at, 0, sizeof at);
    at.op = MK_ATTN;
    at.a.qkv = b->mk_qkv;
    at.a.qkv_stage = s_qkv;
    at.a.ldq = NQ;
    at.a.q_norm = S.q_norm[l];
    at.a.k_norm = S.k_norm[l];
    at.a.inv_freq = S.inv_freq;
    at.a.eps = eps;
    at.a.scale = 1.0f / sqrtf(128.0f);
    at.a.kv = kv;
    at.a.layer = l;
    at.a.nh = nh;
    at.a.part = b->mk_part;
    at.a.out = b->mk_attn;
    at.a.ldo = nh * 128;
    out.push_back(at);
    MkStage o = mk_gemv(S.o[l]);
    o.g.xsrc = MKX_TAGGED;
    o.g.x = MkIn{nullptr, b->mk_attn, s_at, nh * 128};
    o.g.epi = MKE_RESID;
    o.g.res = x;
    const MkIn xo = xbuf((int)out.size());
    o.g.yt = const_cast<uint2 *>(xo.w);
    o.g.ldy = H;
    out.push_back(o);
    x = xo;
    const int s_gu = (int)out.size();
    MkStage gu = mk_gemv(S.gu[l]);
    gu.g.pairs = 1;
    gu.g.xsrc = MKX_NORM;
    gu.g.x = x;
    gu.g.gamma = S.post_norm[l];
    gu.g.eps = eps;
    gu.g.epi = MKE_SILU;
    gu.g.yt = b->mk_act;
    gu.g.ldy = I;
    out.push_back(gu);
    MkStage dn = mk_gemv(S.down[l]);
    dn.g.xsrc = MKX_TAGGED;
    dn.g.x = MkIn{nullptr, b->mk_act, s_gu, I};
    dn.g.epi = MKE_RESID;
    dn.g.res = x;
    const MkIn xd = xbuf((int)out.size());
    dn.g.yt = const_cast<uint2 *>(xd.w);
    dn.g.ldy = H;
    out.push_back(dn);
    x = xd;
  }
  return x;
}

enum MkProg { MKP_TALKER_DECODE = 1 };

// The device copy of a program, built on first use.
static std::pair<MkStage *, int> mk_program(q3t_batch *b, int kind) {
  auto it = b->mk_progs.find(kind);
  if (it != b->mk_progs.end()) return it->second;
  q3t_model *m = b->m;
  std::vector<MkStage> st;
  if (kind == MKP_TALKER_DECODE) {  // talker decode step (model.rs:94-113) + codec_head
    const MkIn x = mk_stack(b, m->talker, talker_kv(b), MkIn{b->x, nullptr, -1, b->H}, st);
    MkStage hd = mk_gemv(m->codec_head);
    hd.g.xsrc = MKX_NORM;
    hd.g.x = x;
    hd.g.gamma = m->talker.final_norm;
    hd.g.eps = m->tc.talker.rms_norm_eps;
    hd.g.hid_out = b->d_hidden;
    hd.g.hid_slot = b->d_meta + b->off_slot();
    hd.g.epi = MKE_F32;
    hd.g.y = b->tlog;
    hd.g.ldy = b->V;
    st.push_back(hd);
  }
  for (const MkStage &s : st) {
    if (s.op == MK_GEMV && ((s.g.K != 1024 && s.g.K != 2048 && s.g.K != 3072) || (s.g.pairs && s.g.N % 128) ||
                            (s.g.epi == MKE_RESID && (s.g.N + b->mk_grid - 1) / b->mk_grid > kMkMaxRes)))
      FAIL(Q3T_INVALID_INPUT, "streamed kernel: unsupported GEMV shape %d x %d", s.g.N, s.g.K);
  }
  if (st.empty() || (int)st.size() > kMkMaxStages) FAIL(Q3T_INVALID_INPUT, "streamed kernel: bad program size");
  MkStage *d = b->ar.alloc<MkStage>(st.size());
  CK(cudaMemcpyAsync(d, st.data(), st.size() * sizeof(MkStage), cudaMemcpyHostToDevice, b->st));
  CK(cudaStreamSynchronize(b->st));
  return b->mk_progs[kind] = std::make_pair(d, (int)st.size());
}

// Reads and clears the device error word; DEVICE_TIMEOUT if a bounded wait gave up.
static void check_device_error(q3t_batch *b, const char *what) {
  CK(cudaMemcpyAsync(b->h_err, b->d_err, sizeof(int), cudaMemcpyDeviceToHost, b->st));
  CK(cudaStreamSynchronize(b->st));
  if (*b->h_err) {
    const int e = *b->h_err;
    *b->h_err = 0;
    CK(cudaMemsetAsync(b->d_err, 0, sizeof(int), b->st));
    FAIL(Q3T_DEVICE_TIMEOUT, "%s: a bounded device wait gave up (code %d)", what, e);
  }
}

// Prompt chunk / isolated step: input rows already in x; normalises them,
// runs the talker stack.
static void run_stack(q3t_batch *b, const LMStack &S, KVView kv, TokView tv, int max_tok, int max_units) {
  const auto &c = S.cfg;
  ProgBuilder P{b, true, {}};
  P.norm(rms_args(b->x, c.hidden_size, 1, 0, Part{}, S.in_norm[0], b->xn, c.hidden_size, c.hidden_size,
                  c.rms_norm_eps, tv.ntok, nullptr, nullptr),
         max_tok);
  P.stack(S, kv, tv, max_tok, max_units, attn_pw(max_tok));
}

static SampleArgs base_sample(q3t_batch *b) {
  SampleArgs a{};
  a.params = b->d_params;
  a.codes = b->d_codes;
  a.G = b->G;
  a.forced = b->d_forced;
  a.force_on = b->d_forced_count;
  a.max_frames = b->maxF;
  a.hist = b->d_thist;
  a.hist_len = b->d_thist_len;
  a.hist_cap = b->hist_cap;
  a.eos = b->d_eos;
  a.raw = b->d_raw;
  return a;
}

// The code-predictor loop of a decode frame over the frame's decode tokens.
static void build_pred(q3t_batch *b, int mt, std::vector<Phase> &out) {
  q3t_model *m = b->m;
  const auto &tc = m->tc;
  const int G = b->G, H = b->H, PV = b->PV;
  int *meta = b->d_meta;
  const int *ntokB = meta + M_NTOK_B, *ntok2B = meta + M_NTOK_2B;
  const int *slot = meta + b->off_slot(), *frame = meta + b->off_frame();
  ProgBuilder P{b, false, {}};
  const auto &pc = tc.predictor;
  // ---- code predictor (infer/mod.rs:434-535) ----
  // pass 0 input rows: [talker hidden, talker codec embedding of code 0]
  {
    RmsArgs a = rms_args(b->x, H, 1, 0, Part{}, m->pred.in_norm[0], b->xn, H, H, pc.rms_norm_eps, ntok2B, nullptr,
                         nullptr);
    a.emb.src = 1;
    a.emb.G = G;
    a.emb.hidden = b->d_hidden;
    a.emb.emb0 = m->talker_emb;
    a.emb.codes = b->d_codes;
    a.emb.slot = slot;
    P.norm(a, 2 * mt);
  }
  for (int j = 0; j < G - 1; j++) {
    if (j == 0) {
      TokView tv0{ntok2B, meta + b->off_p0seq(), meta + b->off_p0pos(), 0};
      P.stack(m->pred, pred_kv(b), tv0, 2 * mt, 1, kPredPages, m->pred.final_norm);
    } else {
      TokView tvj{ntokB, slot, meta + b->off_zero(), j + 1};
      P.stack(m->pred, pred_kv(b), tvj, mt, 1, kPredPages, m->pred.final_norm);
    }
    // lm_head j on the final-normed last position of each token's pass
    GemmArgs hg = P.scaled_x(gemm_args(m->lm_heads[j], ntokB, mt), m->pred.final_norm, pc.rms_norm_eps,
                             j == 0 ? 2 : 1, j == 0 ? 1 : 0);
    hg.epi = GE_F32;
    hg.y = b->hlog;
    hg.ldy = PV;
    P.gemm(hg, mt);
    SampleArgs a = base_sample(b);
    a.part = Part{b->hlog, 1, 0, PV};
    a.logits = b->plog + (size_t)j * b->A * PV;
    a.ldl = PV;
    a.V = PV;
    a.ntok = ntokB;
    a.slot = slot;
    a.use_pred_params = 1;
    a.col = j + 1;
    a.frame = frame;
    a.fadd = 0;
    a.hist_mode = 2;
    a.seed_p = meta + M_SEED;
    a.step_seed = 0;
    // the tail builds the next input row of this token and normalises it
    RmsArgs t;
    if (j + 1 < G - 1) {
      t = rms_args(b->x, H, 1, 0, Part{}, m->pred.in_norm[0], b->xn, H, H, pc.rms_norm_eps, ntokB, nullptr, nullptr);
      t.emb.src = 2;
      t.emb.G = G;
      t.emb.col = j + 1;
      t.emb.emb = m->cp_emb[j];
      t.emb.codes = b->d_codes;
      t.emb.slot = slot;
    } else {  // next talker input: codec-group embedding + trailing text / pad
      t = rms_args(b->x, H, 1, 0, Part{}, m->talker.in_norm[0], b->xn, H, H, tc.talker.rms_norm_eps, ntokB, nullptr,
                   nullptr);
      t.emb.src = 3;
      t.emb.G = G;
      t.emb.emb0 = m->talker_emb;
      t.emb.embs = (const uint16_t *const *)m->cp_emb_dev;
      t.emb.codes = b->d_codes;
      t.emb.slot = slot;
      t.emb.extra = b->d_extra;
      t.emb.frame = frame;
      t.emb.hist = b->d_hist_codes;
      t.emb.hist_frames = b->maxF;
    }
    P.sample(a, mt, &t);
  }
  out.swap(P.ph);
}

// The talker pass of a decode frame (model.rs:94-113) over the decode tokens
// followed by this step's prompt-chunk tokens (chunked prefill, infer/mod.rs:
// 135-147: causal by position, K/V appended to the request's pages), then
// the final norm, codec_head and sampler over the head tokens: the decode
// tokens and the last prompt token of every prompt completed in this step
// (TalkerGenerator::start's first sample with the suppress list,
// :148-157).  with_prefill: the prompt rows were copied into x after the
// code-predictor loop, so every talker row is normalised first.
static void build_talker(q3t_batch *b, int mt, int max_units, bool with_prefill, std::vector<Phase> &out) {
  q3t_model *m = b->m;
  const auto &tc = m->tc;
  const int H = b->H, V = b->V;
  int *meta = b->d_meta;
  const int *ntokT = meta + M_NTOK_T, *ntokH = meta + M_NTOK_H;
  const int *hslot = meta + b->off_hslot();
  ProgBuilder P{b, false, {}};
  if (with_prefill)
    P.norm(rms_args(b->x, H, 1, 0, Part{}, m->talker.in_norm[0], b->xn, H, H, tc.talker.rms_norm_eps, ntokT, nullptr,
                    nullptr),
           mt);
  TokView tvt{ntokT, meta + b->off_tseq(), meta + b->off_ttpos(), 0};
  P.stack(m->talker, talker_kv(b), tvt, mt, max_units, attn_pw(mt));
  RmsArgs fn = rms_args(b->x, H, 1, 0, Part{}, m->talker.final_norm, b->xn, H, H, tc.talker.rms_norm_eps, ntokH,
                        b->d_hidden, hslot);
  fn.row_idx = meta + b->off_hrow();
  P.norm(fn, mt);
  GemmArgs hg = P.bf16_x(gemm_args(m->codec_head, ntokH, mt), b->xn, H);
  hg.epi = GE_F32;
  hg.y = b->hlog;
  hg.ldy = V;
  P.gemm(hg, mt);
  SampleArgs a = base_sample(b);
  a.part = Part{b->hlog, 1, 0, V};
  a.logits = b->tlog;
  a.ldl = V;
  a.V = V;
  a.ntok = ntokH;
  a.slot = hslot;
  a.use_pred_params = 0;
  a.suppress = b->d_suppress;  // applied where sup_on[slot] (a first token of a prompt with a suppress list)
  a.suppress_ld = b->n_suppress_cap;
  a.n_sup = b->d_nsup;
  a.sup_on = b->d_sup_on;
  a.col = 0;
  a.frame = meta + b->off_hframe();  // decode token: its frame; first token: -1 (record index 0)
  a.fadd = 1;
  a.hist_mode = 1;
  a.eos_flag = b->d_eosflag;
  a.seed_p = meta + M_SEED;
  a.step_seed = 1;
  P.sample(a, mt, nullptr);
  out.swap(P.ph);
}

// Prompt rows of a chunk: x rows [row0, row0 + rows) <- src (device rows of H floats).
struct PromptCopy {
  const float *src;
  int rows, row0;
};

// Eager launch of a phase list with an event after each phase; adds the
// per-shape device times to `by_shape` (Q3T_FRAME_PROFILE).
static void profile_phases(q3t_batch *b, const std::vector<Phase> &pr, const char *part,
                           std::map<std::string, std::pair<int, double>> &by_shape, double &total) {
  const size_t n = pr.size();
  std::vector<cudaEvent_t> ev(n + 1);
  for (auto &e : ev) CK(cudaEventCreate(&e));
  CK(cudaEventRecord(ev[0], b->st));
  for (size_t i = 0; i < n; i++) {
    run_phases(&pr[i], 1, b->st);
    CK(cudaEventRecord(ev[i + 1], b->st));
  }
  CK(cudaStreamSynchronize(b->st));
  for (size_t i = 0; i < n; i++) {
    float ms = 0.f;
    CK(cudaEventElapsedTime(&ms, ev[i], ev[i + 1]));
    const Phase &p = pr[i];
    char key[96];
    if (p.type == PH_GEMM)
      snprintf(key, sizeof key, "%s gemm N%d K%d cs%d epi%d", part, p.gemm.N, p.gemm.K, p.gemm.cs, p.gemm.epi);
    else
      snprintf(key, sizeof key, "%s type%d", part, p.type);
    by_shape[key].first++;
    by_shape[key].second += ms * 1e3;
    total += ms * 1e3;
  }
  for (auto &e : ev) cudaEventDestroy(e);
}

// Runs a decode frame: the code-predictor loop over the B decode tokens
// (bucket mt; skipped when B == 0), the prompt-row copies of this step's
// chunks, then the talker pass over the talker tokens (bucket mtT).  Each
// part is one CUDA graph per bucket, captured on first use; the predictor
// loop runs as one persistent k_frame launch where that is switched on.
// Q3T_FRAME_PROFILE=1 instead launches the phases eagerly with an event
// after each and prints per-phase device times.
static void enqueue_frame(q3t_batch *b, int B, int mt, int mtT, int max_units, bool with_prefill,
                          const std::vector<PromptCopy> &copies) {
  const auto pkey = std::make_pair(mt, -1);
  const auto tkey = std::make_pair(mtT, 2 * max_units + (with_prefill ? 1 : 0));
  const std::vector<Phase> *pp = nullptr;
  if (B > 0) {
    auto it = b->programs.find(pkey);
    if (it == b->programs.end()) {
      std::vector<Phase> ph;
      build_pred(b, mt, ph);
      it = b->programs.emplace(pkey, std::move(ph)).first;
    }
    pp = &it->second;
  }
  auto tt = b->programs.find(tkey);
  if (tt == b->programs.end()) {
    std::vector<Phase> ph;
    build_talker(b, mtT, max_units, with_prefill, ph);
    tt = b->programs.emplace(tkey, std::move(ph)).first;
  }
  const std::vector<Phase> &tp = tt->second;
  auto do_copies = [&] {
    for (const PromptCopy &c : copies)
      CK(cudaMemcpyAsync(b->x + (size_t)c.row0 * b->H, c.src, (size_t)c.rows * b->H * 4, cudaMemcpyDeviceToDevice,
                         b->st));
  };
  if (getenv("Q3T_FRAME_PROFILE")) {
    std::map<std::string, std::pair<int, double>> by_shape;
    double pred = 0, talk = 0;
    if (pp) profile_phases(b, *pp, "pred", by_shape, pred);
    do_copies();
    profile_phases(b, tp, "talk", by_shape, talk);
    fprintf(stderr, "phase profile (eager) B=%d mt=%d mtT=%d prefill=%d: pred %.1f us talker %.1f us\n", B, mt, mtT,
            (int)with_prefill, pred, talk);
    for (auto &kv : by_shape)
      fprintf(stderr, "   %-36s %4d x %8.2f us = %9.1f us\n", kv.first.c_str(), kv.second.first,
              kv.second.second / kv.second.first, kv.second.second);
    check_launches();
    return;
  }
  // profiling: Q3T_KERNEL_TRACE=<file> records every kernel of this frame
  // (grid id, per-CTA device timestamps) and writes the records to the file
  const char *ktr = getenv("Q3T_KERNEL_TRACE");
  const bool ktrace = ktr && ktr[0] && trace_start((size_t)1 << 18, b->st);
  CK(cudaEventRecord(b->evf[0], b->st));
  if (pp) {
    const std::vector<Phase> &pr = *pp;
    const int n = (int)pr.size();
    Phase *fp = nullptr;
    if (b->use_frame) {
      auto fit = b->frame_progs.find(pkey);
      if (fit == b->frame_progs.end()) {
        bool ok = true;
        for (int i = 0; i < n && ok; i++) ok = frame_phase_ok(pr[i], b->frame_hc);
        Phase *d = nullptr;
        if (ok) {
          std::vector<Phase> cp(pr);
          int next = -1;  // Phase::pad = the next GEMM phase, which the kernel's weight prefetch follows
          for (int i = n - 1; i >= 0; i--) {
            cp[i].pad = next;
            if (cp[i].type == PH_GEMM) next = i;
          }
          d = b->ar.alloc<Phase>(n);
          CK(cudaMemcpyAsync(d, cp.data(), (size_t)n * sizeof(Phase), cudaMemcpyHostToDevice, b->st));
          CK(cudaStreamSynchronize(b->st));
        }
        fit = b->frame_progs.emplace(pkey, d).first;
      }
      fp = fit->second;
    }
    const char *tr = fp ? getenv("Q3T_FRAME_TRACE") : nullptr;  // profiling: per-phase device timestamps
    if (tr && tr[0]) {
      const size_t nt = (size_t)b->frame_grid * n * 8;
      unsigned long long *d_tr = nullptr;
      CK(cudaMallocAsync((void **)&d_tr, nt * 8, b->st));
      CK(cudaMemsetAsync(d_tr, 0, nt * 8, b->st));
      frame_launch(FrameArgs{fp, n, b->frame_bar, b->d_err, b->frame_hc, d_tr}, b->frame_grid, b->st);
      check_launches();
      std::vector<unsigned long long> h(nt);
      CK(cudaMemcpyAsync(h.data(), d_tr, nt * 8, cudaMemcpyDeviceToHost, b->st));
      CK(cudaStreamSynchronize(b->st));
      CK(cudaFreeAsync(d_tr, b->st));
      if (FILE *f = fopen(tr, "wb")) {
        const int hdr[2] = {b->frame_grid, n};
        fwrite(hdr, sizeof hdr, 1, f);
        std::vector<int> types(n);
        for (int i = 0; i < n; i++) types[i] = pr[i].type;
        fwrite(types.data(), sizeof(int), n, f);
        fwrite(h.data(), 8, nt, f);
        fclose(f);
      }
    } else if (fp) {
      run_graph(b, std::make_tuple(6, mt, 0), [&] {
        frame_launch(FrameArgs{fp, n, b->frame_bar, b->d_err, b->frame_hc, nullptr}, b->frame_grid, b->st);
      });
    } else {
      run_graph(b, std::make_tuple(4, mt, 0), [&] { run_phases(pr.data(), n, b->st); });
    }
  }
  CK(cudaEventRecord(b->evf[1], b->st));
  do_copies();
  run_graph(b, std::make_tuple(5, mtT, tkey.second), [&] { run_phases(tp.data(), (int)tp.size(), b->st); });
  CK(cudaEventRecord(b->evf[2], b->st));
  b->frame_timed = true;
  check_launches();
  if (ktrace) {
    std::vector<TraceRec> rec;
    trace_stop(rec, b->st);
    if (FILE *f = fopen(ktr, "wb")) {
      const int n = (int)rec.size(), sz = (int)sizeof(TraceRec);
      fwrite(&n, 4, 1, f);
      fwrite(&sz, 4, 1, f);
      fwrite(rec.data(), sizeof(TraceRec), rec.size(), f);
      fclose(f);
    }
  }
}

static int alloc_page(q3t_batch *b, Req *r) {
  if (b->free_pages.empty()) return -1;
  const int p = b->free_pages.back();
  b->free_pages.pop_back();
  const int idx = (int)r->pages.size();
  r->pages.push_back(p);
  b->h_pt[(size_t)r->slot * kPtStride + idx] = p;
  b->pt_lo = std::min(b->pt_lo, r->slot);
  b->pt_hi = std::max(b->pt_hi, r->slot);
  return p;
}

// Uploads the page-table rows changed since the last upload (one copy from
// pinned memory, ordered before the kernels that read them).
static void flush_pages(q3t_batch *b) {
  if (b->pt_hi < b->pt_lo) return;
  const size_t off = (size_t)b->pt_lo * kPtStride, n = (size_t)(b->pt_hi - b->pt_lo + 1) * kPtStride;
  CK(cudaMemcpyAsync(b->d_pt + off, b->h_pt + off, n * sizeof(int), cudaMemcpyHostToDevice, b->st));
  b->h2d += (int64_t)n * sizeof(int);
  b->pt_lo = 1 << 30;
  b->pt_hi = -1;
}

// Pages for `len` tokens of r; the page-table rows go to the device with the
// next flush_pages(), which every path calls before its kernels run.
static bool ensure_pages(q3t_batch *b, Req *r, int len) {
  const int need = (len + kPage - 1) / kPage;
  if (need > kPtStride) return false;
  while ((int)r->pages.size() < need)
    if (alloc_page(b, r) < 0) return false;
  return true;
}

static void release(q3t_batch *b, Req *r) {
  for (int p : r->pages) b->free_pages.push_back(p);
  r->pages.clear();
  if (r->slot >= 0) b->slots[r->slot] = nullptr;
  r->slot = -1;
  for (void *p : {(void *)r->d_trailing, (void *)r->d_pad, (void *)r->d_prompt, (void *)r->d_forced,
                  (void *)r->d_suppress})
    if (p) CK(cudaFreeAsync(p, b->st));  // stream-ordered: no device-wide synchronisation
  r->d_trailing = r->d_pad = r->d_prompt = nullptr;
  r->d_forced = r->d_suppress = nullptr;
}

static SampleParams to_params(const q3t_sampling &s) {
  SampleParams p{};
  p.do_sample = s.do_sample;
  p.temperature = s.temperature;
  p.top_k = s.top_k;
  p.top_p = s.top_p;
  const float rp = s.repetition_penalty;
  p.rep_penalty = (std::isfinite(rp) && rp > 0.f && std::fabs(rp - 1.f) > 1.1920929e-7f) ? rp : 0.f;
  p.seed = s.seed;
  return p;
}

// The per-slot state a request's sampling and teacher forcing read (from
// pinned staging, no host round trip): sampling parameters, EOS id, talker
// history length, suppress list (first token only), teacher-forced codes
// (forced[slot][0][0] is the first token).
static void upload_slot_state(q3t_batch *b, Req *r) {
  const int s = r->slot;
  SlotInit &in = b->h_init[s];  // reused only after the step that admitted it synchronised
  in.params[0] = to_params(r->ts);
  in.params[1] = to_params(r->cs);
  in.eos = r->eos;
  int64_t ff = r->forced_first;
  if (ff < 0 && !r->forced.empty()) ff = r->forced[0];
  in.forced_first = ff;
  in.forced_first32 = (int32_t)ff;
  in.zero = 0;
  const int nsup = std::min<int>((int)r->suppress.size(), b->n_suppress_cap);
  in.sup_on = nsup ? 1 : 0;
  in.nsup = nsup;
  in.forced_count = r->forced.empty() ? (ff >= 0 ? 1 : 0) : r->max_new;
  CK(cudaMemcpyAsync(b->d_params + 2 * s, in.params, sizeof in.params, cudaMemcpyHostToDevice, b->st));
  CK(cudaMemcpyAsync(b->d_eos + s, &in.eos, sizeof(int64_t), cudaMemcpyHostToDevice, b->st));
  CK(cudaMemcpyAsync(b->d_thist_len + s, &in.zero, sizeof(int), cudaMemcpyHostToDevice, b->st));
  if (nsup)
    CK(cudaMemcpyAsync(b->d_suppress + (size_t)s * b->n_suppress_cap, r->d_suppress, nsup * 8,
                       cudaMemcpyDeviceToDevice, b->st));
  CK(cudaMemcpyAsync(b->d_nsup + s, &in.nsup, sizeof(int), cudaMemcpyHostToDevice, b->st));
  CK(cudaMemcpyAsync(b->d_sup_on + s, &in.sup_on, sizeof(int), cudaMemcpyHostToDevice, b->st));
  CK(cudaMemcpyAsync(b->d_forced_count + s, &in.forced_count, sizeof(int), cudaMemcpyHostToDevice, b->st));
  if (!r->forced.empty())
    CK(cudaMemcpyAsync(b->d_forced + (size_t)s * b->maxF * b->G, r->d_forced, r->forced.size() * 8,
                       cudaMemcpyDeviceToDevice, b->st));
  else if (ff >= 0)
    CK(cudaMemcpyAsync(b->d_forced + (size_t)s * b->maxF * b->G, &in.forced_first, 8, cudaMemcpyHostToDevice, b->st));
  b->h2d += sizeof(SlotInit);
}

// TalkerGenerator::start for a session (infer/mod.rs:135-157): the whole
// prompt through the talker in 64-token chunks, then codec_head + first
// sample with the suppress list, all enqueued without a host round trip (the
// first token's EOS flag lands in first_eos[slot]).  Batched requests
// instead run their prompt chunks inside the decode frames (batch_step).
static void prefill(q3t_batch *b, Req *r) {
  q3t_model *m = b->m;
  const auto &tc = m->tc;
  const int H = b->H, V = b->V, s = r->slot;
  if (!ensure_pages(b, r, r->S)) FAIL(Q3T_OUT_OF_PAGES, "KV page pool exhausted (prompt of %d tokens)", r->S);
  flush_pages(b);
  upload_slot_state(b, r);
  const float *d_prompt = r->d_prompt;
  // chunks of kPrefillTok tokens; each token attends to [0, pos] (causal by position)
  const int nch = (r->S + kPrefillTok - 1) / kPrefillTok;
  const int ps = b->pmeta_stride();
  if (b->pmeta_used + nch > b->pmeta_blocks) {  // every block is in flight: wait for their copies
    CK(cudaStreamSynchronize(b->st));
    b->pmeta_used = 0;
  }
  const int blk0 = b->pmeta_used;
  b->pmeta_used += nch;
  int last_n = 0;
  for (int c = 0; c < nch; c++) {
    const int c0 = c * kPrefillTok, n = std::min(kPrefillTok, r->S - c0);
    int *hm = b->h_pmeta + (size_t)(blk0 + c) * ps;
    hm[0] = n;
    hm[1] = 1;
    hm[2] = s;
    for (int i = 0; i < n; i++) {
      hm[8 + i] = s;
      hm[8 + kPrefillTok + i] = c0 + i;
    }
    int *dm = b->d_pmeta + (size_t)(blk0 + c) * ps;
    CK(cudaMemcpyAsync(dm, hm, ps * sizeof(int), cudaMemcpyHostToDevice, b->st));
    CK(cudaMemcpyAsync(b->x, d_prompt + (size_t)c0 * H, (size_t)n * H * 4, cudaMemcpyDeviceToDevice, b->st));
    TokView tv{dm, dm + 8, dm + 8 + kPrefillTok, 0};
    run_stack(b, m->talker, talker_kv(b), tv, n, bucket_units(c0 + n, attn_pw(n)));
    last_n = n;
  }
  int *dm = b->d_pmeta + (size_t)(blk0 + nch - 1) * ps;
  // final norm of the last prompt token -> hidden[slot] and codec_head input
  rmsnorm(b->x, H, 1, last_n - 1, Part{nullptr, 0, 0, 0}, m->talker.final_norm, b->xn, H, H, tc.talker.rms_norm_eps,
          dm + 1, 1, b->d_hidden, dm + 2, b->st);
  GemmArgs hg = gemm_bf16_x(b, gemm_args(m->codec_head, dm + 1, 1), b->xn, H);
  hg.epi = GE_F32;
  hg.y = b->hlog;
  hg.ldy = V;
  gemm(hg, 1, b->st);
  const Part head{b->hlog, 1, 0, V};

  SampleArgs a = base_sample(b);
  a.part = head;
  a.logits = b->tlog;
  a.ldl = V;
  a.V = V;
  a.ntok = dm + 1;
  a.slot = dm + 2;
  a.use_pred_params = 0;
  a.suppress = b->d_suppress;
  a.suppress_ld = b->n_suppress_cap;
  a.n_sup = b->d_nsup;
  a.sup_on = b->d_sup_on;
  a.col = 0;
  a.frame = b->d_zero;  // the first token is frame 0, group 0 of the forced / raw records
  a.fadd = 0;
  a.hist_mode = 1;
  a.eos_flag = b->d_first_eos + s;
  sample(a, 1, b->st);
  check_launches();
  if (r->first_logits)  // the reduced logits (the sampler writes them before suppression)
    CK(cudaMemcpyAsync(r->first_logits, b->tlog, (size_t)V * 4, cudaMemcpyDeviceToHost, b->st));
  r->cache_len = r->S;
  r->prefill_pos = r->S;
  r->step_idx = 0;
  r->admitted_now = true;
  r->decoding = true;
}

static void admit(q3t_batch *b, int *admitted) {
  while (!b->queue.empty()) {
    int s = -1;
    for (int i = 0; i < b->A; i++)
      if (!b->slots[i]) {
        s = i;
        break;
      }
    if (s < 0) break;
    Req *r = b->queue.front();
    const int need = (r->S + kPage - 1) / kPage + 1;
    if (need > b->n_pages || r->S + 1 > kMaxSeq) {  // can never fit: fail it, keep serving the queue
      b->queue.pop_front();
      r->state = 3;
      r->fail_status = Q3T_OUT_OF_PAGES;
      r->error = "prompt of " + std::to_string(r->S) + " tokens needs " + std::to_string(need) +
                 " KV pages; the pool holds " + std::to_string(b->n_pages);
      continue;
    }
    if ((int)b->free_pages.size() < need) break;  // wait for pages
    b->queue.pop_front();
    r->slot = s;
    b->slots[s] = r;
    r->state = 1;
    r->admit_order = b->admit_counter++;
    try {
      if (b->session_mode) {
        prefill(b, r);
      } else {  // the prompt runs in chunks inside the next decode frames; its pages are taken now
        if (!ensure_pages(b, r, r->S)) FAIL(Q3T_OUT_OF_PAGES, "KV page pool exhausted (prompt of %d tokens)", r->S);
        upload_slot_state(b, r);
        r->prefill_pos = 0;
        r->cache_len = 0;
        r->step_idx = 0;
        r->decoding = false;
      }
    } catch (const Status &st) {
      r->state = 3;
      r->fail_status = st.code;
      r->error = g_err;
      release(b, r);
      continue;
    }
    if (admitted) (*admitted)++;
  }
}

static void retire(q3t_batch *b, Req *r, int64_t *samples) {
  const int T = r->step_idx, G = b->G;
  std::vector<int64_t> tg((size_t)T * G);
  std::vector<int32_t> rg((size_t)T * G);
  if (T > 0) {
    CK(cudaMemcpyAsync(tg.data(), b->d_hist_codes + (size_t)r->slot * b->maxF * G, tg.size() * 8,
                       cudaMemcpyDeviceToHost, b->st));
    CK(cudaMemcpyAsync(rg.data(), b->d_raw + (size_t)r->slot * b->maxF * G, rg.size() * 4,
                       cudaMemcpyDeviceToHost, b->st));
    CK(cudaStreamSynchronize(b->st));
    b->d2h += (int64_t)T * G * 12;
  }
  r->codes.assign((size_t)G * T, 0);
  r->sampled.assign((size_t)G * T, 0);
  for (int t = 0; t < T; t++)
    for (int q = 0; q < G; q++) {
      r->codes[(size_t)q * T + t] = tg[(size_t)t * G + q];
      r->sampled[(size_t)q * T + t] = rg[(size_t)t * G + q];
    }
  if (b->desc.codec_mode == 1 && b->m->has_codec && T > 0) {
    int64_t n = 0;
    codec_out_len(b->m->codec, T, &n);
    if (b->desc.keep_output) r->wave.resize(n);
    codec_decode_host_codes(b->m, r->codes.data(), 1, T, b->desc.keep_output ? r->wave.data() : nullptr,
                            nullptr, b->st);
    r->samples = n;
    if (samples) *samples += n;
    if (b->desc.keep_output) b->d2h += n * 4;
  }
  if (!b->desc.keep_output && !b->session_mode) r->codes.clear();
  r->state = 2;
  release(b, r);
}

// One scheduler step.  Decode requests (first token known) get one frame:
// the code-predictor loop, then the talker pass, which also carries prompt
// tokens of admitted requests up to kTalkerTok tokens in all (chunked
// prefill, served in admission order); a prompt that completes in this step
// has its last token normed, headed and sampled with the decode tokens, and
// decodes from the next step on.  One synchronisation per step (the flags
// read back).
static void batch_step(q3t_batch *b, q3t_step_stats *stats) {
  q3t_step_stats S{};
  b->pmeta_used = 0;  // the previous step (or call) synchronised the stream
  CK(cudaEventRecord(b->ev0, b->st));
  admit(b, &S.admitted);
  std::vector<Req *> act, pre;
  for (int i = 0; i < b->A; i++) {
    Req *r = b->slots[i];
    if (!r) continue;
    if (r->finished) continue;
    if (!r->decoding) {
      pre.push_back(r);
      continue;
    }
    if (r->eos_seen) {  // infer/mod.rs:197-204
      if (r->step_idx == 0) {
        r->state = 3;
        r->error = "talker emitted EOS before any audio codec token";
        release(b, r);
      } else {
        r->finished = true;
        retire(b, r, &S.samples);
        S.retired++;
      }
      continue;
    }
    act.push_back(r);
  }
  b->frame_timed = false;
  auto report = [&] {
    CK(cudaEventRecord(b->ev1, b->st));
    CK(cudaEventSynchronize(b->ev1));
    CK(cudaEventElapsedTime(&b->last_ms, b->ev0, b->ev1));
    S.device_ms = b->last_ms;
    if (b->frame_timed) {
      CK(cudaEventElapsedTime(&S.predictor_ms, b->evf[0], b->evf[1]));
      CK(cudaEventElapsedTime(&S.talker_ms, b->evf[1], b->evf[2]));
    }
    S.h2d_bytes = b->h2d;
    S.d2h_bytes = b->d2h;
    b->h2d = b->d2h = 0;
    if (stats) *stats = S;
  };
  auto fail_pages = [&](Req *r, int len) {
    r->state = 3;
    r->fail_status = Q3T_OUT_OF_PAGES;
    r->error = "request " + std::to_string(r->id) + ": KV capacity exhausted at " + std::to_string(len) + " tokens";
    release(b, r);
  };
  // KV pages for this frame's token; a request that cannot get one fails
  // alone (the reference slides its 4096-entry window here, kv.rs:109-132;
  // this build stops the request with an explicit error) and the others run
  {
    size_t k = 0;
    for (Req *r : act) {
      if (r->cache_len + 1 > kMaxSeq || r->step_idx >= b->maxF || !ensure_pages(b, r, r->cache_len + 1)) {
        fail_pages(r, r->cache_len);
        continue;
      }
      act[k++] = r;
    }
    act.resize(k);
  }
  // this step's prompt chunks, in admission order, filling the talker pass up to kTalkerTok tokens
  struct Chunk {
    Req *r;
    int pos0, n;
  };
  std::vector<Chunk> chunks;
  std::sort(pre.begin(), pre.end(), [](const Req *x, const Req *y) { return x->admit_order < y->admit_order; });
  {
    int budget = kTalkerTok - (int)act.size();
    for (Req *r : pre) {
      if (budget == 0) break;
      const int n = std::min(budget, r->S - r->prefill_pos);
      if (n <= 0) continue;
      if (!ensure_pages(b, r, r->prefill_pos + n)) {
        fail_pages(r, r->prefill_pos);
        continue;
      }
      chunks.push_back({r, r->prefill_pos, n});
      budget -= n;
    }
  }
  const int B = (int)act.size();
  int P = 0;
  for (const Chunk &c : chunks) P += c.n;
  S.active = B;
  S.prefill_tokens = P;
  if (B == 0 && P == 0) {
    if (b->desc.codec_mode == 2 && b->m->has_codec) codec_stream_join(b, &S.samples);
    report();
    return;
  }
  int *hm = b->h_meta;
  for (int i = 0; i < B; i++) {
    Req *r = act[i];
    hm[b->off_slot() + i] = r->slot;
    hm[b->off_tpos() + i] = r->cache_len;
    hm[b->off_frame() + i] = r->step_idx;
    hm[b->off_zero() + i] = 0;
    hm[b->off_p0seq() + 2 * i] = hm[b->off_p0seq() + 2 * i + 1] = r->slot;
    hm[b->off_p0pos() + 2 * i] = 0;
    hm[b->off_p0pos() + 2 * i + 1] = 1;
    b->h_extra[i] = r->step_idx < r->trailing_len ? r->d_trailing + (size_t)r->step_idx * b->H : r->d_pad;
    hm[b->off_tseq() + i] = r->slot;
    hm[b->off_ttpos() + i] = r->cache_len;
    hm[b->off_hrow() + i] = i;
    hm[b->off_hslot() + i] = r->slot;
    hm[b->off_hframe() + i] = r->step_idx;
    S.kv_tokens += r->cache_len + 1;
  }
  // prompt-chunk tokens follow the decode tokens in the talker pass; a chunk
  // that completes its prompt adds its last token to the head
  std::vector<PromptCopy> copies;
  std::vector<Req *> firsts;
  int t = B, h = B;
  for (const Chunk &c : chunks) {
    for (int j = 0; j < c.n; j++) {
      hm[b->off_tseq() + t + j] = c.r->slot;
      hm[b->off_ttpos() + t + j] = c.pos0 + j;
      S.kv_tokens += c.pos0 + j + 1;
    }
    copies.push_back({c.r->d_prompt + (size_t)c.pos0 * b->H, c.n, t});
    if (c.pos0 + c.n == c.r->S) {
      hm[b->off_hrow() + h] = t + c.n - 1;
      hm[b->off_hslot() + h] = c.r->slot;
      hm[b->off_hframe() + h] = -1;  // the first token: record index 0 of the forced / raw codes
      firsts.push_back(c.r);
      h++;
    }
    t += c.n;
  }
  const int F = (int)firsts.size();
  flush_pages(b);
  hm[M_NTOK_B] = B;
  hm[M_NTOK_2B] = 2 * B;
  hm[M_ONE] = 1;
  hm[M_SEED] = b->step_counter++;
  hm[M_NTOK_T] = B + P;
  hm[M_NTOK_H] = B + F;
  CK(cudaMemcpyAsync(b->d_meta, hm, b->meta_n * sizeof(int), cudaMemcpyHostToDevice, b->st));
  if (B) CK(cudaMemcpyAsync(b->d_extra, b->h_extra, B * sizeof(float *), cudaMemcpyHostToDevice, b->st));
  // the attention's unit bound only sizes its (persistent) grid, so the frame
  // graphs use the largest and are captured once per token bucket
  const int mt = bucket_tok(B), mtT = bucket_tok(B + P), ms = kAttnMaxUnits;
  b->h2d += b->meta_n * sizeof(int) + B * sizeof(float *);
  b->last_ids.resize(B);
  for (int i = 0; i < B; i++) b->last_ids[i] = act[i]->id;
  enqueue_frame(b, B, mt, mtT, ms, P > 0, copies);
  // the previous step's codec windows decode on their own stream under this frame
  if (b->desc.codec_mode == 2 && b->m->has_codec) codec_stream_launch(b);
  CK(cudaMemcpyAsync(b->h_eosflag, b->d_eosflag, (B + F) * sizeof(int), cudaMemcpyDeviceToHost, b->st));
  CK(cudaMemcpyAsync(b->h_err, b->d_err, sizeof(int), cudaMemcpyDeviceToHost, b->st));
  CK(cudaStreamSynchronize(b->st));
  b->d2h += (B + F) * sizeof(int) + sizeof(int);
  if (*b->h_err) {
    const int e = *b->h_err;
    *b->h_err = 0;
    CK(cudaMemsetAsync(b->d_err, 0, sizeof(int), b->st));
    FAIL(Q3T_DEVICE_TIMEOUT, "decode frame: a bounded device wait gave up (code %d)", e);
  }
  for (const Chunk &c : chunks) {
    c.r->prefill_pos += c.n;
    c.r->cache_len = c.r->prefill_pos;
  }
  S.first_tokens = F;
  bool copied = false;
  for (int f = 0; f < F; f++)  // the reduced logits (the sampler writes them before suppression)
    if (firsts[f]->first_logits) {
      CK(cudaMemcpyAsync(firsts[f]->first_logits, b->tlog + (size_t)(B + f) * b->V, (size_t)b->V * 4,
                         cudaMemcpyDeviceToHost, b->st));
      copied = true;
    }
  if (copied) CK(cudaStreamSynchronize(b->st));
  for (int f = 0; f < F; f++) {  // TalkerGenerator::start done: the first token is known
    Req *r = firsts[f];
    if (r->eos >= 0 && b->h_eosflag[B + f]) {  // infer/mod.rs:197-202: EOS before any audio codec token
      r->eos_seen = true;
      r->state = 3;
      r->error = "talker emitted EOS before any audio codec token";
      release(b, r);
      continue;
    }
    r->decoding = true;
    r->cache_len = r->S;
    r->step_idx = 0;
  }
  for (int i = 0; i < B; i++) {
    Req *r = act[i];
    r->step_idx++;
    S.frames++;
    if (r->step_idx >= r->max_new) {
      r->finished = true;
    } else {
      r->cache_len++;
      if (r->forced.empty() && b->h_eosflag[i]) {
        r->eos_seen = true;
        r->finished = true;
      }
    }
  }
  if (b->desc.codec_mode == 2 && b->m->has_codec) codec_stream_step(b->m, b, act, &S.samples);
  for (Req *r : act)
    if (r->finished) {
      retire(b, r, &S.samples);
      S.retired++;
    }
  report();
}

static Req *new_request(q3t_batch *b, const q3t_session_desc *d, const int64_t *forced) {
  const auto &tc = b->m->tc;
  const int H = tc.talker.hidden_size;
  if (d->max_new_tokens <= 0) FAIL(Q3T_INVALID_INPUT, "talker max_new_tokens must be greater than zero");
  if (!d->inputs_embeds || d->prompt_len <= 0) FAIL(Q3T_INVALID_INPUT, "prompt must be non-empty");
  if (!d->trailing_text || d->trailing_len <= 0 || !d->pad_embed)
    FAIL(Q3T_INVALID_INPUT,
         "generation side input length mismatch: trailing length must be > 0 and pad length must be 1");
  if (d->prompt_len + 1 > kMaxSeq) FAIL(Q3T_INVALID_INPUT, "prompt of %d tokens exceeds %d", d->prompt_len, kMaxSeq);
  if (d->max_new_tokens > kMaxSeq) FAIL(Q3T_INVALID_INPUT, "max_new_tokens %d exceeds %d", d->max_new_tokens, kMaxSeq);
  if (d->num_suppress > b->n_suppress_cap) FAIL(Q3T_INVALID_INPUT, "too many suppress ids");
  auto r = std::make_unique<Req>();
  r->id = b->next_id++;
  r->S = d->prompt_len;
  r->prompt.assign(d->inputs_embeds, d->inputs_embeds + (size_t)d->prompt_len * H);
  r->trailing_len = d->trailing_len;
  r->trailing.assign(d->trailing_text, d->trailing_text + (size_t)d->trailing_len * H);
  r->pad.assign(d->pad_embed, d->pad_embed + H);
  r->ts = d->talker_sampling;
  r->cs = d->predictor_sampling;
  r->max_new = d->max_new_tokens;
  r->eos = d->eos_token_id;
  if (d->suppress_ids && d->num_suppress > 0) r->suppress.assign(d->suppress_ids, d->suppress_ids + d->num_suppress);
  r->forced_first = d->forced_first_token;
  r->first_logits = d->first_logits;
  const int G = b->G;
  if (forced) {
    r->forced.assign(forced, forced + (size_t)d->max_new_tokens * G);
    for (int f = 0; f < d->max_new_tokens; f++)
      for (int q = 0; q < G; q++) {
        const int64_t c = r->forced[(size_t)f * G + q];
        const int lim = q == 0 ? tc.talker.vocab_size : tc.predictor.vocab_size;
        if (c < 0 || c >= lim) FAIL(Q3T_INVALID_INPUT, "forced code %lld out of range at frame %d group %d", (long long)c, f, q);
      }
  }
  if (r->forced_first >= tc.talker.vocab_size) FAIL(Q3T_INVALID_INPUT, "forced first token out of range");
  for (auto id : r->suppress)
    if (id < 0) FAIL(Q3T_INVALID_INPUT, "negative suppress id");
  // inputs go to device memory at submit time, so admission finds them
  // resident; the stream-ordered pool keeps its memory, so neither this
  // allocation nor the free at retirement synchronises the device, and a
  // copy from pageable memory returns once the data is staged
  auto up = [&](void **d, const void *h, size_t bytes) {
    CK(cudaMallocFromPoolAsync(d, bytes ? bytes : 8, b->pool, b->st));
    if (bytes) CK(cudaMemcpyAsync(*d, h, bytes, cudaMemcpyHostToDevice, b->st));
    b->h2d += (int64_t)bytes;
  };
  up((void **)&r->d_prompt, r->prompt.data(), r->prompt.size() * 4);
  up((void **)&r->d_trailing, r->trailing.data(), r->trailing.size() * 4);
  up((void **)&r->d_pad, r->pad.data(), r->pad.size() * 4);
  if (!r->forced.empty()) up((void **)&r->d_forced, r->forced.data(), r->forced.size() * 8);
  if (!r->suppress.empty())
    up((void **)&r->d_suppress, r->suppress.data(),
       std::min<size_t>(r->suppress.size(), (size_t)b->n_suppress_cap) * 8);
  std::vector<float>().swap(r->prompt);  // the device copy is the one that is used
  Req *raw = r.get();
  b->reqs[raw->id] = std::move(r);
  return raw;
}

}  // namespace q3t

// ----------------------------------------------------------------------------
// C ABI: batches
// ----------------------------------------------------------------------------
extern "C" q3t_status q3t_batch_create(q3t_model *m, const q3t_batch_desc *d, q3t_batch **out) {
  if (!m || !d || !out) {
    set_error("q3t_batch_create: null argument");
    return Q3T_INVALID_INPUT;
  }
  *out = nullptr;
  if (!m->has_talker) {
    set_error("model has no talker");
    return Q3T_INVALID_INPUT;
  }
  if (d->max_active <= 0 || d->max_active > m->max_active) {
    set_error("max_active %d outside 1..%d", d->max_active, m->max_active);
    return Q3T_INVALID_INPUT;
  }
  if (d->codec_mode < 0 || d->codec_mode > 2 || (d->codec_mode && !m->has_codec)) {
    set_error("codec_mode %d unsupported by this model", d->codec_mode);
    return Q3T_INVALID_INPUT;
  }
  auto *b = new q3t_batch();
  q3t_status rc = guard([&] {
    CK(cudaSetDevice(m->device));
    batch_init(b, m, *d);
    if (d->codec_mode == 2) codec_stream_init(m, b);
  });
  if (rc != Q3T_OK) {
    if (d->codec_mode == 2) codec_stream_free(b);
    batch_destroy(b);
    delete b;
    return rc;
  }
  *out = b;
  return Q3T_OK;
}

extern "C" q3t_status q3t_batch_submit(q3t_batch *b, const q3t_session_desc *req, const int64_t *forced,
                                       int64_t *id) {
  if (!b || !req) {
    set_error("q3t_batch_submit: null argument");
    return Q3T_INVALID_INPUT;
  }
  return guard([&] {
    Req *r = new_request(b, req, forced);
    b->queue.push_back(r);
    if (id) *id = r->id;
  });
}

extern "C" q3t_status q3t_batch_step(q3t_batch *b, q3t_step_stats *stats) {
  if (!b) {
    set_error("q3t_batch_step: null batch");
    return Q3T_INVALID_INPUT;
  }
  return guard([&] {
    CK(cudaSetDevice(b->m->device));
    batch_step(b, stats);
  });
}

extern "C" q3t_status q3t_batch_poll(q3t_batch *b, int64_t id, int *state, int64_t *frames, int64_t *samples) {
  if (!b) return Q3T_INVALID_INPUT;
  auto it = b->reqs.find(id);
  if (it == b->reqs.end()) {
    set_error("unknown request %lld", (long long)id);
    return Q3T_INVALID_INPUT;
  }
  Req *r = it->second.get();
  if (state) *state = r->state;
  if (frames) *frames = r->step_idx;
  if (samples) *samples = r->samples;
  if (r->state == 3) set_error("%s", r->error.c_str());
  return Q3T_OK;
}

extern "C" q3t_status q3t_batch_take(q3t_batch *b, int64_t id, int64_t *codes, int32_t *sampled,
                                     int max_frames, float *wave, int64_t max_samples) {
  if (!b) return Q3T_INVALID_INPUT;
  auto it = b->reqs.find(id);
  if (it == b->reqs.end()) {
    set_error("unknown request %lld", (long long)id);
    return Q3T_INVALID_INPUT;
  }
  Req *r = it->second.get();
  if (r->state != 2) {
    set_error("request %lld is not finished", (long long)id);
    return Q3T_INVALID_INPUT;
  }
  const int T = r->step_idx, G = b->G;
  if (codes) {
    if (max_frames < T || (int64_t)r->codes.size() != (int64_t)G * T) {
      set_error("codes unavailable or buffer too small (%d frames)", T);
      return Q3T_INVALID_INPUT;
    }
    memcpy(codes, r->codes.data(), r->codes.size() * 8);
  }
  if (sampled) {
    if (max_frames < T || (int64_t)r->sampled.size() != (int64_t)G * T) {
      set_error("sampled codes unavailable or buffer too small (%d frames)", T);
      return Q3T_INVALID_INPUT;
    }
    memcpy(sampled, r->sampled.data(), r->sampled.size() * 4);
  }
  if (wave) {
    if ((int64_t)r->wave.size() > max_samples) {
      set_error("wave buffer too small (%lld samples)", (long long)r->wave.size());
      return Q3T_INVALID_INPUT;
    }
    memcpy(wave, r->wave.data(), r->wave.size() * 4);
  }
  b->reqs.erase(it);
  return Q3T_OK;
}

extern "C" q3t_status q3t_batch_logits(q3t_batch *b, int64_t id, float *talker_logits, float *predictor_logits) {
  if (!b) return Q3T_INVALID_INPUT;
  size_t i = 0;
  while (i < b->last_ids.size() && b->last_ids[i] != id) i++;
  if (i == b->last_ids.size()) {
    set_error("request %lld was not in the last decode frame", (long long)id);
    return Q3T_INVALID_INPUT;
  }
  return guard([&] {
    CK(cudaSetDevice(b->m->device));
    if (talker_logits)
      CK(cudaMemcpyAsync(talker_logits, b->tlog + i * b->V, (size_t)b->V * 4, cudaMemcpyDeviceToHost, b->st));
    if (predictor_logits)
      for (int j = 0; j < b->G - 1; j++)
        CK(cudaMemcpyAsync(predictor_logits + (size_t)j * b->PV, b->plog + ((size_t)j * b->A + i) * b->PV,
                           (size_t)b->PV * 4, cudaMemcpyDeviceToHost, b->st));
    CK(cudaStreamSynchronize(b->st));
  });
}

extern "C" q3t_status q3t_batch_pending(q3t_batch *b, int *queued, int *active) {
  if (!b) return Q3T_INVALID_INPUT;
  int a = 0;
  for (auto *r : b->slots) a += r != nullptr;
  if (queued) *queued = (int)b->queue.size();
  if (active) *active = a;
  return Q3T_OK;
}

extern "C" q3t_status q3t_batch_stream(q3t_batch *b, void **stream) {
  if (!b || !stream) return Q3T_INVALID_INPUT;
  *stream = (void *)b->st;
  return Q3T_OK;
}

extern "C" void q3t_batch_free(q3t_batch *b) {
  if (!b) return;
  cudaSetDevice(b->m->device);
  if (b->desc.codec_mode == 2) codec_stream_free(b);
  batch_destroy(b);
  delete b;
}

// ----------------------------------------------------------------------------
// C ABI: sessions (batch of one, reference TalkerGenerator semantics)
// ----------------------------------------------------------------------------
struct q3t_session {
  q3t_batch *b = nullptr;
  q3t::Req *r = nullptr;
};

extern "C" q3t_status q3t_session_start(q3t_model *m, const q3t_session_desc *d, q3t_session **out) {
  if (!m || !d || !out) {
    set_error("q3t_session_start: null argument");
    return Q3T_INVALID_INPUT;
  }
  *out = nullptr;
  q3t_batch_desc bd{};
  bd.max_active = 1;
  bd.codec_mode = 0;
  bd.keep_output = 1;
  q3t_batch *b = nullptr;
  q3t_status rc = q3t_batch_create(m, &bd, &b);
  if (rc != Q3T_OK) return rc;
  b->session_mode = true;
  auto *s = new q3t_session();
  s->b = b;
  rc = guard([&] {
    s->r = new_request(b, d, nullptr);
    b->queue.push_back(s->r);
    admit(b, nullptr);
    if (s->r->state == 3) FAIL(s->r->fail_status, "%s", s->r->error.c_str());
    if (s->r->state != 1) FAIL(Q3T_OUT_OF_PAGES, "prompt of %d tokens does not fit the KV pool", s->r->S);
    // TalkerGenerator::start returns with the first token known: read its EOS flag now
    CK(cudaMemcpyAsync(b->h_first_eos, b->d_first_eos, b->A * sizeof(int), cudaMemcpyDeviceToHost, b->st));
    CK(cudaStreamSynchronize(b->st));
    s->r->admitted_now = false;
    s->r->eos_seen = s->r->eos >= 0 && b->h_first_eos[s->r->slot];
  });
  if (rc != Q3T_OK) {
    q3t_batch_free(b);
    delete s;
    return rc;
  }
  *out = s;
  return Q3T_OK;
}

static q3t_status session_step(q3t_session *s, const int64_t *forced, float *tl, float *pl, float *hid,
                               int *state) {
  if (!s) {
    set_error("null session");
    return Q3T_INVALID_INPUT;
  }
  q3t_batch *b = s->b;
  Req *r = s->r;
  return guard([&] {
    CK(cudaSetDevice(b->m->device));
    if (state) *state = 0;
    if (r->state == 2 || r->finished) return;  // Ok(None)
    if (r->state == 3) FAIL(r->fail_status, "%s", r->error.c_str());
    if (r->eos_seen) {
      if (r->step_idx == 0) {
        r->state = 3;
        r->error = "talker emitted EOS before any audio codec token";
        FAIL(Q3T_INVALID_INPUT, "talker emitted EOS before any audio codec token");
      }
      r->finished = true;
      r->state = 2;
      return;
    }
    const int G = b->G, sl = r->slot, f = r->step_idx;
    if (forced) {
      for (int q = 0; q < G; q++) {
        const int lim = q == 0 ? b->V : b->PV;
        if (forced[q] < 0 || forced[q] >= lim) FAIL(Q3T_INVALID_INPUT, "forced code out of range");
      }
      CK(cudaMemcpyAsync(b->d_forced + ((size_t)sl * b->maxF + f) * G, forced, G * 8, cudaMemcpyHostToDevice, b->st));
      const int fc = f + 1;
      CK(cudaMemcpyAsync(b->d_forced_count + sl, &fc, 4, cudaMemcpyHostToDevice, b->st));
      const int32_t c0 = (int32_t)forced[0];
      CK(cudaMemcpyAsync(b->d_codes + (size_t)sl * G, forced, 8, cudaMemcpyHostToDevice, b->st));
      CK(cudaMemcpyAsync(b->d_thist + (size_t)sl * b->hist_cap + f, &c0, 4, cudaMemcpyHostToDevice, b->st));
    }
    batch_step(b, nullptr);
    if (r->state == 3) FAIL(r->fail_status, "%s", r->error.c_str());
    if (tl) CK(cudaMemcpyAsync(tl, b->tlog, (size_t)b->V * 4, cudaMemcpyDeviceToHost, b->st));
    if (pl)
      for (int j = 0; j < G - 1; j++)
        CK(cudaMemcpyAsync(pl + (size_t)j * b->PV, b->plog + (size_t)j * b->A * b->PV, (size_t)b->PV * 4,
                           cudaMemcpyDeviceToHost, b->st));
    if (hid)
      CK(cudaMemcpyAsync(hid, b->d_hidden + (size_t)sl * b->H, (size_t)b->H * 4, cudaMemcpyDeviceToHost, b->st));
    CK(cudaStreamSynchronize(b->st));
    if (state) *state = r->finished ? 2 : 1;
  });
}

extern "C" q3t_status q3t_session_step(q3t_session *s, int *state) {
  return session_step(s, nullptr, nullptr, nullptr, nullptr, state);
}

extern "C" q3t_status q3t_session_step_forced(q3t_session *s, const int64_t *codes, float *tl, float *pl,
                                              float *hid, int *state) {
  if (!codes) {
    set_error("q3t_session_step_forced: null codes");
    return Q3T_INVALID_INPUT;
  }
  return session_step(s, codes, tl, pl, hid, state);
}

extern "C" q3t_status q3t_session_codes(q3t_session *s, int64_t *out, int *num_frames) {
  if (!s) return Q3T_INVALID_INPUT;
  return guard([&] {
    q3t_batch *b = s->b;
    Req *r = s->r;
    const int T = r->step_idx, G = b->G;
    if (num_frames) *num_frames = T;
    if (T == 0) FAIL(Q3T_INVALID_INPUT, "no codec tokens were generated");
    if (!out) return;
    if ((int)r->codes.size() == G * T) {
      memcpy(out, r->codes.data(), r->codes.size() * 8);
      return;
    }
    std::vector<int64_t> tg((size_t)T * G);
    CK(cudaMemcpyAsync(tg.data(), b->d_hist_codes + (size_t)r->slot * b->maxF * G, tg.size() * 8,
                       cudaMemcpyDeviceToHost, b->st));
    CK(cudaStreamSynchronize(b->st));
    for (int t = 0; t < T; t++)
      for (int q = 0; q < G; q++) out[(size_t)q * T + t] = tg[(size_t)t * G + q];
  });
}

extern "C" q3t_status q3t_session_finish(q3t_session *s, float *wave, int16_t *pcm, int64_t capacity,
                                         int64_t *num_samples) {
  if (!s) return Q3T_INVALID_INPUT;
  return guard([&] {
    q3t_batch *b = s->b;
    if (!b->m->has_codec) FAIL(Q3T_INVALID_INPUT, "model has no codec");
    int T = 0;
    q3t_status rc = q3t_session_codes(s, nullptr, &T);
    if (rc != Q3T_OK) throw Status{rc, ""};
    std::vector<int64_t> codes((size_t)b->G * T);
    rc = q3t_session_codes(s, codes.data(), &T);
    if (rc != Q3T_OK) throw Status{rc, ""};
    int64_t n = 0;
    codec_out_len(b->m->codec, T, &n);
    if (num_samples) *num_samples = n;
    if ((wave || pcm) && capacity < n) FAIL(Q3T_INVALID_INPUT, "output buffer holds %lld samples, need %lld",
                                            (long long)capacity, (long long)n);
    codec_decode_host_codes(b->m, codes.data(), 1, T, wave, pcm, b->st);
  });
}

extern "C" q3t_status q3t_session_decode_embeds(q3t_session *s, const float *embeds, float *logits,
                                                float *hidden) {
  if (!s || !embeds) {
    set_error("q3t_session_decode_embeds: null argument");
    return Q3T_INVALID_INPUT;
  }
  return guard([&] {
    q3t_batch *b = s->b;
    Req *r = s->r;
    q3t_model *m = b->m;
    CK(cudaSetDevice(m->device));
    if (r->slot < 0) FAIL(Q3T_INVALID_INPUT, "session is finished");
    if (r->cache_len + 1 > kMaxSeq || !ensure_pages(b, r, r->cache_len + 1))
      FAIL(Q3T_OUT_OF_PAGES, "KV capacity exhausted at %d tokens", r->cache_len);
    flush_pages(b);
    int *hm = b->h_meta;
    hm[b->off_slot()] = r->slot;
    hm[b->off_tpos()] = r->cache_len;
    hm[M_NTOK_B] = 1;
    hm[M_NTOK_2B] = 2;
    hm[M_ONE] = 1;
    CK(cudaMemcpyAsync(b->d_meta, hm, b->meta_n * sizeof(int), cudaMemcpyHostToDevice, b->st));
    CK(cudaMemcpyAsync(b->x, embeds, (size_t)b->H * 4, cudaMemcpyHostToDevice, b->st));
    const int ms = bucket_units(r->cache_len + 1, attn_pw(1));
    CK(cudaEventRecord(b->ev0, b->st));
    if (b->use_mk) {
      const auto prog = mk_program(b, MKP_TALKER_DECODE);
      MkArgs ma{prog.first, prog.second,
                TokView{b->d_meta + M_NTOK_B, b->d_meta + b->off_slot(), b->d_meta + b->off_tpos(), 0}, b->mk_ctr,
                b->d_err, nullptr, b->wait_polls, b->stall_waits ? (const int *)(b->mk_ctr + 2) : nullptr};
      const char *tr = getenv("Q3T_MK_TRACE");  // profiling: per-stage device timestamps to this file
      if (tr && tr[0]) {
        const size_t nt = (size_t)b->mk_grid * prog.second * 8;
        CK(cudaMallocAsync((void **)&ma.trace, nt * 8, b->st));
        CK(cudaMemsetAsync(ma.trace, 0, nt * 8, b->st));
        mk_launch(ma, b->mk_grid, b->st);
        check_launches();
        std::vector<unsigned long long> h(nt);
        CK(cudaMemcpyAsync(h.data(), ma.trace, nt * 8, cudaMemcpyDeviceToHost, b->st));
        CK(cudaStreamSynchronize(b->st));
        CK(cudaFreeAsync(ma.trace, b->st));
        if (FILE *f = fopen(tr, "wb")) {
          const int hdr[2] = {b->mk_grid, prog.second};
          fwrite(hdr, sizeof hdr, 1, f);
          fwrite(h.data(), 8, nt, f);
          fclose(f);
        }
      } else {
        run_graph(b, std::make_tuple(3, MKP_TALKER_DECODE, 0), [&] { mk_launch(ma, b->mk_grid, b->st); });
      }
    } else
    run_graph(b, std::make_tuple(1, 1, ms), [&] {
      const int *ntok = b->d_meta + M_NTOK_B, *slot = b->d_meta + b->off_slot();
      TokView tvt{ntok, slot, b->d_meta + b->off_tpos(), 0};
      run_stack(b, m->talker, talker_kv(b), tvt, 1, ms);
      rmsnorm(b->x, b->H, 1, 0, Part{}, m->talker.final_norm, b->xn, b->H, b->H, m->tc.talker.rms_norm_eps, ntok, 1,
              b->d_hidden, slot, b->st);
      GemmArgs hg = gemm_bf16_x(b, gemm_args(m->codec_head, ntok, 1), b->xn, b->H);
      hg.epi = GE_F32;
      hg.y = b->tlog;
      hg.ldy = b->V;
      gemm(hg, 1, b->st);
    });
    CK(cudaEventRecord(b->ev1, b->st));
    if (logits) CK(cudaMemcpyAsync(logits, b->tlog, (size_t)b->V * 4, cudaMemcpyDeviceToHost, b->st));
    if (hidden)
      CK(cudaMemcpyAsync(hidden, b->d_hidden + (size_t)r->slot * b->H, (size_t)b->H * 4, cudaMemcpyDeviceToHost,
                         b->st));
    CK(cudaStreamSynchronize(b->st));
    CK(cudaEventElapsedTime(&b->last_ms, b->ev0, b->ev1));
    check_device_error(b, "talker decode step");
    r->cache_len++;
  });
}

extern "C" q3t_status q3t_session_load_kv(q3t_session *s, const uint16_t *k, const uint16_t *v, int len,
                                          const float *hidden) {
  if (!s || (len > 0 && (!k || !v)) || len < 0) {
    set_error("q3t_session_load_kv: bad argument");
    return Q3T_INVALID_INPUT;
  }
  return guard([&] {
    q3t_batch *b = s->b;
    Req *r = s->r;
    q3t_model *m = b->m;
    CK(cudaSetDevice(m->device));
    if (r->slot < 0) FAIL(Q3T_INVALID_INPUT, "session is finished");
    if (len + 1 > kMaxSeq || !ensure_pages(b, r, len + 1)) FAIL(Q3T_OUT_OF_PAGES, "KV capacity exhausted");
    flush_pages(b);
    const auto &c = m->tc.talker;
    const size_t n = (size_t)c.num_hidden_layers * c.num_key_value_heads * len * 128;
    if (len > 0) {
      uint16_t *dk, *dv;
      CK(cudaMalloc(&dk, n * 2));
      CK(cudaMalloc(&dv, n * 2));
      CK(cudaMemcpyAsync(dk, k, n * 2, cudaMemcpyHostToDevice, b->st));
      CK(cudaMemcpyAsync(dv, v, n * 2, cudaMemcpyHostToDevice, b->st));
      kv_import(dk, dv, c.num_hidden_layers, len, talker_kv(b), r->slot, b->st);
      CK(cudaStreamSynchronize(b->st));
      CK(cudaFree(dk));
      CK(cudaFree(dv));
    }
    r->cache_len = len;
    if (hidden)
      CK(cudaMemcpyAsync(b->d_hidden + (size_t)r->slot * b->H, hidden, (size_t)b->H * 4, cudaMemcpyHostToDevice,
                         b->st));
    CK(cudaStreamSynchronize(b->st));
  });
}

extern "C" q3t_status q3t_session_last_ms(q3t_session *s, float *ms) {
  if (!s || !ms) return Q3T_INVALID_INPUT;
  *ms = s->b->last_ms;
  return Q3T_OK;
}

extern "C" void q3t_session_free(q3t_session *s) {
  if (!s) return;
  q3t_batch_free(s->b);
  delete s;
}

// ----------------------------------------------------------------------------
// Text projection of prompt token ids (project_text_ids,
// execution/compiler/session_seed.rs:668-679; Qwen3TtsTalkerResizeMlp,
// talker/network/mlp.rs:36-40): embedding gather, linear_fc1 + bias, SiLU
// (rounded to bf16), linear_fc2 + bias (rounded to bf16), 64 ids per pass on
// the tensor-core GEMM.
// ----------------------------------------------------------------------------
// project_text_ids (session_seed.rs:668-679) of n validated ids in chunks of
// 64 through the text-projection workspace (tp_mu held); rows go to `out`
// with copy kind `kind` (device -> host or device -> device) on m->tp_st.
static void text_project_rows(q3t_model *m, const int64_t *ids, int n, float *out, cudaMemcpyKind kind) {
  const int Ht = m->text_hidden, H = m->tc.talker.hidden_size, TB = 64;
  if (!m->tp_st) {
    CK(cudaStreamCreateWithFlags(&m->tp_st, cudaStreamNonBlocking));
    m->tp_x = m->arena.alloc<uint16_t>((size_t)TB * Ht);
    m->tp_h = m->arena.alloc<uint16_t>((size_t)TB * Ht);
    m->tp_out = m->arena.alloc<float>((size_t)TB * H);
    m->tp_ids = m->arena.alloc<int>(TB);
    m->tp_ntok = m->arena.alloc<int>(1);
    m->tp_err = m->arena.zalloc<int>(1);
    CK(cudaDeviceSynchronize());
    if (!make_tmap_bf16(&m->tp_xmap, m->tp_x, Ht, TB, (uint64_t)Ht * 2, 64, TB) ||
        !make_tmap_bf16(&m->tp_hmap, m->tp_h, Ht, TB, (uint64_t)Ht * 2, 64, TB))
      FAIL(Q3T_CUDA_ERROR, "TMA descriptor encoding failed for the text projection workspace");
  }
  cudaStream_t st = m->tp_st;
  std::vector<int> hid(TB);
  for (int c0 = 0; c0 < n; c0 += TB) {
    const int cnt = std::min(TB, n - c0);
    for (int i = 0; i < cnt; i++) hid[i] = (int)ids[c0 + i];
    CK(cudaMemcpyAsync(m->tp_ids, hid.data(), cnt * sizeof(int), cudaMemcpyHostToDevice, st));
    CK(cudaMemcpyAsync(m->tp_ntok, &cnt, sizeof(int), cudaMemcpyHostToDevice, st));
    gather_rows_bf16(m->text_emb, m->tp_ids, cnt, Ht, m->tp_x, st);
    GemmArgs g1 = gemm_args(m->tp_fc1, m->tp_ntok, TB);
    g1.xmode = GX_BF16;
    g1.tx = m->tp_xmap;
    g1.xb = m->tp_x;
    g1.ldx = Ht;
    g1.epi = GE_BIAS_SILU;
    g1.h = m->tp_h;
    g1.ldh = Ht;
    g1.bias = m->tp_b1;
    g1.err = m->tp_err;
    gemm(g1, TB, st);
    GemmArgs g2 = gemm_args(m->tp_fc2, m->tp_ntok, TB);
    g2.xmode = GX_BF16;
    g2.tx = m->tp_hmap;
    g2.xb = m->tp_h;
    g2.ldx = Ht;
    g2.epi = GE_BIAS_BF16;
    g2.y = m->tp_out;
    g2.ldy = H;
    g2.bias = m->tp_b2;
    g2.err = m->tp_err;
    gemm(g2, TB, st);
    check_launches();
    CK(cudaMemcpyAsync(out + (size_t)c0 * H, m->tp_out, (size_t)cnt * H * sizeof(float), kind, st));
    CK(cudaStreamSynchronize(st));  // hid and the workspace are reused by the next pass
  }
  int e = 0;
  CK(cudaMemcpy(&e, m->tp_err, sizeof(int), cudaMemcpyDeviceToHost));
  if (e) {
    CK(cudaMemset(m->tp_err, 0, sizeof(int)));
    FAIL(Q3T_DEVICE_TIMEOUT, "text projection: a bounded device wait gave up (code %d)", e);
  }
}

extern "C" q3t_status q3t_text_project(q3t_model *m, const int64_t *ids, int n, float *out) {
  if (!m || n < 0 || (n > 0 && (!ids || !out))) {
    set_error("q3t_text_project: bad argument");
    return Q3T_INVALID_INPUT;
  }
  if (!m->text_emb) {
    set_error("q3t_text_project: the model has no text_embedding / text_projection tensors");
    return Q3T_INVALID_INPUT;
  }
  for (int i = 0; i < n; i++)
    if (ids[i] < 0 || ids[i] >= m->text_vocab) {
      set_error("q3t_text_project: token id %lld outside [0, %d)", (long long)ids[i], m->text_vocab);
      return Q3T_INVALID_INPUT;
    }
  std::lock_guard<std::mutex> lock(m->tp_mu);
  return guard([&] {
    CK(cudaSetDevice(m->device));
    text_project_rows(m, ids, n, out, cudaMemcpyDeviceToHost);
  });
}

extern "C" q3t_status q3t_session_seed(q3t_model *m, const int64_t *text_ids, int n_text, const int64_t *leading_ids,
                                       int n_leading, const q3t_seed_controls *c, float *inputs_embeds, int max_rows,
                                       int *rows, float *pad_embed) {
  if (!m || !text_ids || !c || !rows || n_leading < 0 || (n_leading > 0 && !leading_ids) ||
      (c->n_codec_prefix > 0 && !c->codec_prefix_ids)) {
    set_error("q3t_session_seed: bad argument");
    return Q3T_INVALID_INPUT;
  }
  if (!m->text_emb) {
    set_error("q3t_session_seed: the model has no text_embedding / text_projection tensors");
    return Q3T_INVALID_INPUT;
  }
  // text_ids = 3 role ids, the body, 5 trailing ids (session_seed.rs:159-160)
  if (n_text < 8 || c->n_codec_prefix < 2) {
    set_error("q3t_session_seed: %d text ids (>= 8: role 3 + body + 5) and %d codec prefix ids (>= 2)", n_text,
              c->n_codec_prefix);
    return Q3T_INVALID_INPUT;
  }
  const int H = m->tc.talker.hidden_size, V = m->tc.talker.vocab_size, ncp = c->n_codec_prefix;
  const int body = n_text - 8, S = n_leading + 3 + (ncp - 1) + body + 2;
  *rows = S;
  if (!inputs_embeds) return Q3T_OK;
  if (max_rows < S) {
    set_error("q3t_session_seed: the seed has %d rows, the output holds %d", S, max_rows);
    return Q3T_INVALID_INPUT;
  }
  // projected ids: [bos, eos, pad] + role (3) + body + leading
  std::vector<int64_t> pid = {c->tts_bos_token_id, c->tts_eos_token_id, c->tts_pad_token_id};
  for (int i = 0; i < 3 + body; i++) pid.push_back(text_ids[i]);
  for (int i = 0; i < n_leading; i++) pid.push_back(leading_ids[i]);
  for (int64_t id : pid)
    if (id < 0 || id >= m->text_vocab) {
      set_error("q3t_session_seed: text token id %lld outside [0, %d)", (long long)id, m->text_vocab);
      return Q3T_INVALID_INPUT;
    }
  std::vector<int64_t> cid(c->codec_prefix_ids, c->codec_prefix_ids + ncp - 1);
  cid.push_back(c->codec_pad_id);
  cid.push_back(c->codec_bos_id);
  for (int64_t id : cid)
    if (id < 0 || id >= V) {
      set_error("q3t_session_seed: codec token id %lld outside [0, %d)", (long long)id, V);
      return Q3T_INVALID_INPUT;
    }
  enum { BOS = 0, EOS = 1, PAD = 2, ROLE = 3, BODY = 6 };
  const int LEAD = BODY + body;
  std::vector<int> tr, ci;  // per output row: projected row, codec id (-1: none)
  for (int i = 0; i < n_leading; i++) tr.push_back(LEAD + i), ci.push_back(-1);
  for (int i = 0; i < 3; i++) tr.push_back(ROLE + i), ci.push_back(-1);
  for (int i = 0; i < ncp - 1; i++) tr.push_back(i < ncp - 2 ? PAD : BOS), ci.push_back((int)c->codec_prefix_ids[i]);
  for (int i = 0; i < body; i++) tr.push_back(BODY + i), ci.push_back((int)c->codec_pad_id);
  tr.push_back(EOS), ci.push_back((int)c->codec_pad_id);
  tr.push_back(PAD), ci.push_back((int)c->codec_bos_id);
  std::lock_guard<std::mutex> lock(m->tp_mu);
  return guard([&] {
    CK(cudaSetDevice(m->device));
    const int np = (int)pid.size();
    float *P = nullptr, *out = nullptr;
    int *d_tr = nullptr, *d_ci = nullptr;
    CK(cudaMalloc(&P, (size_t)np * H * sizeof(float)));
    CK(cudaMalloc(&out, (size_t)S * H * sizeof(float)));
    CK(cudaMalloc(&d_tr, (size_t)S * 2 * sizeof(int)));
    d_ci = d_tr + S;
    struct Free {
      void *p[3];
      ~Free() {
        for (void *q : p) cudaFree(q);
      }
    } fr{{P, out, d_tr}};
    text_project_rows(m, pid.data(), np, P, cudaMemcpyDeviceToDevice);
    cudaStream_t st = m->tp_st;
    CK(cudaMemcpyAsync(d_tr, tr.data(), S * sizeof(int), cudaMemcpyHostToDevice, st));
    CK(cudaMemcpyAsync(d_ci, ci.data(), S * sizeof(int), cudaMemcpyHostToDevice, st));
    seed_rows(P, m->talker_emb, d_tr, d_ci, S, H, out, st);
    check_launches();
    CK(cudaMemcpyAsync(inputs_embeds, out, (size_t)S * H * sizeof(float), cudaMemcpyDeviceToHost, st));
    if (pad_embed)
      CK(cudaMemcpyAsync(pad_embed, P + (size_t)PAD * H, H * sizeof(float), cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
  });
}

extern "C" q3t_status q3t_session_seed_voice_clone(q3t_model *m, const int64_t *text_ids, int n_text,
                                                   const float *speaker, const int64_t *ref_text_ids, int n_ref_text,
                                                   const int64_t *ref_codes, int ref_frames,
                                                   const q3t_seed_controls *c, float *inputs_embeds, int max_rows,
                                                   int *rows, float *trailing, int max_trailing, int *trailing_rows,
                                                   float *pad_embed) {
  const bool icl = ref_text_ids != nullptr;
  if (!m || !text_ids || !speaker || !c || !rows || !trailing_rows ||
      (c->n_codec_prefix > 0 && !c->codec_prefix_ids) || (icl && (!ref_codes || ref_frames < 1))) {
    set_error("q3t_session_seed_voice_clone: bad argument");
    return Q3T_INVALID_INPUT;
  }
  if (!m->text_emb || !m->has_talker) {
    set_error("q3t_session_seed_voice_clone: the model has no talker / text_embedding / text_projection tensors");
    return Q3T_INVALID_INPUT;
  }
  // text_ids = 3 role ids, the body, 5 trailing ids; reference text = 3 role
  // ids, its body, 2 trailing ids (session_seed.rs:337-338)
  if (n_text < 8 || c->n_codec_prefix < 2 || (icl && n_ref_text < 5)) {
    set_error("q3t_session_seed_voice_clone: %d text ids (>= 8), %d reference text ids (>= 5) and %d codec prefix "
              "ids (>= 2)",
              n_text, n_ref_text, c->n_codec_prefix);
    return Q3T_INVALID_INPUT;
  }
  const int H = m->tc.talker.hidden_size, V = m->tc.talker.vocab_size, PV = m->tc.predictor.vocab_size;
  const int G = m->tc.num_code_groups, ncp = c->n_codec_prefix, body = n_text - 8;
  const int T = icl ? ref_frames : 0;
  // projected rows: [bos, eos, pad], role (3), then the body (x-vector
  // recipe) or reference body + target body + eos (in-context recipe)
  enum { BOS = 0, EOS = 1, PAD = 2, ROLE = 3, TXT = 6 };
  std::vector<int64_t> pid = {c->tts_bos_token_id, c->tts_eos_token_id, c->tts_pad_token_id};
  for (int i = 0; i < 3; i++) pid.push_back(text_ids[i]);
  if (icl)
    for (int i = 3; i < n_ref_text - 2; i++) pid.push_back(ref_text_ids[i]);
  for (int i = 3; i < n_text - 5; i++) pid.push_back(text_ids[i]);
  if (icl) pid.push_back(c->tts_eos_token_id);
  const int text_len = (int)pid.size() - TXT;
  for (int64_t id : pid)
    if (id < 0 || id >= m->text_vocab) {
      set_error("q3t_session_seed_voice_clone: text token id %lld outside [0, %d)", (long long)id, m->text_vocab);
      return Q3T_INVALID_INPUT;
    }
  std::vector<int64_t> cid(c->codec_prefix_ids, c->codec_prefix_ids + ncp - 2);
  cid.push_back(c->codec_pad_id);
  cid.push_back(c->codec_bos_id);
  for (int64_t id : cid)
    if (id < 0 || id >= V) {
      set_error("q3t_session_seed_voice_clone: codec token id %lld outside [0, %d)", (long long)id, V);
      return Q3T_INVALID_INPUT;
    }
  for (int g = 0; g < (icl ? G : 0); g++)
    for (int t = 0; t < T; t++) {
      const int64_t id = ref_codes[(size_t)g * T + t];
      if (id < 0 || id >= (g == 0 ? V : PV)) {
        set_error("q3t_session_seed_voice_clone: reference code %lld of group %d outside [0, %d)", (long long)id, g,
                  g == 0 ? V : PV);
        return Q3T_INVALID_INPUT;
      }
    }
  // per output row: projected row, codec id, X row (-1: none); X row 0 is
  // the x-vector, X row 1 + t reference frame t
  std::vector<int> tr, ci, xr;
  auto row = [&](int t, int c_id, int x) {
    tr.push_back(t);
    ci.push_back(c_id);
    xr.push_back(x);
  };
  for (int i = 0; i < 3; i++) row(ROLE + i, -1, -1);
  // voice_clone_codec_prefix (session_seed.rs:538-584)
  for (int i = 0; i < ncp - 2; i++) row(PAD, (int)c->codec_prefix_ids[i], -1);
  row(PAD, -1, 0);
  row(BOS, (int)c->codec_pad_id, -1);
  std::vector<int> trail;  // trailing text hidden: projected rows
  if (!icl) {  // x-vector recipe (:299-318)
    if (body > 0) row(TXT, (int)c->codec_bos_id, -1);
    for (int i = 1; i < body; i++) trail.push_back(TXT + i);
    trail.push_back(EOS);
  } else {  // build_voice_clone_icl_seed (:324-396)
    const int codec_len = 1 + T;
    for (int i = 0; i < codec_len; i++) row(i < text_len ? TXT + i : PAD, i == 0 ? (int)c->codec_bos_id : -1, i);
    if (text_len > codec_len)
      for (int i = codec_len; i < text_len; i++) trail.push_back(TXT + i);
    else
      trail.push_back(PAD);
  }
  const int S = (int)tr.size(), NT = (int)trail.size();
  *rows = S;
  *trailing_rows = NT;
  if (!inputs_embeds) return Q3T_OK;
  if (max_rows < S || max_trailing < NT || !trailing) {
    set_error("q3t_session_seed_voice_clone: the seed has %d rows and %d trailing rows, the outputs hold %d and %d",
              S, NT, max_rows, max_trailing);
    return Q3T_INVALID_INPUT;
  }
  for (int t : trail) row(t, -1, -1);  // trailing rows: the projected rows as they are
  std::lock_guard<std::mutex> lock(m->tp_mu);
  return guard([&] {
    CK(cudaSetDevice(m->device));
    const int np = (int)pid.size(), R = S + NT;
    float *P = nullptr, *out = nullptr, *X = nullptr;
    int *d_idx = nullptr;
    int64_t *d_codes = nullptr;
    CK(cudaMalloc(&P, (size_t)np * H * sizeof(float)));
    struct Free {
      std::vector<void *> p;
      ~Free() {
        for (void *q : p) cudaFree(q);
      }
    } fr;
    fr.p.push_back(P);
    CK(cudaMalloc(&out, (size_t)R * H * sizeof(float)));
    fr.p.push_back(out);
    CK(cudaMalloc(&X, (size_t)(1 + T) * H * sizeof(float)));
    fr.p.push_back(X);
    CK(cudaMalloc(&d_idx, (size_t)R * 3 * sizeof(int)));
    fr.p.push_back(d_idx);
    CK(cudaMalloc(&d_codes, (size_t)std::max(1, G * T) * sizeof(int64_t)));
    fr.p.push_back(d_codes);
    float *d_spk = X;  // the x-vector in row 0 of X, rounded there in place
    text_project_rows(m, pid.data(), np, P, cudaMemcpyDeviceToDevice);
    cudaStream_t st = m->tp_st;
    CK(cudaMemcpyAsync(d_spk, speaker, (size_t)H * sizeof(float), cudaMemcpyHostToDevice, st));
    if (T > 0)
      CK(cudaMemcpyAsync(d_codes, ref_codes, (size_t)G * T * sizeof(int64_t), cudaMemcpyHostToDevice, st));
    CK(cudaMemcpyAsync(d_idx, tr.data(), R * sizeof(int), cudaMemcpyHostToDevice, st));
    CK(cudaMemcpyAsync(d_idx + R, ci.data(), R * sizeof(int), cudaMemcpyHostToDevice, st));
    CK(cudaMemcpyAsync(d_idx + 2 * R, xr.data(), R * sizeof(int), cudaMemcpyHostToDevice, st));
    clone_rows(d_spk, d_codes, G, T, m->talker_emb, m->cp_emb_dev, H, X, st);
    seed_rows(P, m->talker_emb, d_idx, d_idx + R, R, H, out, st, X, d_idx + 2 * R);
    check_launches();
    CK(cudaMemcpyAsync(inputs_embeds, out, (size_t)S * H * sizeof(float), cudaMemcpyDeviceToHost, st));
    CK(cudaMemcpyAsync(trailing, out + (size_t)S * H, (size_t)NT * H * sizeof(float), cudaMemcpyDeviceToHost, st));
    if (pad_embed)
      CK(cudaMemcpyAsync(pad_embed, P + (size_t)PAD * H, H * sizeof(float), cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
  });
}

extern "C" q3t_status q3t_text_dims(const q3t_model *m, int *text_vocab, int *text_hidden) {
  if (!m) return Q3T_INVALID_INPUT;
  if (text_vocab) *text_vocab = m->text_vocab;
  if (text_hidden) *text_hidden = m->text_hidden;
  return Q3T_OK;
}

// ----------------------------------------------------------------------------
// The device sampler on one row of logits with a given uniform draw (test
// hook of sample_token, talker/infer/sampling.rs:33-90): the same k_sample the
// decode frames run, with the draw and the candidate mask exposed.
extern "C" q3t_status q3t_sample_logits(q3t_model *m, const float *logits, int vocab, const q3t_sampling *smp,
                                        const int64_t *suppress, int n_suppress, double u, int64_t *token,
                                        uint8_t *kept) {
  if (!m || !logits || !smp || !token || vocab <= 0 || vocab > kSampleMaxV || n_suppress < 0 ||
      (n_suppress > 0 && !suppress) || !(u >= 0.0 && u < 1.0)) {
    set_error("q3t_sample_logits: bad argument (vocab 1..%d, u in [0, 1))", kSampleMaxV);
    return Q3T_INVALID_INPUT;
  }
  return guard([&] {
    CK(cudaSetDevice(m->device));
    cudaStream_t st;
    CK(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    struct Buf {
      float *lg, *row;
      int64_t *sup, *codes;
      SampleParams *params;
      int *ntok, *zero, *sup_on;
      double *u;
      uint8_t *kept;
    } d{};
    const size_t nsup = (size_t)std::max(n_suppress, 1);
    const size_t bytes = (size_t)vocab * 8 + nsup * 8 + 8 + 2 * sizeof(SampleParams) + 16 + 8 + (size_t)vocab + 256;
    unsigned char *base = nullptr;
    CK(cudaMallocAsync((void **)&base, bytes, st));
    unsigned char *p = base;
    auto take = [&](size_t n) {
      unsigned char *r = p;
      p += (n + 15) & ~(size_t)15;
      return r;
    };
    d.lg = (float *)take((size_t)vocab * 4);
    d.row = (float *)take((size_t)vocab * 4);
    d.sup = (int64_t *)take(nsup * 8);
    d.codes = (int64_t *)take(8);
    d.params = (SampleParams *)take(2 * sizeof(SampleParams));
    d.ntok = (int *)take(4);
    d.zero = (int *)take(4);
    d.sup_on = (int *)take(4);
    d.u = (double *)take(8);
    d.kept = (uint8_t *)take((size_t)vocab);
    SampleParams hp[2] = {to_params(*smp), to_params(*smp)};
    const int one = 1, zero = 0;
    CK(cudaMemcpyAsync(d.lg, logits, (size_t)vocab * 4, cudaMemcpyHostToDevice, st));
    if (n_suppress) CK(cudaMemcpyAsync(d.sup, suppress, (size_t)n_suppress * 8, cudaMemcpyHostToDevice, st));
    CK(cudaMemcpyAsync(d.params, hp, sizeof hp, cudaMemcpyHostToDevice, st));
    CK(cudaMemcpyAsync(d.ntok, &one, 4, cudaMemcpyHostToDevice, st));
    CK(cudaMemcpyAsync(d.zero, &zero, 4, cudaMemcpyHostToDevice, st));
    CK(cudaMemcpyAsync(d.sup_on, &one, 4, cudaMemcpyHostToDevice, st));
    CK(cudaMemcpyAsync(d.u, &u, 8, cudaMemcpyHostToDevice, st));
    SampleArgs a{};
    a.part = Part{d.lg, 1, 0, vocab};
    a.logits = d.row;
    a.ldl = vocab;
    a.V = vocab;
    a.ntok = d.ntok;
    a.slot = d.zero;
    a.params = d.params;
    a.suppress = n_suppress ? d.sup : nullptr;
    a.n_suppress = n_suppress;
    a.sup_on = d.sup_on;
    a.codes = d.codes;
    a.G = 1;
    a.col = 0;
    a.frame = d.zero;
    a.u = d.u;
    a.kept = d.kept;
    sample(a, 1, st);
    check_launches();
    CK(cudaMemcpyAsync(token, d.codes, 8, cudaMemcpyDeviceToHost, st));
    if (kept) CK(cudaMemcpyAsync(kept, d.kept, (size_t)vocab, cudaMemcpyDeviceToHost, st));
    CK(cudaFreeAsync(base, st));
    CK(cudaStreamSynchronize(st));
    CK(cudaStreamDestroy(st));
  });
}

extern "C" const char *q3t_last_error(void) { return q3t::g_err.c_str(); }
extern "C" const char *q3t_version(void) { return "q3t-b200 0.1 (sm_100a)"; }
extern "C" int64_t q3t_kernel_launches(void) { return q3t::g_launches; }

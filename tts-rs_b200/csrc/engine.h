// Host runtime shared by the C ABI (engine.cu) and the codec (codec.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <deque>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

#include "../../include/q3t.h"
#include "frame.cuh"
#include "lm_kernels.cuh"
#include "mk.cuh"

namespace q3t {

void set_error(const char *fmt, ...);

struct CudaFail {
  cudaError_t err;
  std::string what;
};

// Throws CudaFail; every ABI entry point converts it to Q3T_CUDA_ERROR.
#define CK(call)                                                   \
  do {                                                             \
    cudaError_t e_ = (call);                                       \
    if (e_ != cudaSuccess) throw ::q3t::CudaFail{e_, #call};       \
  } while (0)

struct Status {
  q3t_status code;
  std::string msg;
};
#define FAIL(code, ...)                   \
  do {                                    \
    ::q3t::set_error(__VA_ARGS__);        \
    throw ::q3t::Status{code, ""};        \
  } while (0)

// The other checkpoint spelling of a tensor name, or "" if it has none: the
// codec's quantizer statistics are stored under `._codebook.` in legacy
// checkpoints and `.codebook.` in newer ones, and the reference accepts both
// (codec/weights.rs:27-33 remaps the legacy spelling at load).
inline std::string checkpoint_alias(const std::string &n) {
  const std::string legacy = "._codebook.", modern = ".codebook.";
  size_t i = n.find(legacy);
  if (i != std::string::npos) return n.substr(0, i) + modern + n.substr(i + legacy.size());
  i = n.find(modern);
  if (i != std::string::npos) return n.substr(0, i) + legacy + n.substr(i + modern.size());
  return "";
}

// Device allocations owned by an object, released together.
struct DevArena {
  std::vector<void *> ptrs;
  template <typename T>
  T *alloc(size_t n) {
    void *p = nullptr;
    if (n == 0) n = 1;
    CK(cudaMalloc(&p, n * sizeof(T)));
    ptrs.push_back(p);
    return reinterpret_cast<T *>(p);
  }
  template <typename T>
  T *zalloc(size_t n) {
    T *p = alloc<T>(n);
    CK(cudaMemset(p, 0, (n ? n : 1) * sizeof(T)));
    return p;
  }
  void release() {
    for (void *p : ptrs) cudaFree(p);
    ptrs.clear();
  }
  ~DevArena() { release(); }
};

// Device-side decoder stack (talker or code predictor).
struct LMStack {
  q3t_lm_config cfg{};
  std::vector<float *> in_norm, post_norm, q_norm, k_norm;  // f32
  std::vector<q3t::Linear> qkv, o, gu, down;  // bf16 row-major (gate/up interleaved per 64 rows)
  float *final_norm = nullptr;
  float *inv_freq = nullptr;  // [head_dim / 2]
};

struct CodecModel;  // codec.cu

// host tensor -> device (engine.cu); copies run on `st`
float *upload_f32(const q3t_tensor *t, DevArena &ar, cudaStream_t st);
uint16_t *upload_bf16(const q3t_tensor *t, DevArena &ar, cudaStream_t st);

constexpr int kPage = 16;
constexpr int kMaxSeq = 4096;                 // the reference's talker cache capacity
constexpr int kPtStride = kMaxSeq / kPage;    // pages per sequence
constexpr int kPredPages = 2;                 // predictor KV pages per slot (num_code_groups + 1 <= 32 keys)
constexpr int kPrefillTok = 64;               // prompt tokens per chunk of a session's prefill
constexpr int kTalkerTok = 128;               // tokens of a batched talker pass: decode tokens + prompt-chunk tokens

struct Req {
  int64_t id = 0;
  int state = 0;  // 0 queued, 1 active, 2 finished, 3 failed
  int slot = -1;
  std::vector<float> prompt, trailing, pad;
  int S = 0, trailing_len = 0;
  q3t_sampling ts{}, cs{};
  int max_new = 0;
  int64_t eos = -1;
  std::vector<int64_t> suppress;
  std::vector<int64_t> forced;  // [max_new][G]
  int64_t forced_first = -1;
  float *first_logits = nullptr;
  int step_idx = 0;
  bool eos_seen = false, finished = false;
  int cache_len = 0;
  std::vector<int> pages;
  float *d_trailing = nullptr, *d_pad = nullptr, *d_prompt = nullptr;
  int64_t *d_forced = nullptr, *d_suppress = nullptr;
  bool admitted_now = false;  // prefilled in the current step (its first-token EOS flag is read after the frame)
  bool decoding = false;      // first token known: the request takes part in decode frames
  int prefill_pos = 0;        // prompt tokens already run through the talker (chunked prefill inside frames)
  int64_t admit_order = 0;    // admission sequence number (prompt chunks are served in this order)
  std::vector<int64_t> codes;  // [G][T] once retired
  std::vector<int32_t> sampled;  // [G][T] sampled tokens before teacher forcing
  std::vector<float> wave;
  int64_t samples = 0;
  std::string error;
  q3t_status fail_status = Q3T_INVALID_INPUT;  // the status of the failure (state 3)
};

// Slot state a prefill uploads, staged in pinned memory (one per slot).
struct SlotInit {
  SampleParams params[2];
  int64_t eos, forced_first;
  int32_t forced_first32, zero, sup_on, forced_count, nsup, pad;
};

struct GraphEntry {
  cudaGraphExec_t exec = nullptr;
  int64_t nodes = 0;
};

enum MetaOff {
  M_NTOK_B = 0,   // decode tokens of the frame (the code-predictor loop's batch)
  M_NTOK_2B = 1,
  M_ONE = 2,
  M_NPRE = 3,
  M_SEED = 4,
  M_NTOK_T = 5,   // tokens of the talker pass: decode tokens, then prompt-chunk tokens
  M_NTOK_H = 6,   // tokens sampled by the talker head: decode tokens, then completed prompts' last tokens
  M_HDR = 8,
};

}  // namespace q3t

struct q3t_model {
  int device = 0;
  q3t_talker_config tc{};
  q3t_codec_config cc{};
  bool has_talker = false, has_codec = false;
  q3t::LMStack talker, pred;
  q3t::Linear codec_head;                    // [vocab][H]
  uint16_t *talker_emb = nullptr;            // row-major bf16 [vocab][H]
  std::vector<uint16_t *> cp_emb;            // row-major bf16
  std::vector<q3t::Linear> lm_heads;
  uint16_t **cp_emb_dev = nullptr;           // device array of cp_emb pointers
  int64_t kv_pages = 8192;
  int max_active = 64;
  q3t::CodecModel *codec = nullptr;
  // text projection (optional tensors): text_embedding [text_vocab][text_hidden]
  // bf16, linear_fc1 [text_hidden][text_hidden] + bias, linear_fc2 [hidden][text_hidden] + bias
  int text_vocab = 0, text_hidden = 0;
  uint16_t *text_emb = nullptr;
  q3t::Linear tp_fc1, tp_fc2;
  float *tp_b1 = nullptr, *tp_b2 = nullptr;
  std::mutex tp_mu;  // guards the workspace below (model handles are shared by threads)
  cudaStream_t tp_st = nullptr;
  uint16_t *tp_x = nullptr, *tp_h = nullptr;
  float *tp_out = nullptr;
  int *tp_ids = nullptr, *tp_ntok = nullptr, *tp_err = nullptr;
  CUtensorMap tp_xmap, tp_hmap;
  q3t::DevArena arena;
};

struct q3t_batch {
  q3t_model *m = nullptr;
  q3t_batch_desc desc{};
  int A = 0, G = 0, H = 0, V = 0, PV = 0, NQKV = 0, NQKVP = 0, I2 = 0;
  cudaStream_t st = nullptr;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  cudaEvent_t evf[3] = {nullptr, nullptr, nullptr};  // decode frame: start, predictor done, talker done
  bool frame_timed = false;
  q3t::DevArena ar;
  // talker pool
  uint16_t *tk = nullptr, *tv = nullptr;
  int64_t t_layer_stride = 0;
  int n_pages = 0;
  std::vector<int> free_pages;
  int *d_pt = nullptr;
  int *h_pt = nullptr;                   // pinned host copy of the page table [A][kPtStride]
  int pt_lo = 1 << 30, pt_hi = -1;       // slot rows changed since the last upload
  // predictor pool (2 pages per slot)
  uint16_t *pk = nullptr, *pv = nullptr;
  int64_t p_layer_stride = 0;
  int *d_ppt = nullptr;
  // slot state
  int maxF = 0;
  int64_t *d_codes = nullptr, *d_hist_codes = nullptr, *d_forced = nullptr, *d_eos = nullptr;
  int64_t *d_suppress = nullptr;   // [slot][n_suppress_cap] suppress list of each slot's request
  int *d_nsup = nullptr;           // [slot] its length
  int32_t *d_raw = nullptr;
  int n_suppress_cap = 4096;
  float *d_hidden = nullptr;
  int32_t *d_thist = nullptr;
  int *d_thist_len = nullptr, *d_sup_on = nullptr, *d_forced_count = nullptr;
  int hist_cap = 0;
  q3t::SampleParams *d_params = nullptr;
  // activations
  int Tmax = 0;
  float *x = nullptr, *tlog = nullptr, *plog = nullptr;
  float *ss = nullptr;    // [hidden / 128][Tmax] sum-of-squares partials of the residual rows
  float *hlog = nullptr;  // [Tmax][max(V, PV)] head GEMM output
  uint16_t *xn = nullptr, *q = nullptr, *attn = nullptr, *act = nullptr;
  uint16_t *xg = nullptr;  // [Tmax][hidden] bf16(x * gamma of the next RMSNorm), written with x
  q3t::AttnWork ws{};
  // metadata
  int meta_n = 0;
  int *d_meta = nullptr, *h_meta = nullptr;
  const float **d_extra = nullptr, **h_extra = nullptr;
  int *d_pmeta = nullptr, *h_pmeta = nullptr;  // prefill metadata blocks (pinned staging + device)
  int pmeta_blocks = 0, pmeta_used = 0;        // capacity; blocks handed out since the stream last synchronised
  int *d_eosflag = nullptr, *h_eosflag = nullptr;
  int64_t *h_codes = nullptr;
  // admission without host round trips: per-slot pinned staging of the slot
  // state a prefill uploads, and the first token's EOS flag per slot (read
  // back with the step's other flags)
  q3t::SlotInit *h_init = nullptr;
  int *d_first_eos = nullptr, *h_first_eos = nullptr;
  int *d_zero = nullptr;                 // one device int that stays 0 (frame index of a first token)
  cudaMemPool_t pool = nullptr;          // stream-ordered pool for request inputs (no device-wide syncs)
  // graphs
  bool use_graphs = true;
  std::map<std::tuple<int, int, int>, q3t::GraphEntry> graphs;
  std::map<std::pair<int, int>, std::vector<q3t::Phase>> programs;  // decode-frame phase lists
  std::map<std::tuple<const void *, int, int>, CUtensorMap> xmaps;  // (X buffer, K, token tiles) -> TMA map
  int *d_err = nullptr, *h_err = nullptr;  // bounded-wait timeouts reported by the GEMM kernels
  // streamed small-batch kernel (mk.cu): programs by kind, raw q/k/v rows, stage counters
  bool use_mk = false;
  int mk_grid = 0;
  uint2 *mk_x = nullptr;     // [2][kMkMaxTok][hidden] tagged residual rows (alternating)
  uint2 *mk_qkv = nullptr;   // [kMkMaxTok][max NQKV] tagged raw q/k/v rows
  uint2 *mk_act = nullptr;   // [kMkMaxTok][max intermediate] tagged SwiGLU rows
  uint2 *mk_attn = nullptr;  // [kMkMaxTok][max heads x 128] tagged attention output rows
  uint2 *mk_part = nullptr;  // [kMkMaxTok][max kv heads][kAttnMaxUnits][2][kMkPartLd] tagged attention partials
  unsigned *mk_ctr = nullptr;  // launch epoch, finished CTAs, a word nothing sets (the stall test's flag)
  int wait_polls = 0;          // poll limit of k_mk's tagged-data waits (0: the kernel's default)
  bool stall_waits = false;    // k_mk first waits on the never-set word (timeout tests)
  std::map<int, std::pair<q3t::MkStage *, int>> mk_progs;
  // persistent frame kernel (frame.cu) for the code-predictor loop
  bool use_frame = false;
  int frame_grid = 0, frame_hc = 0;
  unsigned *frame_bar = nullptr;
  std::map<std::pair<int, int>, q3t::Phase *> frame_progs;  // device copies of the predictor phases
  int step_counter = 0;
  // requests
  std::vector<q3t::Req *> slots;
  std::deque<q3t::Req *> queue;
  std::map<int64_t, std::unique_ptr<q3t::Req>> reqs;
  int64_t next_id = 1;
  float last_ms = 0.f;
  bool session_mode = false;
  int64_t h2d = 0, d2h = 0;  // bytes copied since the last step report
  std::vector<int64_t> last_ids;  // request ids of the last decode frame, in token order

  int off_slot() const { return q3t::M_HDR; }
  int off_tpos() const { return q3t::M_HDR + A; }
  int off_frame() const { return q3t::M_HDR + 2 * A; }
  int off_zero() const { return q3t::M_HDR + 3 * A; }
  int off_p0seq() const { return q3t::M_HDR + 4 * A; }
  int off_p0pos() const { return q3t::M_HDR + 6 * A; }
  // talker pass and talker head token lists (decode tokens first), TT entries each
  int TT() const { return q3t::kTalkerTok; }
  int off_tseq() const { return q3t::M_HDR + 8 * A; }
  int off_ttpos() const { return off_tseq() + TT(); }
  int off_hslot() const { return off_tseq() + 2 * TT(); }
  int off_hframe() const { return off_tseq() + 3 * TT(); }
  int off_hrow() const { return off_tseq() + 4 * TT(); }
  int64_t admit_counter = 0;
  int pmeta_stride() const { return 8 + 2 * q3t::kPrefillTok + 8; }
};


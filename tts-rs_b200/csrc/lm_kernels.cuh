// Host-side launchers of the talker / code-predictor kernels (lm_kernels.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace q3t {

// Paged KV cache of one decoder stack.  Layout per layer l:
//   K at k + l * layer_stride, V at v + l * layer_stride, each
//   [num_pages][n_kv][16][head_dim] bf16, i.e. one 4 KB contiguous slab per
//   (page, kv head).  page_table[seq * pt_stride + j / 16] is the physical
//   page holding token j of sequence `seq`.
struct KVView {
  uint16_t *k, *v;
  int64_t layer_stride;  // elements between layers
  const int *page_table;
  int pt_stride;
  int n_kv;
};

// Per-token batch description (device arrays, ntok read from device).
struct TokView {
  const int *ntok;     // number of active tokens
  const int *seq;      // [tok] sequence (page-table row)
  const int *pos;      // [tok] position (kv length after append = pos + 1)
  int pos_add;         // added to pos[] (code-predictor passes use pos[] = 0)
};

struct AttnWork {
  float *part;    // [max_tok][n_kv][max_split][2][132]
  int *counters;  // [max_tok][n_kv], zero between launches
  int max_split;
};

// Split-K partial sums of one linear's output: value(t, n) =
// sum over s < splits of p[s * stride + t * ld + n].  Consumers reduce them
// in a fixed order, so results do not depend on scheduling.
struct Part {
  const float *p;
  int splits;
  long long stride;
  int ld;
};

extern bool g_use_pdl;
// one-time kernel attribute setup (dynamic shared memory limits)
void init_kernel_attributes();
extern int64_t g_launches;
// first launch error since the last call (cudaSuccess if none)
cudaError_t take_launch_error(const char **kernel);

// Packs W [N][K] bf16 row-major into m16n8k16 A-fragment order.
void pack_weight(const uint16_t *src, uint16_t *dst, int N, int K, cudaStream_t st);
// f32 -> bf16 conversion on device.
void f32_to_bf16(const float *src, uint16_t *dst, int64_t n, cudaStream_t st);

// Decode-step input rows built from embeddings before a norm (src != 0);
// see d_rmsnorm in lm_device.cuh.
struct EmbedArgs {
  int src;  // 0 none, 1 predictor prefill pair, 2 predictor code embedding, 3 talker input
  int G, col;
  const float *hidden;         // [slot][H]
  const uint16_t *emb0;        // talker codec embedding [vocab][H]
  const uint16_t *const *embs; // predictor codec embeddings (device array)
  const uint16_t *emb;         // one predictor codec embedding (src 2)
  const int64_t *codes;        // [slot][G]
  const int *slot;             // [t]
  const float *const *extra;   // [t] trailing-text / pad row (src 3)
  const int *frame;            // [t]
  int64_t *hist;               // [slot][hist_frames][G] (src 3, nullable)
  int hist_frames;
};

// Row r = t*row_mul + row_add of the residual stream (optionally built from
// embeddings first): x[r] += sum of the pending partials `add` (written
// back), then out[t] = bf16(rmsnorm(x[r]) * gamma); optional f32 copy
// scattered to out_f32[slot[t]].
struct RmsArgs {
  float *x;
  int ldx, row_mul, row_add;
  Part add;
  const float *gamma;
  uint16_t *out;
  int ldo, H;
  float eps;
  const int *ntok;
  float *out_f32;
  const int *slot;
  EmbedArgs emb;
};
RmsArgs rms_args(float *x, int ldx, int row_mul, int row_add, Part add, const float *gamma, uint16_t *out, int ldo,
                 int H, float eps, const int *ntok, float *out_f32, const int *slot);
void rmsnorm(const RmsArgs &a, int grid_rows, cudaStream_t st);
// legacy form (no embedding source)
void rmsnorm(float *x, int ldx, int row_mul, int row_add, Part add, const float *gamma, uint16_t *out,
             int ldo, int H, float eps, const int *ntok, int grid_rows, float *out_f32, const int *slot,
             cudaStream_t st);

struct LinArgs {
  const uint4 *W;  // fragment-packed weights
  int N, K, fr, nt; // fragments per warp (K chunk = 16 fr), token tiles of 8
  const uint16_t *X;
  int ldx;
  float *P;
  long long pstride;
  int ldy;
  const int *ntok;
  int ntc;          // token chunks of 64
};
// Plans a linear: split count (fr), token tiles and the partial layout.
LinArgs linear_plan(const uint16_t *Wp, int N, int K, const void *X, int ldx, float *ws, long long ws_elems,
                    int rows_cap, const int *ntok, int max_tok, int target_items, Part *out);
__host__ __device__ int linear_items(const LinArgs &a);

// Y = X . W^T for t < ntok: writes split-K partials into ws (capacity
// ws_elems floats, rows_cap token rows per split) and returns their layout.
Part linear(const uint16_t *Wp, int N, int K, const void *X, int ldx, float *ws, long long ws_elems,
            int rows_cap, const int *ntok, int max_tok, cudaStream_t st);

struct SiluArgs {
  Part gu;
  int I;
  const int *ntok;
  uint16_t *out;
};

struct QkvArgs {
  Part qkv;
  const float *q_norm, *k_norm, *inv_freq;
  float eps;
  int nh, nkv;
  TokView tv;
  uint16_t *qout;
  KVView kv;
  int layer;
};

struct AttnArgs {
  Part qkv;
  const float *q_norm, *k_norm, *inv_freq;
  float eps;
  const uint16_t *qin;
  KVView kv;
  int layer;
  TokView tv;
  int nh, chunk, max_split, fused;
  float scale;
  AttnWork ws;
  uint16_t *out;
};

// out[t][n] = reduced partials, t < ntok
void reduce_rows(Part P, int N, const int *ntok, int max_tok, float *out, cudaStream_t st);

// out[t][i] = bf16(silu(g) * u) with g, u the reduced gate|up partials
void silu_mul(Part gu, int I, const int *ntok, int max_tok, uint16_t *out, cudaStream_t st);

// q/k RMSNorm + rotate-half RoPE + bf16 q out + K/V append into pages.
void qkv_post(Part qkv, const float *q_norm, const float *k_norm,
              const float *inv_freq, float eps, int nh, int nkv, TokView tv, int max_tok,
              uint16_t *qout, KVView kv, int layer, cudaStream_t st);

// Split-K flash-decoding over the paged cache, one token per (t): attends to
// positions [0, pos]; fused=1 also does qkv_post for its own head group
// (valid only when every token of the batch belongs to a distinct sequence).
void attention(int fused, Part qkv, const float *q_norm, const float *k_norm,
               const float *inv_freq, float eps, const uint16_t *qin, KVView kv, int layer,
               TokView tv, int max_tok, int nh, int chunk, int max_split, AttnWork ws,
               uint16_t *out, cudaStream_t st);

struct SampleParams {
  int do_sample;
  float temperature;
  int top_k;
  float top_p;
  float rep_penalty;  // <= 0: disabled
  int pad;
  unsigned long long seed;
};

// Per-token sampling from logits [t][V] (in place: the repetition penalty is
// written back).  Writes codes[slot[t]][col]; forced (nullable)
// [slot][frames][G]: if force[slot] the value forced[slot][frame[t] + fadd][col]
// replaces the sample.  Talker mode (col 0) also appends the token to
// hist[slot][hist_len[slot]++] and sets eos_flag[t].
struct SampleArgs {
  Part part;      // split-K partials of the logits
  float *logits;  // reduced (and penalised) logits are written here [t][ldl]
  int ldl;
  int V;
  const int *ntok;
  const int *slot;
  const SampleParams *params;  // [slot]
  int use_pred_params;         // 0: params[slot*2], 1: params[slot*2+1]
  const int64_t *suppress;     // [n_suppress] (applied where sup_on[slot] != 0)
  int n_suppress;
  int *sup_on;                 // [slot], cleared after use
  int64_t *codes;              // [slot][G]
  int G;
  int col;
  const int64_t *forced;       // [slot][max_frames][G] or null
  const int *force_on;         // [slot] number of teacher-forced frames
  int max_frames;
  const int *frame;            // [t]
  int fadd;
  int32_t *hist;               // [slot][hist_cap]
  int *hist_len;               // [slot]
  int hist_cap;
  int hist_mode;               // 0 none, 1 talker history (append), 2 predictor (codes 1..col-1)
  const int64_t *eos;          // [slot]
  int *eos_flag;               // [t]
  int step_seed;               // added to *seed_p (device step counter, nullable)
  const int *seed_p;
  int32_t *raw;                // [slot][max_frames][G] sampled tokens before forcing, or null
};
void sample(const SampleArgs &a, int max_tok, cudaStream_t st);

// ---------------------------------------------------------------------------
// Persistent frame kernel: one cooperative launch runs a whole decode frame
// as a list of phases separated by grid barriers (bounded spins; on timeout
// the kernel sets *err and every CTA returns).
// ---------------------------------------------------------------------------
enum PhaseType { PH_NORM = 1, PH_GEMM = 2, PH_QKV = 3, PH_ATTN = 4, PH_SILU = 5, PH_SAMPLE = 6 };

struct Phase {
  int type;
  int max_tok;   // rows / tokens the phase spans (items beyond ntok exit)
  int has_tail;  // PH_SAMPLE: run `tail` (embed + norm of the next input) per token
  int pad;
  union {
    RmsArgs norm;
    LinArgs lin;
    QkvArgs qkv;
    AttnArgs attn;
    SiluArgs silu;
    SampleArgs smp;
  };
  RmsArgs tail;
};

struct FrameCtl {
  unsigned *ctr;          // barrier counters, kFrameCtrWords words, zeroed before each launch
  int *err;               // set to 1 when a barrier wait times out
  unsigned long long *t;  // optional [n_phases + 1] %globaltimer stamps at phase starts (CTA 0)
};
constexpr int kFrameCtrWords = 17 * 32;
// grid size (CTAs) the frame kernel runs with on the current device
int frame_grid();
// items a GEMM phase should have so that every CTA holds at most one
int frame_target_items();
void frame_launch(const Phase *d_phases, int n_phases, FrameCtl ctl, cudaStream_t st);
// the same phase list run as one standalone kernel launch per phase
void run_phases(const Phase *phases, int n_phases, cudaStream_t st);

// Scatter dense bf16 K/V [layers][n_kv][len][hd] into the pages of `seq`.
void kv_import(const uint16_t *k, const uint16_t *v, int layers, int len, KVView kv, int seq,
               cudaStream_t st);

}  // namespace q3t

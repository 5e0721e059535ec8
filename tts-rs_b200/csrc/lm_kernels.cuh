// Host-side launchers of the talker / code-predictor kernels (lm_kernels.cu).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

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

// Attention work units: a warp handles up to `pw` pages of one (token, kv
// head); a (token, head) has at most kAttnMaxUnits units.
constexpr int kAttnMaxUnits = 64;
constexpr int kAttnMaxTok = 128;  // tokens per attention launch

struct AttnWork {
  float *part;    // [max_tok][n_kv][kAttnMaxUnits][2][132] unit partials (o, m, l)
  int *counters;  // [max_tok][n_kv], zero between launches
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

// Launch trace (profiling): while enabled, thread 0 of every CTA of k_gemm,
// k_attn, k_sample and k_rmsnorm appends one record with the launch's grid
// id and device timestamps (%globaltimer, ns): entry, after the dependency
// wait, after X staging, after the MMAs, after the split-K reduction
// barrier, after the epilogue, exit (stamps a kernel does not have are 0).
struct TraceRec {
  unsigned long long grid;
  unsigned long long t[7];
  int kind;  // 1 rmsnorm, 2 gemm, 3 attention, 4 sampler
  int cta;
  int n, k;  // k_gemm: N, K
};
// Starts recording into a device buffer of `cap` records (false if it
// cannot be allocated); trace_stop copies the records out and stops.
bool trace_start(size_t cap, cudaStream_t st);
void trace_stop(std::vector<TraceRec> &out, cudaStream_t st);
// one-time kernel attribute setup (dynamic shared memory limits)
void init_kernel_attributes();
extern int64_t g_launches;
// first launch error since the last call (cudaSuccess if none)
cudaError_t take_launch_error(const char **kernel);
// records a launch error (kept until take_launch_error)
void note_launch(cudaError_t e, const char *what);

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
  const int *row_idx;  // nullable: row t is x[row_idx[t]] instead of t * row_mul + row_add
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

// ---------------------------------------------------------------------------
// Skinny GEMM Y[t][n] = X[t] . W[n] for up to 64 tokens per CTA tile, as
// thread-block clusters: the cs CTAs of a cluster share one 128-row output
// block and split K; their f32 tiles are summed through distributed shared
// memory in cluster-rank order (deterministic), and the epilogue runs on the
// reduced rows.  X is bf16 rows; f32 residual rows normalised on the fly
// (RMSNorm from sum-of-squares partials); or bf16 rows of x * gamma written
// by the residual epilogue that produced x, loaded like plain bf16 rows, with
// the RMSNorm scale 1 / rms(x) of every token applied to the reduced
// accumulator (W (x * gamma) / rms(x) = W RMSNorm(x)).
// ---------------------------------------------------------------------------
enum GemmX { GX_BF16 = 0, GX_NORM = 1, GX_SCALED = 2 };
enum GemmEpi {
  GE_F32 = 0,    // y[t][n] = acc
  GE_QKV = 1,    // q/k RMSNorm + RoPE; q -> bf16 q[t], k / v appended to the paged cache
  GE_RESID = 2,  // y[t][n] += acc (residual stream), ss_out[n / 128][t] = sum of squares of the new rows;
                 // with xg_out also xg_out[t][n] = bf16(y[t][n] * xg_gamma[n]) (the next GX_SCALED input)
  GE_SILU = 3,   // row block r = [gate 64r..64r+63 | up 64r..64r+63]: h[t][64r + i] = bf16(silu(g) * u)
  GE_BIAS_SILU = 4,  // h[t][n] = bf16(silu(acc + bias[n]))
  GE_BIAS_BF16 = 5,  // y[t][n] = bf16-rounded (acc + bias[n]), stored as f32
};

// A weight matrix W [N][K] bf16 row-major with its TMA descriptor (box 64 x
// 128, SWIZZLE_128B).
struct Linear {
  const uint16_t *w = nullptr;
  int N = 0, K = 0;
  CUtensorMap tm;
};
// Encodes a 2-D bf16 TMA descriptor over rows x inner elements (row pitch
// row_bytes) with boxes of box_inner x box_rows, SWIZZLE_128B; false on error.
bool make_tmap_bf16(CUtensorMap *m, const void *base, uint64_t inner, uint64_t rows, uint64_t row_bytes,
                    uint32_t box_inner, uint32_t box_rows);
// General form: rank dims (innermost first), rank - 1 byte strides.
bool make_tmap(CUtensorMap *m, CUtensorMapDataType type, int rank, const void *base, const uint64_t *dims,
               const uint64_t *strides, const uint32_t *box, CUtensorMapSwizzle swizzle);

struct GemmArgs {
  CUtensorMap tw;      // weights W [N][K] (Linear::tm)
  CUtensorMap tx;      // GX_BF16 / GX_SCALED: X rows [rows][K], box 64 x 8*nt
  int N, K;
  int cs;              // cluster size = K splits (1, 2, 4 or 8)
  int nt;              // 8-token MMA tiles per CTA (1, 2, 4 or 8)
  const int *ntok;     // token count (device)
  int xmode;
  const uint16_t *xb;  // GX_BF16: X[t][ldx]
  const float *x;      // GX_NORM: row t is x[t * xrow_mul + xrow_add][0..K)
  int ldx, xrow_mul, xrow_add;
  const float *ss;     // GX_NORM / GX_SCALED: sum of squares of row r = sum_i ss[i * ss_ld + r], i < nss
                       // (GX_SCALED: row r = t * xrow_mul + xrow_add of token t)
  int nss, ss_ld;
  const float *gamma;  // GX_NORM: RMSNorm weight [K]
  float eps;
  int epi;
  float *y;            // GE_F32 output / GE_RESID residual, [t][ldy]
  int ldy;
  float *ss_out;       // GE_RESID: [N / 128][ss_ld]
  uint16_t *xg_out;    // GE_RESID, nullable: bf16 rows [t][ldy] of the new residual times xg_gamma
  const float *xg_gamma;
  uint16_t *h;         // GE_SILU / GE_BIAS_SILU: [t][ldh]
  int ldh;
  const float *bias;   // GE_BIAS_SILU / GE_BIAS_BF16: [N]
  const float *q_norm, *k_norm, *inv_freq;  // GE_QKV
  int nh, nkv;
  TokView tv;
  uint16_t *q;         // GE_QKV: [t][nh * 128]
  KVView kv;
  int layer;
  int *err;            // set (bitwise or) when a bounded wait gave up; nullable
};

// Cluster size and token tiles for an N x K GEMM over up to max_tok tokens
// (N % 128 == 0, K % 128 == 0); the caller fills X and the epilogue.
GemmArgs gemm_args(const Linear &W, const int *ntok, int max_tok);
void gemm(const GemmArgs &a, int max_tok, cudaStream_t st);

struct AttnArgs {
  const uint16_t *q;  // [t][nh * 128] bf16, normed and rotated
  KVView kv;
  int layer;
  TokView tv;
  int nh;
  int pw;         // minimum pages per work unit (more when a sequence would need > kAttnMaxUnits)
  int max_units;  // upper bound of units per (token, head): sizes the grid only
  float scale;
  AttnWork ws;
  uint16_t *out;
};

// Split-K flash-decoding over the paged cache for every token t < ntok:
// attends to positions [0, pos]; the token's own K/V are already appended.
// pw / max_units: see AttnArgs; max_tok <= kAttnMaxTok.
void attention(const uint16_t *q, KVView kv, int layer, TokView tv, int max_tok, int nh, int pw,
               int max_units, AttnWork ws, uint16_t *out, cudaStream_t st);

constexpr int kSampleMaxV = 4096;  // widest vocabulary the sampler handles

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
  const int64_t *suppress;     // slot s's list at suppress + s * suppress_ld (applied where sup_on[slot] != 0)
  int n_suppress;              // its length, or n_sup[s] when n_sup is set
  int suppress_ld;
  const int *n_sup;            // [slot] or null
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
  const double *u;             // nullable: [t] categorical draws in [0, 1) instead of the counter hash
  uint8_t *kept;               // nullable: [t][ldl] 1 where a token stays a candidate after suppress,
                               // top-k and top-p
};
// tail (nullable): the next input row of each token (RmsArgs over the same
// tokens), built and normalised by the sampler's CTA right after its sample
void sample(const SampleArgs &a, int max_tok, cudaStream_t st, const RmsArgs *tail = nullptr);

// ---------------------------------------------------------------------------
// A decode frame as a list of phases, each one kernel launch (captured once
// into a CUDA graph and replayed).
// ---------------------------------------------------------------------------
enum PhaseType { PH_NORM = 1, PH_GEMM = 2, PH_ATTN = 3, PH_SAMPLE = 4 };

struct Phase {
  int type;
  int max_tok;   // rows / tokens the phase spans (items beyond ntok exit)
  int has_tail;  // PH_SAMPLE: run `tail` (embed + norm of the next input) per token
  int pad;
  union {
    RmsArgs norm;
    GemmArgs gemm;
    AttnArgs attn;
    SampleArgs smp;
  };
  RmsArgs tail;
};
void run_phases(const Phase *phases, int n_phases, cudaStream_t st);

// out[i] = table[ids[i]] (device ids, i < n): rows of `width` bf16.
void gather_rows_bf16(const uint16_t *table, const int *ids, int n, int width, uint16_t *out, cudaStream_t st);
// out[s] = bf16-rounded P[text_row[s]] + (codec_emb[codec_id[s]], or when
// codec_id[s] < 0, X[x_row[s]]) (negative index: term absent), S rows of H
void seed_rows(const float *P, const uint16_t *codec_emb, const int *text_row, const int *codec_id, int S, int H,
               float *out, cudaStream_t st, const float *X = nullptr, const int *x_row = nullptr);
// X [1 + T][H]: row 0 = bf16(spk), row 1 + t = the bf16 group-order sum of
// frame t's code embeddings (codes [G][T]: group 0 from emb0, group g from
// embs[g - 1], device pointer array)
void clone_rows(const float *spk, const int64_t *codes, int G, int T, const uint16_t *emb0,
                const uint16_t *const *embs, int H, float *X, cudaStream_t st);

// Scatter dense bf16 K/V [layers][n_kv][len][hd] into the pages of `seq`.
void kv_import(const uint16_t *k, const uint16_t *v, int layers, int len, KVView kv, int seq,
               cudaStream_t st);

}  // namespace q3t

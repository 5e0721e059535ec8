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

// out[t] = bf16(rmsnorm(x[t*row_mul + row_add]) * gamma); optional f32 copy
// scattered to out_f32[slot[t]]; zero[t][0:zero_cols] = 0.
void rmsnorm(const float *x, int ldx, int row_mul, int row_add, const float *gamma,
             uint16_t *out, int ldo, int H, float eps, const int *ntok, int grid_rows,
             float *zero, int ldz, int zero_cols, float *out_f32, const int *slot,
             cudaStream_t st);

// Y[t][n] += sum_k W[n][k] * X[t][k] for t < ntok (split-K, f32 atomics).
// xmode 0: X bf16 [t][ldx]; xmode 1: X f32 gate|up [t][ldx], X = silu(g)*u.
void linear(const uint16_t *Wp, int N, int K, const void *X, int ldx, int xmode, float *Y,
            int ldy, const int *ntok, int max_tok, cudaStream_t st);

// q/k RMSNorm + rotate-half RoPE + bf16 q out + K/V append into pages.
void qkv_post(const float *qkv, int ldqkv, const float *q_norm, const float *k_norm,
              const float *inv_freq, float eps, int nh, int nkv, TokView tv, int max_tok,
              uint16_t *qout, KVView kv, int layer, cudaStream_t st);

// Split-K flash-decoding over the paged cache, one token per (t): attends to
// positions [0, pos]; fused=1 also does qkv_post for its own head group
// (valid only when every token of the batch belongs to a distinct sequence).
void attention(int fused, const float *qkv, int ldqkv, const float *q_norm, const float *k_norm,
               const float *inv_freq, float eps, const uint16_t *qin, KVView kv, int layer,
               TokView tv, int max_tok, int nh, int chunk, int max_split, AttnWork ws,
               uint16_t *out, cudaStream_t st);

// x[t] = sum_g emb_g[codes[slot[t]][g]] + extra[t]; records the frame's codes
// into hist[slot][frame[t]][:] when hist != null.
void embed_codes(const uint16_t *emb0, const uint16_t *const *embs, int G, int H,
                 const int64_t *codes, const int *slot, const float *const *extra,
                 const int *frame, int64_t *hist, int hist_frames, const int *ntok, int max_tok,
                 float *x, cudaStream_t st);

// Code-predictor prefill rows: x[2b] = hidden[slot[b]], x[2b+1] = emb0[codes[slot[b]][0]].
void pred_input0(const float *hidden, const uint16_t *emb0, const int64_t *codes, int G,
                 const int *slot, const int *ntok, int max_tok, int H, float *x, cudaStream_t st);
// x[b] = emb[codes[slot[b]][col]]
void pred_input(const uint16_t *emb, const int64_t *codes, int G, int col, const int *slot,
                const int *ntok, int max_tok, int H, float *x, cudaStream_t st);

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
  float *logits;
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
  int step_seed;
  int32_t *raw;                // [slot][max_frames][G] sampled tokens before forcing, or null
};
void sample(const SampleArgs &a, int max_tok, cudaStream_t st);

// Scatter dense bf16 K/V [layers][n_kv][len][hd] into the pages of `seq`.
void kv_import(const uint16_t *k, const uint16_t *v, int layers, int len, KVView kv, int seq,
               cudaStream_t st);

}  // namespace q3t

// Streamed small-batch decoder kernel (k_mk): one persistent cooperative
// launch runs a whole program of decoder stages (GEMVs and paged attention)
// for up to kMkMaxTok tokens.
//
// Why: at batch 1..4 a decoder layer is five dependent steps whose weights
// take ~5 us of HBM time, while a kernel boundary plus the dependent loads of
// a launch cost ~5 us each.  Here a producer warp per CTA streams every
// stage's weight slice (and the cached K/V pages of the attention stages)
// into a shared-memory ring with bulk async copies, running up to the ring's
// depth (~0.9 of a talker layer) ahead of the dependency chain; eight compute
// warps consume the ring stage by stage.
//
// Stages hand data to each other through tagged words: every value passed
// between stages is stored as 8 bytes {f32 value, tag} with one store, tag =
// (launch epoch << 10) | writing stage.  A consumer spins on the words it
// needs until their tags match, so a hop costs one L2 round trip and needs no
// fence, counter or grid barrier; 8-byte aligned stores and loads are
// single-copy atomic, so a matching tag implies its value.  Buffers are
// reused across stages only after every reader of the previous contents has
// provably finished (each stage reads the whole output of the stage before
// it), and the residual stream alternates between two buffers.
//
// Every wait is bounded: a timeout sets a bit in *err and later waits of the
// CTA are skipped, so a launch always ends; the last CTA to finish advances
// the epoch for the next launch.
#pragma once
#include "lm_kernels.cuh"

namespace q3t {

constexpr int kMkWarps = 15;                       // compute warps (+ producer = 4 warps per scheduler)
constexpr int kMkThreads = (kMkWarps + 1) * 32;    // + one producer warp
constexpr int kMkSlot = 32768;                     // ring slot bytes
constexpr int kMkSlots = 6;
constexpr int kMkMaxTok = 2;                       // tokens per launch
constexpr int kMkMaxK = 3072;                      // widest GEMV input
constexpr int kMkChunkPages = 4;                   // KV pages per ring slot (K 16 KB + V 16 KB)
constexpr int kMkMaxRes = 64;                      // residual rows per CTA kept in shared memory
constexpr int kMkMaxStages = 1024;                 // the tag keeps 10 bits of stage index
constexpr int kMkPartLd = 130;                     // tagged words per attention partial row: o[128], m, l

enum MkOp { MK_GEMV = 1, MK_ATTN = 2 };
// X sources: RMSNorm(x) * gamma of f32 rows; tagged f32 values that are
// bf16-exact (a bf16 activation).
enum MkXSrc { MKX_NORM = 0, MKX_TAGGED = 1 };
// Epilogues: plain f32 out; tagged f32 out; residual (tagged out = residual
// in + acc); SwiGLU pairs (tagged bf16-rounded silu(gate) * up).
enum MkEpi { MKE_F32 = 0, MKE_TAG = 1, MKE_RESID = 2, MKE_SILU = 3 };

// An f32 row buffer that is either plain (stage < 0, `f`) or tagged words
// written by stage `stage` of this launch (`w`).
struct MkIn {
  const float *f;
  const uint2 *w;
  int stage;
  int ld;
};

// y[t][n] = X[t] . W[n] over the CTA's row slice.  W is bf16 row-major
// [N][K]; with pairs = 1 its rows are gate/up interleaved per 64
// ([gate 64r..64r+63 ; up 64r..64r+63]) and the output is
// h[t][p] = bf16(silu(gate_p) * up_p) for the N / 2 pairs.
struct MkGemv {
  const uint16_t *w;
  int N, K, pairs;
  int xsrc;
  MkIn x;                  // MKX_NORM / MKX_TAGGED input rows
  const float *gamma;
  float eps;
  float *hid_out;          // MKX_NORM, nullable: CTA 0 also stores the f32 normed row t at hid_out[hid_slot[t] * K]
  const int *hid_slot;
  int epi;
  float *y;                // MKE_F32 output [t][ldy]
  uint2 *yt;               // MKE_TAG / MKE_RESID / MKE_SILU tagged output [t][ldy]
  int ldy;
  MkIn res;                // MKE_RESID: residual rows in
};

// Split-K flash-decoding GQA attention of every token over its paged keys
// [0, pos].  Inputs are the raw (pre-norm) q/k/v rows of the QKV GEMV
// (tagged, [t][ldq] = [q heads | k heads | v heads] x 128); q / k get the
// per-head RMSNorm and rotate-half RoPE here, each token's own k / v are
// appended to the cache by the unit that covers its position.  Units that
// cover part of a token's keys write (o, m, l) partials, which unit 0 of the
// (token, kv head) merges; the stage's output is the bf16-exact attention
// output rows (tagged).
struct MkAttn {
  const uint2 *qkv;
  int qkv_stage, ldq;
  const float *q_norm, *k_norm, *inv_freq;
  float eps, scale;
  KVView kv;
  int layer, nh;
  uint2 *part;             // [t][nkv][kAttnMaxUnits][2][kMkPartLd]
  uint2 *out;              // [t][ldo = nh * 128]
  int ldo;
};

struct alignas(16) MkStage {
  int op;
  MkGemv g;
  MkAttn a;
};

struct MkArgs {
  const MkStage *st;       // device array of n stages
  int n;
  TokView tv;              // tokens (ntok <= kMkMaxTok), sequences, positions
  unsigned *ctr;           // [2]: launch epoch (>= 1), finished CTAs (0 between launches)
  int *err;                // bit 8: a tagged-data wait gave up, bit 9: a ring wait gave up
  unsigned long long *trace;  // nullable: [grid][n][8] globaltimer ns per CTA and stage: inputs ready,
                              // X staged, first chunk landed, stage done; producer: stage reached,
                              // first chunk issued
  int polls;               // polls of a tagged-data wait before it gives up (<= 0: the default, ~0.25 s)
  const int *stall;        // nullable: each CTA first waits for *stall == 1, a word nothing sets, so the
                           // wait runs out (tests of the timeout path; null in production)
};

// Dynamic shared memory of k_mk.
size_t mk_smem_bytes();
// Sets the kernel's shared-memory limit; false if the device cannot host it.
bool mk_init_attributes();
// CTAs of one launch on `device`: SMs x co-resident CTAs (0 if it cannot run).
int mk_grid(int device);
// Cooperative launch of the program on `st` with `grid` CTAs.
void mk_launch(const MkArgs &a, int grid, cudaStream_t st);

}  // namespace q3t

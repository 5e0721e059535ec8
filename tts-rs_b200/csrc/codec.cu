// Speech-tokenizer decoder (codec/network/decoder.rs:250-278) for sm_100a.
//
// Activations are time-major [B][L][C].  Every convolution and linear is one
// implicit GEMM on the tensor cores (mma.sync m16n8k16, fp16 operands, f32
// accumulation): output row m = (sequence b, step tq) of one phase p; for tap
// j it reads input row tq + in_off + j * dil of the same sequence (zero
// outside [0, L_in)), i.e.
//   causal Conv1d k, dilation d  : taps k, in_off = -(k-1)d, 1 phase
//   ConvTranspose1d k = r, s = r : 1 tap, r phases, output row tq*r + p
//   ConvTranspose1d k = 2r, s = r with the both-side trim of r
//     (conv.rs:19-31)            : 2 taps {x[tq] * w[.,.,p+r], x[tq+1] * w[.,.,p]},
//                                  r phases, L_in - 1 steps per phase
// The epilogue fuses bias, LayerScale / ConvNeXt gamma, the residual add,
// and the activation that the NEXT layer applies to its input (SnakeBeta,
// GELU), so each SnakeBeta is evaluated once per element.  fp16 (10-bit
// mantissa) keeps the waveform well above the 40 dB SNR bar against the f32
// decode; the residual streams stay f32.
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>

#include "codec.cuh"
#include "common.cuh"
#include "umma.cuh"

namespace q3t {

// ---------------------------------------------------------------------------
// device helpers
// ---------------------------------------------------------------------------
Q3T_DEV void ldmatrix_x4(uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3, const void *p) {
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(p);
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(s));
}
Q3T_DEV void ldmatrix_x2(uint32_t &r0, uint32_t &r1, const void *p) {
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(p);
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];\n" : "=r"(r0), "=r"(r1) : "r"(s));
}
Q3T_DEV void mma_f16(float *c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// sin^2(y) in f32.  sin^2 has period pi, so y is reduced to r = y - k pi,
// k = rint(y / pi), with pi split into three floats (Cody-Waite reduction:
// k * 3.140625 and k * PI_B are exact for |k| < 4096), and sin r on
// [-pi/2, pi/2] is the __sinf intrinsic, whose documented absolute error on
// [-pi, pi] is 2^-21.41.  Max abs error of the square below 1e-6 for
// |y| <= 3000, far under the fp16 step of the activations it produces.
Q3T_DEV float sin_sq(float y) {
  const float k = rintf(y * 0.318309886183790672f);
  float r = fmaf(-k, 3.140625f, y);
  r = fmaf(-k, 9.675025939941406e-4f, r);
  r = fmaf(-k, 1.5099580252808664e-7f, r);
  const float sn = __sinf(r);
  return sn * sn;
}

// SnakeBeta x + sin^2(e^alpha x) / (e^beta + 1e-9) (activation.rs:16-37) with
// ea = e^alpha and ib = 1 / (e^beta + 1e-9) precomputed per channel.
Q3T_DEV float snake(float x, float ea, float ib) { return fmaf(sin_sq(x * ea), ib, x); }
Q3T_DEV float gelu_erf(float x) { return 0.5f * x * (1.f + erff(x * 0.70710678118654752f)); }

enum { ACT_NONE = 0, ACT_SNAKE = 1, ACT_GELU = 2 };

struct ConvArgs {
  const __half *X;  // [B][Lin][Cin]
  int Lin, Cin, B;
  const __half *W;  // [phases][taps][Cout][Cin]
  int Cout, taps;
  long long w_phase_stride;
  const float *bias;  // [Cout] or null
  int in_off, dil;
  int Lq;       // output steps per sequence per phase
  int ostride;  // output row = tq * ostride + phase
  int Lout;     // output rows per sequence
  float *Yf;    // f32 out [B][Lout][Cout] (nullable)
  const float *R;      // residual, same indexing as Yf (nullable; may alias Yf)
  const float *scale;  // per-channel multiplier applied before the residual
  __half *Yh;          // fp16 out of act(y) (nullable)
  int act;
  const float *act_a, *act_b;
};

constexpr int kBM = 128, kBK = 32, kLDS = kBK + 8, kStages = 3;

template <int BN>
__global__ void __launch_bounds__(256) k_conv(ConvArgs a) {
  extern __shared__ __align__(16) __half smem_h[];
  constexpr int WN = BN / 4, NT = WN / 8;
  __half *As = smem_h;
  __half *Bs = smem_h + kStages * kBM * kLDS;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int wm = warp >> 2, wn = warp & 3;
  const int m0 = blockIdx.x * kBM, n0 = blockIdx.y * BN, phase = blockIdx.z;
  const __half *W = a.W + (long long)phase * a.w_phase_stride;
  const int M = a.B * a.Lq;
  const int kcn = a.Cin / kBK;
  const int KT = a.taps * kcn;
  // this thread's two A rows (16 B chunk (tid & 3) of rows tid/4 and tid/4 + 64)
  int ab[2], atq[2];
  bool am[2];
#pragma unroll
  for (int i = 0; i < 2; i++) {
    const int m = m0 + (tid >> 2) + i * 64;
    am[i] = m < M;
    ab[i] = am[i] ? m / a.Lq : 0;
    atq[i] = am[i] ? m - ab[i] * a.Lq : 0;
  }
  auto load_stage = [&](int kt, int st) {
    const int tap = kt / kcn, c0 = (kt - tap * kcn) * kBK;
    const int col = (tid & 3) * 8;
#pragma unroll
    for (int i = 0; i < 2; i++) {
      const int r = (tid >> 2) + i * 64;
      const int in_row = atq[i] + a.in_off + tap * a.dil;
      const bool ok = am[i] && in_row >= 0 && in_row < a.Lin;
      const __half *src = ok ? a.X + ((size_t)ab[i] * a.Lin + in_row) * a.Cin + c0 + col : a.X;
      cp_async16(As + ((size_t)st * kBM + r) * kLDS + col, src, ok ? 16 : 0);
    }
    for (int idx = tid; idx < BN * 4; idx += 256) {
      const int n = idx >> 2, c = (idx & 3) * 8;
      const __half *src = W + ((size_t)(tap * a.Cout + n0 + n)) * a.Cin + c0 + c;
      cp_async16(Bs + ((size_t)st * BN + n) * kLDS + c, src, 16);
    }
  };
  float acc[4][NT][4];
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < NT; j++) acc[i][j][0] = acc[i][j][1] = acc[i][j][2] = acc[i][j][3] = 0.f;
#pragma unroll
  for (int s = 0; s < kStages - 1; s++) {
    if (s < KT) load_stage(s, s);
    cp_async_commit();
  }
  for (int kt = 0; kt < KT; kt++) {
    cp_async_wait<kStages - 2>();
    __syncthreads();
    const int nk = kt + kStages - 1;
    if (nk < KT) load_stage(nk, nk % kStages);
    cp_async_commit();
    const int st = kt % kStages;
    const __half *Ab = As + (size_t)st * kBM * kLDS;
    const __half *Bb = Bs + (size_t)st * BN * kLDS;
#pragma unroll
    for (int ks = 0; ks < 2; ks++) {
      uint32_t af[4][4];
#pragma unroll
      for (int mi = 0; mi < 4; mi++) {
        const __half *p = Ab + (wm * 64 + mi * 16 + (lane & 15)) * kLDS + ks * 16 + (lane >> 4) * 8;
        ldmatrix_x4(af[mi][0], af[mi][1], af[mi][2], af[mi][3], p);
      }
#pragma unroll
      for (int ni = 0; ni < NT; ni++) {
        uint32_t b0, b1;
        const __half *p = Bb + (wn * WN + ni * 8 + (lane & 7)) * kLDS + ks * 16 + ((lane >> 3) & 1) * 8;
        ldmatrix_x2(b0, b1, p);
#pragma unroll
        for (int mi = 0; mi < 4; mi++) mma_f16(acc[mi][ni], af[mi][0], af[mi][1], af[mi][2], af[mi][3], b0, b1);
      }
    }
  }
  cp_async_wait<0>();
  // epilogue
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int mi = 0; mi < 4; mi++)
#pragma unroll
    for (int hh = 0; hh < 2; hh++) {
      const int m = m0 + wm * 64 + mi * 16 + g + hh * 8;
      if (m >= M) continue;
      const int b = m / a.Lq, tq = m - b * a.Lq;
      const size_t orow = (size_t)b * a.Lout + (size_t)tq * a.ostride + phase;
#pragma unroll
      for (int ni = 0; ni < NT; ni++) {
        const int n = n0 + wn * WN + ni * 8 + 2 * t;
        float v0 = acc[mi][ni][hh * 2], v1 = acc[mi][ni][hh * 2 + 1];
        if (a.bias) {
          v0 += a.bias[n];
          v1 += a.bias[n + 1];
        }
        if (a.scale) {
          v0 *= a.scale[n];
          v1 *= a.scale[n + 1];
        }
        const size_t e = orow * a.Cout + n;
        if (a.R) {
          const float2 r = *reinterpret_cast<const float2 *>(a.R + e);
          v0 += r.x;
          v1 += r.y;
        }
        if (a.Yf) *reinterpret_cast<float2 *>(a.Yf + e) = make_float2(v0, v1);
        if (a.Yh) {
          float h0 = v0, h1 = v1;
          if (a.act == ACT_SNAKE) {
            h0 = snake(v0, a.act_a[n], a.act_b[n]);
            h1 = snake(v1, a.act_a[n + 1], a.act_b[n + 1]);
          } else if (a.act == ACT_GELU) {
            h0 = gelu_erf(v0);
            h1 = gelu_erf(v1);
          }
          *reinterpret_cast<__half2 *>(a.Yh + e) = __floats2half2_rn(h0, h1);
        }
      }
    }
}

static size_t conv_smem(int BN) { return (size_t)kStages * (kBM + BN) * kLDS * sizeof(__half); }

// ---------------------------------------------------------------------------
// The same convolution on the 5th-generation tensor cores.  A CTA computes a
// tile of 128 output steps of one sequence and phase x N output channels:
//   warp 0 lane 0  streams, per K step (tap j, ACH input channels), the
//                  im2col tile X[b][tq0 + in_off + j*dil + 0..127][c0..c0+ACH)
//                  (a 3-D TMA box: rows outside [0, Lin) read zeros, which is
//                  the causal padding) and the weight tile W[phase][j][n0..
//                  n0+N)[c0..c0+ACH) into a ring of S stages;
//   warp 1 lane 0  issues tcgen05.mma (M = 128, N, K = 16) into a TMEM
//                  accumulator and releases each stage with tcgen05.commit;
//   warps 0..3     read the accumulator back (thread = output step, 16
//                  channels per tcgen05.ld) into an f32 tile in shared memory;
//   all 8 warps    then sweep the tile row-major (coalesced) through the
//                  k_conv epilogue.
// Operands are K-major with SWIZZLE_128B (ACH = 64) or SWIZZLE_64B (ACH = 32)
// atoms.  Every mbarrier wait is bounded; a timeout sets a bit in *err.
//
// FUSE = 1 runs a whole residual unit (wave.rs:37-56) when the CTA owns all
// N = C channels:  y = x + conv1(snake2(conv7_d(h) + b7)) + b1.  After the
// k7 accumulator is complete, all 8 warps read it back, apply b7 and SnakeBeta
// act2 and store the fp16 result, swizzled exactly as TMA would have stored
// it, into the A halves of the next Cin / ACH ring stages; the producer
// streams the k1 weight chunks into the B halves of the same stages; the MMA
// warp runs the k1 GEMM into the same TMEM columns, and the epilogue above
// finishes it (b1, residual, next SnakeBeta).  The intermediate activation
// never leaves shared memory.
// ---------------------------------------------------------------------------
struct ConvTc {
  CUtensorMap tx;  // X [B][Lin][Cin], box ACH x 128 x 1
  CUtensorMap tw;  // W [phases * taps * Cout][Cin], box ACH x N
  CUtensorMap tw1; // FUSE: k1 weights W1 [Cout][Cout], box ACH x N
  ConvArgs a;      // FUSE: a.bias is b1 (the k1 bias); the epilogue fields describe the unit's output
  const float *mid_bias;  // FUSE: b7
  const float *mid_a, *mid_b;  // FUSE: act2 SnakeBeta (e^alpha, 1 / (e^beta + 1e-9))
  int tiles;       // 128-step tiles per sequence
  int *err;
};

// Byte offset of 16-byte chunk j of row r in a K-major tile of ACH fp16 per
// row, SWIZZLE_128B (ACH = 64) or SWIZZLE_64B (ACH = 32), as TMA stores it
// into a 1024-byte-aligned buffer.
template <int ACH>
Q3T_DEV uint32_t swz_off(int r, int j) {
  return ACH == 64 ? (uint32_t)(r * 128 + ((j ^ (r & 7)) << 4)) : (uint32_t)(r * 64 + ((j ^ ((r >> 1) & 3)) << 4));
}

// Epilogue of one output tile: the f32 accumulator tile [128 steps][N + 4]
// in shared memory is swept row-major (NTH threads, consecutive threads on
// consecutive 4-channel groups of a row, so global accesses coalesce) through
// bias, scale, residual, the f32 store and act() -> fp16.
template <int N, int NTH>
Q3T_DEV void conv_sweep(const ConvArgs &a, const float *tile, int b, int tq0, int n0, int phase, int tid) {
  constexpr int TP = N + 4, G4 = N / 4, UN = 4;
  const int rows = min(128, a.Lq - tq0);
  const int total = rows * G4;
  const size_t base0 = (size_t)b * a.Lout + phase;
  for (int f0 = tid; f0 < total; f0 += NTH * UN) {
    float4 v[UN], r[UN];
    size_t e[UN];
    int nn[UN];
#pragma unroll
    for (int u = 0; u < UN; u++) {
      const int f = f0 + NTH * u;
      const int ff = f < total ? f : 0, row = ff / G4, c4 = ff - row * G4;
      nn[u] = f < total ? n0 + 4 * c4 : -1;
      v[u] = *reinterpret_cast<const float4 *>(tile + row * TP + 4 * c4);
      e[u] = (base0 + (size_t)(tq0 + row) * a.ostride) * a.Cout + n0 + 4 * c4;
      if (nn[u] >= 0 && a.R) r[u] = *reinterpret_cast<const float4 *>(a.R + e[u]);
    }
#pragma unroll
    for (int u = 0; u < UN; u++) {
      const int n = nn[u];
      if (n < 0) continue;
      float y[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
      if (a.bias) {
        const float4 bb = *reinterpret_cast<const float4 *>(a.bias + n);
        y[0] += bb.x;
        y[1] += bb.y;
        y[2] += bb.z;
        y[3] += bb.w;
      }
      if (a.scale) {
        const float4 sc = *reinterpret_cast<const float4 *>(a.scale + n);
        y[0] *= sc.x;
        y[1] *= sc.y;
        y[2] *= sc.z;
        y[3] *= sc.w;
      }
      if (a.R) {
        y[0] += r[u].x;
        y[1] += r[u].y;
        y[2] += r[u].z;
        y[3] += r[u].w;
      }
      if (a.Yf) *reinterpret_cast<float4 *>(a.Yf + e[u]) = make_float4(y[0], y[1], y[2], y[3]);
      if (a.Yh) {
        float h[4] = {y[0], y[1], y[2], y[3]};
        if (a.act == ACT_SNAKE) {
          const float4 ea = *reinterpret_cast<const float4 *>(a.act_a + n);
          const float4 ib = *reinterpret_cast<const float4 *>(a.act_b + n);
          h[0] = snake(y[0], ea.x, ib.x);
          h[1] = snake(y[1], ea.y, ib.y);
          h[2] = snake(y[2], ea.z, ib.z);
          h[3] = snake(y[3], ea.w, ib.w);
        } else if (a.act == ACT_GELU) {
#pragma unroll
          for (int j = 0; j < 4; j++) h[j] = gelu_erf(y[j]);
        }
        __half2 p[2] = {__floats2half2_rn(h[0], h[1]), __floats2half2_rn(h[2], h[3])};
        *reinterpret_cast<uint2 *>(a.Yh + e[u]) = *reinterpret_cast<const uint2 *>(p);
      }
    }
  }
}

// conv_sweep for the persistent kernel: thread tid owns the 4-channel column
// group tid % (N / 4) of rows tid / (N / 4) + k * RP (RP = NTH / (N / 4) rows
// per pass, consecutive threads still cover a row contiguously), so its
// per-channel parameters load once per tile and UN rows' residual loads are
// in flight together.
template <int N, int NTH>
Q3T_DEV void conv_sweep_cols(const ConvArgs &a, const float *tile, int b, int tq0, int n0, int phase, int tid) {
  constexpr int TP = N + 4, G4 = N / 4, RP = NTH / G4, UN = 4;
  const int c4 = tid % G4, r0 = tid / G4;
  if (r0 >= RP) return;
  const int n = n0 + 4 * c4;
  const float4 bb = a.bias ? *reinterpret_cast<const float4 *>(a.bias + n) : make_float4(0.f, 0.f, 0.f, 0.f);
  const float4 sc = a.scale ? *reinterpret_cast<const float4 *>(a.scale + n) : make_float4(1.f, 1.f, 1.f, 1.f);
  float4 ea = make_float4(0.f, 0.f, 0.f, 0.f), ib = ea;
  if (a.act == ACT_SNAKE) {
    ea = *reinterpret_cast<const float4 *>(a.act_a + n);
    ib = *reinterpret_cast<const float4 *>(a.act_b + n);
  }
  const int rows = min(128, a.Lq - tq0);
  const size_t rstride = (size_t)a.ostride * a.Cout;
  const size_t e0 = (((size_t)b * a.Lout + phase) + (size_t)tq0 * a.ostride) * a.Cout + n;
  for (int row0 = r0; row0 < rows; row0 += RP * UN) {
    float4 v[UN], r[UN];
#pragma unroll
    for (int u = 0; u < UN; u++) {
      const int row = row0 + RP * u;
      if (row < rows) {
        v[u] = *reinterpret_cast<const float4 *>(tile + row * TP + 4 * c4);
        if (a.R) r[u] = *reinterpret_cast<const float4 *>(a.R + e0 + row * rstride);
      }
    }
#pragma unroll
    for (int u = 0; u < UN; u++) {
      const int row = row0 + RP * u;
      if (row >= rows) break;
      const size_t e = e0 + row * rstride;
      float y[4] = {(v[u].x + bb.x) * sc.x, (v[u].y + bb.y) * sc.y, (v[u].z + bb.z) * sc.z, (v[u].w + bb.w) * sc.w};
      if (a.R) {
        y[0] += r[u].x;
        y[1] += r[u].y;
        y[2] += r[u].z;
        y[3] += r[u].w;
      }
      if (a.Yf) *reinterpret_cast<float4 *>(a.Yf + e) = make_float4(y[0], y[1], y[2], y[3]);
      if (a.Yh) {
        float h[4] = {y[0], y[1], y[2], y[3]};
        if (a.act == ACT_SNAKE) {
          h[0] = snake(y[0], ea.x, ib.x);
          h[1] = snake(y[1], ea.y, ib.y);
          h[2] = snake(y[2], ea.z, ib.z);
          h[3] = snake(y[3], ea.w, ib.w);
        } else if (a.act == ACT_GELU) {
#pragma unroll
          for (int j = 0; j < 4; j++) h[j] = gelu_erf(y[j]);
        }
        __half2 hp[2] = {__floats2half2_rn(h[0], h[1]), __floats2half2_rn(h[2], h[3])};
        *reinterpret_cast<uint2 *>(a.Yh + e) = *reinterpret_cast<const uint2 *>(hp);
      }
    }
  }
}

template <int N, int ACH, int S>
struct ConvTcSmem {
  static constexpr int kA = 128 * ACH * 2, kB = N * ACH * 2, kStage = kA + kB;
  static constexpr size_t kBytes = (size_t)S * kStage + (2 * S + 2) * 8 + 1024;
};

template <int N, int ACH, int S, int FUSE>
__global__ void __launch_bounds__(256) k_conv_tc(const __grid_constant__ ConvTc c) {
  using L = ConvTcSmem<N, ACH, S>;
  static_assert(!FUSE || N / ACH <= S, "the fused k1 GEMM needs one ring stage per input chunk");
  constexpr uint32_t kCols = N <= 128 ? 128 : 256;
  extern __shared__ unsigned char csm_raw[];
  unsigned char *sm = csm_raw + ((1024 - (smem_addr(csm_raw) & 1023)) & 1023);
  uint64_t *full = reinterpret_cast<uint64_t *>(sm + S * L::kStage), *empty = full + S, *accb = empty + S;
  uint32_t *tslot = reinterpret_cast<uint32_t *>(accb + 1);
  const ConvArgs &a = c.a;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x / c.tiles, tq0 = (blockIdx.x - b * c.tiles) * 128;
  const int n0 = blockIdx.y * N, phase = blockIdx.z;
  const int kc = a.Cin / ACH, KS = a.taps * kc;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accb, 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(tslot, kCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  uint32_t err = 0;
  if (warp == 0 && lane == 0) {  // TMA producer
    for (int ks = 0; ks < KS; ks++) {
      const int s = ks % S, i = ks / S;
      if (i > 0 && !mbar_wait(&empty[s], (i - 1) & 1)) {
        err |= 1u;
        break;
      }
      const int tap = ks / kc, c0 = (ks - tap * kc) * ACH;
      unsigned char *st = sm + s * L::kStage;
      mbar_expect_tx(&full[s], L::kStage);
      tma_load_3d(st, &c.tx, c0, tq0 + a.in_off + tap * a.dil, b, &full[s]);
      tma_load_2d(st + L::kA, &c.tw, c0, (phase * a.taps + tap) * a.Cout + n0, &full[s]);
    }
    if (FUSE && !err) {  // k1 weight chunks into the B halves of the next stages
      for (int ks = KS; ks < KS + N / ACH; ks++) {
        const int s = ks % S, i = ks / S;
        if (i > 0 && !mbar_wait(&empty[s], (i - 1) & 1)) {
          err |= 1u;
          break;
        }
        mbar_expect_tx(&full[s], L::kB);
        tma_load_2d(sm + s * L::kStage + L::kA, &c.tw1, (ks - KS) * ACH, 0, &full[s]);
      }
    }
  } else if (warp == 1 && lane == 0) {  // MMA issuer
    constexpr uint32_t idesc = umma_idesc_f16(128, N);
    for (int ks = 0; ks < KS; ks++) {
      const int s = ks % S;
      if (!mbar_wait(&full[s], (ks / S) & 1)) {
        err |= 2u;
        break;
      }
      tc_fence_after();
      const unsigned char *st = sm + s * L::kStage;
#pragma unroll
      for (int kk = 0; kk < ACH / 16; kk++) {
        const uint64_t ad = ACH == 64 ? sw128_desc(st + kk * 32) : sw64_desc(st + kk * 32);
        const uint64_t bd = ACH == 64 ? sw128_desc(st + L::kA + kk * 32) : sw64_desc(st + L::kA + kk * 32);
        umma_kf16(tmem, ad, bd, idesc, (ks | kk) != 0 ? 1u : 0u);
      }
      umma_commit(&empty[s]);
    }
    umma_commit(accb);
    if (!FUSE && !mbar_wait(accb, 0)) err |= 4u;  // the other threads block in the barrier below, not polling
  }
  if (FUSE) {
    // act2(acc + b7) -> fp16 A operand of the k1 GEMM, chunk q of ACH
    // channels in the A half of ring stage (KS + q) % S
    if (!mbar_wait(accb, 0)) err |= 4u;
    tc_fence_after();
    __syncwarp();  // lane 0 of warps 0 / 1 comes from its producer / MMA loop; tcgen05.ld is warp-aligned
    const int r = 32 * (warp & 3) + lane;
    const uint32_t trow = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
    constexpr int G = N / 16;
#pragma unroll 1
    for (int g = (warp >> 2) * (G / 2); g < ((warp >> 2) + 1) * (G / 2); g++) {
      float v[16];
      tmem_ld16(trow + 16 * g, v);
      const int col = 16 * g, q = col / ACH, j0 = (col - q * ACH) / 8;
      unsigned char *dst = sm + ((KS + q) % S) * L::kStage;
      uint32_t h[8];
#pragma unroll
      for (int e = 0; e < 16; e += 2) {
        const int n = col + e;
        const float y0 = snake(v[e] + c.mid_bias[n], c.mid_a[n], c.mid_b[n]);
        const float y1 = snake(v[e + 1] + c.mid_bias[n + 1], c.mid_a[n + 1], c.mid_b[n + 1]);
        const __half2 p = __floats2half2_rn(y0, y1);
        h[e / 2] = *reinterpret_cast<const uint32_t *>(&p);
      }
      *reinterpret_cast<uint4 *>(dst + swz_off<ACH>(r, j0)) = make_uint4(h[0], h[1], h[2], h[3]);
      *reinterpret_cast<uint4 *>(dst + swz_off<ACH>(r, j0 + 1)) = make_uint4(h[4], h[5], h[6], h[7]);
    }
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    if (warp == 1 && lane == 0) {
      tc_fence_after();
      constexpr uint32_t idesc = umma_idesc_f16(128, N);
      for (int ks = KS; ks < KS + N / ACH && !err; ks++) {
        const int s = ks % S;
        if (!mbar_wait(&full[s], (ks / S) & 1)) {
          err |= 2u;
          break;
        }
        tc_fence_after();
        const unsigned char *st = sm + s * L::kStage;
#pragma unroll
        for (int kk = 0; kk < ACH / 16; kk++) {
          const uint64_t ad = ACH == 64 ? sw128_desc(st + kk * 32) : sw64_desc(st + kk * 32);
          const uint64_t bd = ACH == 64 ? sw128_desc(st + L::kA + kk * 32) : sw64_desc(st + L::kA + kk * 32);
          umma_kf16(tmem, ad, bd, idesc, (ks > KS || kk > 0) ? 1u : 0u);
        }
      }
      umma_commit(accb);
      if (!mbar_wait(accb, 1)) err |= 4u;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // accumulator -> f32 tile [128 steps][N + 4] over the (drained) stage ring
  constexpr int TP = N + 4;
  float *tile = reinterpret_cast<float *>(sm);
  if (warp < 4) {
    const uint32_t trow = tmem + ((uint32_t)(32 * warp) << 16);
    float *dst = tile + (32 * warp + lane) * TP;
#pragma unroll 1
    for (int cc = 0; cc < N; cc += 16) {
      float v[16];
      tmem_ld16(trow + cc, v);
#pragma unroll
      for (int j = 0; j < 16; j++) dst[cc + j] = v[j];
    }
  }
  __syncthreads();
  conv_sweep<N, 256>(a, tile, b, tq0, n0, phase, threadIdx.x);
  if (err && c.err) atomicOr(c.err, (int)err);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kCols);
}

// Device word for the bounded-wait timeouts of k_conv_tc / k_conv_pt.  Each
// decode path owns its own word (the allocating decode one per call, the
// static decode one inside its static array, a streaming batch one per
// batch), zeroes it on its stream before its kernels and reads it back on the
// same stream after them, so decodes that run at the same time on one device
// never see or clear each other's timeouts.  The word of the decode being
// enqueued by this thread is set by ConvErrScope.
static thread_local int *t_conv_err = nullptr;

struct ConvErrScope {
  int *prev;
  explicit ConvErrScope(int *w) : prev(t_conv_err) { t_conv_err = w; }
  ~ConvErrScope() { t_conv_err = prev; }
};

static int *conv_err_word() {
  if (!t_conv_err) FAIL(Q3T_INVALID_INPUT, "internal: codec convolution enqueued without a timeout word");
  return t_conv_err;
}

// True the first time it is called for the current device with this mask
// (kernel attributes are per device).
static bool first_on_device(uint64_t &mask) {
  int dev = 0;
  CK(cudaGetDevice(&dev));
  const uint64_t bit = 1ull << (dev & 63);
  if (mask & bit) return false;
  mask |= bit;
  return true;
}

// Raises Q3T_DEVICE_TIMEOUT if the timeout word read back after a decode
// (host copy, taken on the decode's stream after its kernels) is set.
static void conv_check_err(int e, const char *what) {
  if (e) FAIL(Q3T_DEVICE_TIMEOUT, "%s: a bounded device wait of a convolution gave up (code %#x)", what, e);
}

// The fused residual unit's extra operands (FUSE = 1).
struct ConvFuse {
  const __half *W1;  // [C][C]
  const float *mid_bias, *mid_a, *mid_b;
};

template <int N, int ACH, int S, int FUSE>
static void conv_tc_launch(const ConvArgs &a, int phases, cudaStream_t st, const ConvFuse *fu = nullptr) {
  using L = ConvTcSmem<N, ACH, S>;
  static uint64_t attr = 0;
  if (first_on_device(attr))
    CK(cudaFuncSetAttribute(k_conv_tc<N, ACH, S, FUSE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                            (int)L::kBytes));
  ConvTc c;
  memset(&c, 0, sizeof c);
  const CUtensorMapSwizzle sw = ACH == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  if (FUSE) {
    if (!fu || a.Cout != N || a.Cin != N || phases != 1)
      FAIL(Q3T_INVALID_INPUT, "codec fused residual unit: %d -> %d channels, %d phases (%d -> %d, 1 expected)",
           a.Cin, a.Cout, phases, N, N);
    const uint64_t dims[2] = {(uint64_t)N, (uint64_t)N};
    const uint64_t strides[1] = {(uint64_t)N * 2};
    const uint32_t box[2] = {(uint32_t)ACH, (uint32_t)N};
    if (!make_tmap(&c.tw1, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, fu->W1, dims, strides, box, sw))
      FAIL(Q3T_CUDA_ERROR, "codec conv: TMA descriptor of the k1 weights failed");
    c.mid_bias = fu->mid_bias;
    c.mid_a = fu->mid_a;
    c.mid_b = fu->mid_b;
  }
  {
    const uint64_t dims[3] = {(uint64_t)a.Cin, (uint64_t)a.Lin, (uint64_t)a.B};
    const uint64_t strides[2] = {(uint64_t)a.Cin * 2, (uint64_t)a.Lin * a.Cin * 2};
    const uint32_t box[3] = {(uint32_t)ACH, 128, 1};
    if (!make_tmap(&c.tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, a.X, dims, strides, box, sw))
      FAIL(Q3T_CUDA_ERROR, "codec conv: TMA descriptor of the input failed");
  }
  {
    const uint64_t dims[2] = {(uint64_t)a.Cin, (uint64_t)phases * a.taps * a.Cout};
    const uint64_t strides[1] = {(uint64_t)a.Cin * 2};
    const uint32_t box[2] = {(uint32_t)ACH, (uint32_t)N};
    if (!make_tmap(&c.tw, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a.W, dims, strides, box, sw))
      FAIL(Q3T_CUDA_ERROR, "codec conv: TMA descriptor of the weights failed");
  }
  c.a = a;
  c.tiles = (a.Lq + 127) / 128;
  c.err = conv_err_word();
  const dim3 grid((unsigned)(a.B * c.tiles), a.Cout / N, phases);
  k_conv_tc<N, ACH, S, FUSE><<<grid, 256, L::kBytes, st>>>(c);
}

// ---------------------------------------------------------------------------
// Persistent, warp-specialised form of k_conv_tc (and of its fused residual
// unit).  One CTA per SM walks the output tiles t = blockIdx.x + i * gridDim.x
// (128 steps x N channels of one sequence and phase; channel blocks vary
// fastest, then phases, so neighbouring tiles share their input rows in L2):
//   warp 0 lane 0   TMA producer: im2col input and weight tiles into a ring
//                   of S stages, running ahead across tile boundaries;
//   warp 1 lane 0   MMA issuer: tile i into TMEM accumulator i & 1 (columns
//                   128 (i & 1) ..), released by the epilogue, so tile i + 1's
//                   MMAs run while tile i's epilogue drains;
//   warps 2..17     epilogue: warp w reads TMEM lanes 32 (w & 3) .. + 31 (its
//                   row quadrant) and column quarter (w - 2) >> 2 into an f32
//                   staging tile, then all sixteen sweep it row-major through
//                   conv_sweep.
// FUSE = 1 (residual unit, N = C): the k7 accumulator i is turned into the k1
// GEMM's A operand (act2(acc + b7), fp16, swizzled as TMA would store it) in
// its own tile; the k1 weights stay resident; the MMA warp issues tile i's k1
// GEMM into a third accumulator (columns 256 ..) after tile i + 1's k7 MMAs,
// and the epilogue drains it (b1, residual, next SnakeBeta) before it builds
// tile i + 1's A operand.  Every mbarrier wait is bounded; after a timeout a
// thread skips its remaining waits (the loops keep their trip counts, so
// every named barrier is still reached) and the kernel reports *err.
// ---------------------------------------------------------------------------
constexpr int kPtEpiWarps = 16, kPtThreads = (2 + kPtEpiWarps) * 32;

struct ConvPt {
  CUtensorMap tx, tw, tw1;  // as ConvTc
  ConvArgs a;
  const float *mid_bias, *mid_a, *mid_b;
  int tiles;                // 128-step tiles per sequence
  int nb, phases, total;    // channel blocks, phases, tiles of the launch
  int *err;
};

template <int N, int ACH, int S, int FUSE>
struct ConvPtSmem {
  static constexpr int NS = N > 128 ? N / 2 : N;  // columns drained per staging pass
  static constexpr int kA = 128 * ACH * 2, kB = N * ACH * 2, kStage = kA + kB;
  static constexpr int kStg = 128 * (NS + 4) * 4;
  static constexpr int kA2 = FUSE ? 128 * N * 2 : 0;
  static constexpr int kW1 = FUSE ? N * N * 2 : 0;
  static constexpr int kPar = FUSE ? 3 * N * 4 : 0;
  static constexpr int oStg = S * kStage, oA2 = oStg + kStg, oW1 = oA2 + kA2, oPar = oW1 + kW1, oBar = oPar + kPar;
  static constexpr int kBars = 2 * S + 8;
  static constexpr size_t kBytes = (size_t)oBar + kBars * 8 + 16 + 1024;
  static_assert(kStage % 1024 == 0 && kStg % 1024 == 0 && kA2 % 1024 == 0 && kW1 % 1024 == 0, "1024-byte operands");
  static_assert(kBytes <= 232448, "shared memory per CTA");
};

Q3T_DEV void bar_epi() { asm volatile("bar.sync 1, %0;" ::"n"(kPtEpiWarps * 32) : "memory"); }
Q3T_DEV void mbar_arrive1(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

struct PtTile {
  int b, tq0, n0, phase;
};
Q3T_DEV PtTile pt_tile(const ConvPt &c, int t, int N) {
  PtTile p;
  const int nbk = t % c.nb, u = t / c.nb;
  p.phase = u % c.phases;
  const int mt = u / c.phases;
  p.b = mt / c.tiles;
  p.tq0 = (mt - p.b * c.tiles) * 128;
  p.n0 = nbk * N;
  return p;
}

template <int N, int ACH, int S, int FUSE>
__global__ void __launch_bounds__(kPtThreads, 1) k_conv_pt(const __grid_constant__ ConvPt c) {
  using L = ConvPtSmem<N, ACH, S, FUSE>;
  constexpr int NS = L::NS;
  static_assert(N <= 256 && NS % 32 == 0 && (!FUSE || N <= 128), "accumulator / staging shapes");
  // accumulators: tile i in columns kAccStride * (i & 1) .., the fused k1 GEMM in 256 ..
  constexpr uint32_t kAccStride = N > 128 ? 256 : 128;
  constexpr uint32_t kCols = (FUSE || N > 128) ? 512 : 256, kAcc2 = 256;
  extern __shared__ unsigned char csm_raw[];
  unsigned char *sm = csm_raw + ((1024 - (smem_addr(csm_raw) & 1023)) & 1023);
  uint64_t *full = reinterpret_cast<uint64_t *>(sm + L::oBar), *empty = full + S;
  uint64_t *accf = empty + S, *acce = accf + 2, *a2f = acce + 2, *acc2f = a2f + 1, *w1f = acc2f + 1, *fin = w1f + 1;
  uint32_t *tslot = reinterpret_cast<uint32_t *>(fin + 1);
  float *stg = reinterpret_cast<float *>(sm + L::oStg);
  unsigned char *a2 = sm + L::oA2, *w1 = sm + L::oW1;
  float *par = reinterpret_cast<float *>(sm + L::oPar);
  const ConvArgs &a = c.a;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kc = a.Cin / ACH, KS = a.taps * kc;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&accf[i], 1);
      mbar_init(&acce[i], kPtEpiWarps);
    }
    mbar_init(a2f, kPtEpiWarps);
    mbar_init(acc2f, 1);
    mbar_init(w1f, 1);
    mbar_init(fin, 1);
    fence_mbar_init();
  }
  if (FUSE)
    for (int i = threadIdx.x; i < N; i += blockDim.x) {
      par[i] = c.mid_bias[i];
      par[N + i] = c.mid_a[i];
      par[2 * N + i] = c.mid_b[i];
    }
  if (warp == 0) tmem_alloc(tslot, kCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  uint32_t err = 0;
  if (warp == 0) {
    if (lane == 0) {  // TMA producer
      if (FUSE) {
        mbar_expect_tx(w1f, L::kW1);
        for (int q = 0; q < N / ACH; q++) tma_load_2d(w1 + q * L::kB, &c.tw1, q * ACH, 0, w1f);
      }
      int ks = 0;
      for (int t = blockIdx.x; t < c.total && !err; t += gridDim.x) {
        const PtTile p = pt_tile(c, t, N);
        for (int tap = 0; tap < a.taps && !err; tap++) {
          const int row = p.tq0 + a.in_off + tap * a.dil, wrow = (p.phase * a.taps + tap) * a.Cout + p.n0;
          for (int c0 = 0; c0 < kc * ACH; c0 += ACH, ks++) {
            const int s = ks % S, i = ks / S;
            if (i > 0 && !mbar_wait(&empty[s], (i - 1) & 1)) {
              err |= 1u;
              break;
            }
            unsigned char *st = sm + s * L::kStage;
            mbar_expect_tx(&full[s], L::kStage);
            tma_load_3d(st, &c.tx, c0, row, p.b, &full[s]);
            tma_load_2d(st + L::kA, &c.tw, c0, wrow, &full[s]);
          }
        }
      }
      // the copies still in flight (none unless a wait above gave up) land before the CTA ends
      for (int j = ks - 1; j >= 0 && j >= ks - S; j--)
        if (!mbar_wait(&full[j % S], (j / S) & 1)) err |= 1u;
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      constexpr uint32_t idesc = umma_idesc_f16(128, N);
      if (FUSE && !mbar_wait(w1f, 0)) err |= 8u;
      // operand descriptors: the start-address field is (address >> 4) in
      // bits 0..13, so stepping 32 bytes along K adds 2 and a stage adds
      // kStage >> 4 (shared addresses stay below 256 KB: no carry)
      const uint64_t da0 = ACH == 64 ? sw128_desc(sm) : sw64_desc(sm);
      const uint64_t db0 = ACH == 64 ? sw128_desc(sm + L::kA) : sw64_desc(sm + L::kA);
      auto mma2 = [&](int j) {  // k1 GEMM of tile j: A2 x W1 -> accumulator 2
        if (!err && !mbar_wait(a2f, j & 1)) err |= 16u;
        tc_fence_after();
        if (!err) {
          const uint64_t a2d = ACH == 64 ? sw128_desc(a2) : sw64_desc(a2);
          const uint64_t w1d = ACH == 64 ? sw128_desc(w1) : sw64_desc(w1);
#pragma unroll
          for (int q = 0; q < N / ACH; q++)
#pragma unroll
            for (int kk = 0; kk < ACH / 16; kk++)
              umma_kf16(tmem + kAcc2, a2d + (uint64_t)((q * L::kA) >> 4) + 2 * kk,
                        w1d + (uint64_t)((q * L::kB) >> 4) + 2 * kk, idesc, (q | kk) != 0 ? 1u : 0u);
        }
        umma_commit(acc2f);
      };
      int ks = 0, it = 0;
      for (int t = blockIdx.x; t < c.total; t += gridDim.x, it++) {
        const int buf = it & 1;
        if (!err && it >= 2 && !mbar_wait(&acce[buf], ((it >> 1) - 1) & 1)) err |= 4u;
        tc_fence_after();
        const uint32_t d = tmem + kAccStride * buf;
        for (int k = 0; k < KS && !err; k++, ks++) {
          const int s = ks % S;
          if (!mbar_wait(&full[s], (ks / S) & 1)) {
            err |= 2u;
            break;
          }
          tc_fence_after();
          const uint64_t so = (uint64_t)((s * L::kStage) >> 4);
#pragma unroll
          for (int kk = 0; kk < ACH / 16; kk++)
            umma_kf16(d, da0 + so + 2 * kk, db0 + so + 2 * kk, idesc, (k | kk) != 0 ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        umma_commit(&accf[buf]);
        if (FUSE && it >= 1) mma2(it - 1);
      }
      if (FUSE && it >= 1) mma2(it - 1);
      umma_commit(fin);  // every MMA issued has completed before TMEM is freed
      if (!mbar_wait(fin, 0)) err |= 4u;
    }
  } else {  // epilogue warps
    const int ew = warp - 2, quad = warp & 3, part = ew >> 2, r = 32 * quad + lane, etid = threadIdx.x - 64;
    const uint32_t tl = (uint32_t)(32 * quad) << 16;
    constexpr int G8 = NS / 32;  // 8-column groups per quarter of a staging pass
    const int col0 = part * G8 * 8;
    auto drain = [&](uint32_t taddr, uint64_t *release) {  // NS accumulator columns -> staging tile
      uint32_t v[G8][8];
#pragma unroll
      for (int g = 0; g < G8; g++) tmem_ld8_async(taddr + col0 + 8 * g, v[g]);
      tmem_wait_ld();
      float4 *dst = reinterpret_cast<float4 *>(stg + r * (NS + 4) + col0);
#pragma unroll
      for (int g = 0; g < G8; g++) {
        dst[2 * g] = make_float4(__uint_as_float(v[g][0]), __uint_as_float(v[g][1]), __uint_as_float(v[g][2]),
                                 __uint_as_float(v[g][3]));
        dst[2 * g + 1] = make_float4(__uint_as_float(v[g][4]), __uint_as_float(v[g][5]), __uint_as_float(v[g][6]),
                                     __uint_as_float(v[g][7]));
      }
      tc_fence_before();
      __syncwarp();
      if (release && lane == 0) mbar_arrive1(release);
    };
    int it = 0;
    PtTile prev{0, 0, 0, 0};
    for (int t = blockIdx.x; t < c.total; t += gridDim.x, it++) {
      const PtTile p = pt_tile(c, t, N);
      const int buf = it & 1;
      if (!err && !mbar_wait(&accf[buf], (it >> 1) & 1)) err |= 32u;
      tc_fence_after();
      __syncwarp();
      const uint32_t acc = tmem + tl + kAccStride * buf;
      if (FUSE) {
        if (it >= 1) {  // tile it - 1's k1 result; also frees A2
          if (!err && !mbar_wait(acc2f, (it - 1) & 1)) err |= 64u;
          tc_fence_after();
          __syncwarp();
          drain(tmem + tl + kAcc2, nullptr);
          bar_epi();
          conv_sweep_cols<NS, kPtEpiWarps * 32>(a, stg, prev.b, prev.tq0, prev.n0, prev.phase, etid);
          bar_epi();
        }
        // act2(acc + b7) -> fp16 A operand of the k1 GEMM
        {
          uint32_t v[G8][8];
#pragma unroll
          for (int g = 0; g < G8; g++) tmem_ld8_async(acc + col0 + 8 * g, v[g]);
          tmem_wait_ld();
#pragma unroll
          for (int g = 0; g < G8; g++) {
            const int col = col0 + 8 * g, q = col / ACH, j = (col - q * ACH) / 8;
            uint32_t h[4];
            float pb[8], pa[8], pi[8];
#pragma unroll
            for (int e = 0; e < 8; e += 4) {
              *reinterpret_cast<float4 *>(pb + e) = *reinterpret_cast<const float4 *>(par + col + e);
              *reinterpret_cast<float4 *>(pa + e) = *reinterpret_cast<const float4 *>(par + N + col + e);
              *reinterpret_cast<float4 *>(pi + e) = *reinterpret_cast<const float4 *>(par + 2 * N + col + e);
            }
#pragma unroll
            for (int e = 0; e < 8; e += 2) {
              const float y0 = snake(__uint_as_float(v[g][e]) + pb[e], pa[e], pi[e]);
              const float y1 = snake(__uint_as_float(v[g][e + 1]) + pb[e + 1], pa[e + 1], pi[e + 1]);
              const __half2 hp = __floats2half2_rn(y0, y1);
              h[e / 2] = *reinterpret_cast<const uint32_t *>(&hp);
            }
            *reinterpret_cast<uint4 *>(a2 + q * L::kA + swz_off<ACH>(r, j)) = make_uint4(h[0], h[1], h[2], h[3]);
          }
        }
        fence_proxy_async();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive1(&acce[buf]);
          mbar_arrive1(a2f);
        }
        prev = p;
      } else {
#pragma unroll 1
        for (int cb = 0; cb < N / NS; cb++) {
          drain(acc + cb * NS, cb == N / NS - 1 ? &acce[buf] : nullptr);
          bar_epi();
          conv_sweep_cols<NS, kPtEpiWarps * 32>(a, stg, p.b, p.tq0, p.n0 + cb * NS, p.phase, etid);
          bar_epi();
        }
      }
    }
    if (FUSE && it >= 1) {
      if (!err && !mbar_wait(acc2f, (it - 1) & 1)) err |= 64u;
      tc_fence_after();
      __syncwarp();
      drain(tmem + tl + kAcc2, nullptr);
      bar_epi();
      conv_sweep_cols<NS, kPtEpiWarps * 32>(a, stg, prev.b, prev.tq0, prev.n0, prev.phase, etid);
    }
  }
  if (err && c.err) atomicOr(c.err, (int)(err << 8));
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kCols);
}

static int g_sm_count = 0;

template <int N, int ACH, int S, int FUSE>
static void conv_pt_launch(const ConvArgs &a, int phases, cudaStream_t st, const ConvFuse *fu = nullptr) {
  using L = ConvPtSmem<N, ACH, S, FUSE>;
  static uint64_t attr = 0;
  if (first_on_device(attr))
    CK(cudaFuncSetAttribute(k_conv_pt<N, ACH, S, FUSE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                            (int)L::kBytes));
  if (!g_sm_count) {
    int dev = 0;
    CK(cudaGetDevice(&dev));
    CK(cudaDeviceGetAttribute(&g_sm_count, cudaDevAttrMultiProcessorCount, dev));
  }
  ConvPt c;
  memset(&c, 0, sizeof c);
  const CUtensorMapSwizzle sw = ACH == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  if (FUSE) {
    if (!fu || a.Cout != N || a.Cin != N || phases != 1)
      FAIL(Q3T_INVALID_INPUT, "codec fused residual unit: %d -> %d channels, %d phases (%d -> %d, 1 expected)",
           a.Cin, a.Cout, phases, N, N);
    const uint64_t dims[2] = {(uint64_t)N, (uint64_t)N};
    const uint64_t strides[1] = {(uint64_t)N * 2};
    const uint32_t box[2] = {(uint32_t)ACH, (uint32_t)N};
    if (!make_tmap(&c.tw1, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, fu->W1, dims, strides, box, sw))
      FAIL(Q3T_CUDA_ERROR, "codec conv: TMA descriptor of the k1 weights failed");
    c.mid_bias = fu->mid_bias;
    c.mid_a = fu->mid_a;
    c.mid_b = fu->mid_b;
  }
  {
    const uint64_t dims[3] = {(uint64_t)a.Cin, (uint64_t)a.Lin, (uint64_t)a.B};
    const uint64_t strides[2] = {(uint64_t)a.Cin * 2, (uint64_t)a.Lin * a.Cin * 2};
    const uint32_t box[3] = {(uint32_t)ACH, 128, 1};
    if (!make_tmap(&c.tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, a.X, dims, strides, box, sw))
      FAIL(Q3T_CUDA_ERROR, "codec conv: TMA descriptor of the input failed");
  }
  {
    const uint64_t dims[2] = {(uint64_t)a.Cin, (uint64_t)phases * a.taps * a.Cout};
    const uint64_t strides[1] = {(uint64_t)a.Cin * 2};
    const uint32_t box[2] = {(uint32_t)ACH, (uint32_t)N};
    if (!make_tmap(&c.tw, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a.W, dims, strides, box, sw))
      FAIL(Q3T_CUDA_ERROR, "codec conv: TMA descriptor of the weights failed");
  }
  c.a = a;
  c.tiles = (a.Lq + 127) / 128;
  c.nb = a.Cout / N;
  c.phases = phases;
  const int64_t total = (int64_t)a.B * c.tiles * c.nb * phases;
  if (total > INT32_MAX) FAIL(Q3T_INVALID_INPUT, "codec conv: %lld output tiles", (long long)total);
  c.total = (int)total;
  c.err = conv_err_word();
  const int grid = (int)std::min<int64_t>(total, g_sm_count);
  k_conv_pt<N, ACH, S, FUSE><<<grid, kPtThreads, L::kBytes, st>>>(c);
}

static void launch_conv(const ConvArgs &a, int phases, cudaStream_t st) {
  const int M = a.B * a.Lq;
  if (M <= 0) return;
  const bool tc = a.Cin % 32 == 0 && (a.Cout % 128 == 0 || a.Cout % 96 == 0) && !getenv("Q3T_CONV_MMA_SYNC");
  static const bool per_tile = getenv("Q3T_CONV_PER_TILE") != nullptr;  // one CTA per tile (k_conv_tc)
  if (tc && !per_tile) {
    const bool wide = a.Cin % 64 == 0, n128 = a.Cout % 128 == 0;
    if (wide && a.Cout % 256 == 0)
      conv_pt_launch<256, 64, 3, 0>(a, phases, st);
    else if (wide && a.Cout % 192 == 0)
      conv_pt_launch<192, 64, 4, 0>(a, phases, st);
    else if (wide && n128)
      conv_pt_launch<128, 64, 4, 0>(a, phases, st);
    else if (wide)
      conv_pt_launch<96, 64, 6, 0>(a, phases, st);
    else if (n128)
      conv_pt_launch<128, 32, 8, 0>(a, phases, st);
    else
      conv_pt_launch<96, 32, 8, 0>(a, phases, st);
  } else if (tc) {
    const bool wide = a.Cin % 64 == 0, n128 = a.Cout % 128 == 0;
    if (wide && n128)
      conv_tc_launch<128, 64, 3, 0>(a, phases, st);
    else if (wide)
      conv_tc_launch<96, 64, 3, 0>(a, phases, st);
    else if (n128)
      conv_tc_launch<128, 32, 6, 0>(a, phases, st);
    else
      conv_tc_launch<96, 32, 6, 0>(a, phases, st);
  } else if (a.Cout % 128 == 0) {
    dim3 grid((M + kBM - 1) / kBM, a.Cout / 128, phases);
    k_conv<128><<<grid, 256, conv_smem(128), st>>>(a);
  } else if (a.Cout % 96 == 0) {
    dim3 grid((M + kBM - 1) / kBM, a.Cout / 96, phases);
    k_conv<96><<<grid, 256, conv_smem(96), st>>>(a);
  } else {
    FAIL(Q3T_INVALID_INPUT, "codec conv: Cout %d is not a multiple of 96 or 128", a.Cout);
  }
  CK(cudaGetLastError());
  g_launches++;
}

// A whole residual unit in one launch (k_conv_tc FUSE = 1) where the stage
// has 96 channels on the tensor-core path; false if the caller must run the
// k7 and k1 convolutions as two launches.
static bool fused_unit_ok(int C) { return C == 96 && !getenv("Q3T_CONV_MMA_SYNC") && !getenv("Q3T_CODEC_UNFUSED"); }

static void launch_unit(const ConvArgs &a, const ConvFuse &fu, cudaStream_t st) {
  if (a.B * a.Lq <= 0) return;
  if (getenv("Q3T_CONV_PER_TILE"))
    conv_tc_launch<96, 32, 6, 1>(a, 1, st, &fu);
  else
    conv_pt_launch<96, 32, 8, 1>(a, 1, st, &fu);
  CK(cudaGetLastError());
  g_launches++;
}

// ---------------------------------------------------------------------------
// small kernels
// ---------------------------------------------------------------------------
// RVQ gather-sum (decoder.rs:196-247, codebook.rs:4-41): codes [B][nq][T] ->
// out [B*T][2*half] fp16 = [sum of semantic rows | sum of acoustic rows].
__global__ void k_gather(const int64_t *codes, int nq, int nsem, int T, const float *cent, int cb, int half,
                         __half *out) {
  const int bt = blockIdx.x, b = bt / T, t = bt - b * T;
  for (int d = threadIdx.x; d < half; d += blockDim.x) {
    float s = 0.f, r = 0.f;
    for (int q = 0; q < nq; q++) {
      int64_t id = codes[((size_t)b * nq + q) * T + t];
      id = (id < 0 || id >= cb) ? 0 : id;  // host-validated; streaming windows clamp talker specials
      const float v = cent[((size_t)q * cb + id) * half + d];
      if (q < nsem)
        s += v;
      else
        r += v;
    }
    out[(size_t)bt * 2 * half + d] = __float2half_rn(s);
    out[(size_t)bt * 2 * half + half + d] = __float2half_rn(r);
  }
}

// RMSNorm of f32 rows -> fp16 (burn::nn::RmsNorm)
__global__ void k_rmsnorm_h(const float *x, const float *gamma, int C, float eps, __half *out) {
  __shared__ float red[33];
  const float *xr = x + (size_t)blockIdx.x * C;
  float ss = 0.f;
  for (int i = threadIdx.x; i < C; i += blockDim.x) ss += xr[i] * xr[i];
  ss = block_sum(ss, red);
  const float rms = sqrtf(ss / (float)C + eps);
  for (int i = threadIdx.x; i < C; i += blockDim.x)
    out[(size_t)blockIdx.x * C + i] = __float2half_rn(xr[i] / rms * gamma[i]);
}

// adjacent-pair RoPE (burn::nn::RotaryEncoding, offset 0) on q and k, and the
// [M][3 * 1024] -> [B][heads][T][hd] split
__global__ void k_codec_rope(const float *qkv, int T, int nh, int nkv, int hd, const float *th, float *q,
                             float *k, float *v) {
  const int bt = blockIdx.x, b = bt / T, t = bt - b * T;
  const int qd = nh * hd, kd = nkv * hd;
  const float *row = qkv + (size_t)bt * (qd + 2 * kd);
  for (int e = threadIdx.x; e < (qd + kd) / 2; e += blockDim.x) {
    const int pe = e * 2;
    const bool isq = pe < qd;
    const int off = isq ? pe : pe - qd;
    const int h = off / hd, d = off - h * hd;
    float s, c;
    sincosf((float)t * th[d >> 1], &s, &c);
    const float x0 = row[pe], x1 = row[pe + 1];
    float *dst = (isq ? q + (((size_t)b * nh + h) * T + t) * hd : k + (((size_t)b * nkv + h) * T + t) * hd) + d;
    dst[0] = x0 * c - x1 * s;
    dst[1] = x1 * c + x0 * s;
  }
  for (int e = threadIdx.x; e < kd; e += blockDim.x) {
    const int h = e / hd, d = e - h * hd;
    v[(((size_t)b * nkv + h) * T + t) * hd + d] = row[qd + kd + e];
  }
}

// non-causal full attention (mask None, decoder.rs:265): one thread per
// query, keys streamed through shared memory in tiles with an online softmax.
constexpr int kAttKeys = 16;
__global__ void __launch_bounds__(128) k_codec_attn(const float *q, const float *k, const float *v, int T,
                                                    int nh, int nkv, float scale, __half *out) {
  constexpr int HD = 64;
  __shared__ float ks[kAttKeys][HD], vs[kAttKeys][HD];
  const int b = blockIdx.z, h = blockIdx.y, t = blockIdx.x * blockDim.x + threadIdx.x;
  const int hk = h / (nh / nkv);
  const float *kb = k + ((size_t)b * nkv + hk) * T * HD;
  const float *vb = v + ((size_t)b * nkv + hk) * T * HD;
  float qr[HD], acc[HD];
  const bool active = t < T;
#pragma unroll
  for (int d = 0; d < HD; d++) {
    qr[d] = active ? q[(((size_t)b * nh + h) * T + t) * HD + d] * scale : 0.f;
    acc[d] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  for (int j0 = 0; j0 < T; j0 += kAttKeys) {
    const int nk = min(kAttKeys, T - j0);
    __syncthreads();
    for (int e = threadIdx.x; e < kAttKeys * HD; e += blockDim.x) {
      const int j = e / HD, d = e - j * HD;
      ks[j][d] = j < nk ? kb[(size_t)(j0 + j) * HD + d] : 0.f;
      vs[j][d] = j < nk ? vb[(size_t)(j0 + j) * HD + d] : 0.f;
    }
    __syncthreads();
    float s[kAttKeys];
    float mt = m;
#pragma unroll
    for (int j = 0; j < kAttKeys; j++) {
      float a = 0.f;
#pragma unroll
      for (int d = 0; d < HD; d++) a += qr[d] * ks[j][d];
      s[j] = j < nk ? a : -INFINITY;
      mt = fmaxf(mt, s[j]);
    }
    const float corr = expf(m - mt);
    l *= corr;
#pragma unroll
    for (int d = 0; d < HD; d++) acc[d] *= corr;
#pragma unroll
    for (int j = 0; j < kAttKeys; j++) {
      const float p = expf(s[j] - mt);
      l += p;
#pragma unroll
      for (int d = 0; d < HD; d++) acc[d] += p * vs[j][d];
    }
    m = mt;
  }
  if (active) {
    __half *o = out + ((size_t)b * T + t) * nh * HD + h * HD;
    for (int d = 0; d < HD; d += 2) *reinterpret_cast<__half2 *>(o + d) = __floats2half2_rn(acc[d] / l, acc[d + 1] / l);
  }
}

// The same attention on the tensor cores (flash-attention style): a CTA takes
// 64 queries of one head, 4 warps x 16 query rows; keys and values stream
// through shared memory in tiles of 64.  S = Q K^T and O += P V run as
// mma.sync m16n8k16 with fp16 operands and f32 accumulators (the S
// accumulators are reused as the A fragments of P), the softmax is online in
// f32, keys beyond T are masked, and the output is rounded to fp16 as above.
constexpr int kCaRows = 64, kCaLd = 72;  // padded rows: conflict-free ldmatrix

Q3T_DEV void ldmatrix_x2_trans(uint32_t &r0, uint32_t &r1, const void *p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];\n"
               : "=r"(r0), "=r"(r1)
               : "r"(smem_addr(p)));
}

Q3T_DEV uint32_t pack_half2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t *>(&h);
}

// rows [r0, r0 + 64) of a [T][64] f32 head matrix -> fp16 [64][kCaLd] in shared memory (zeros past T)
Q3T_DEV void ca_load_tile(__half *dst, const float *src, int r0, int T) {
  for (int e = threadIdx.x; e < kCaRows * 16; e += blockDim.x) {
    const int row = e >> 4, c4 = e & 15;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r0 + row < T) v = *reinterpret_cast<const float4 *>(src + (size_t)(r0 + row) * 64 + c4 * 4);
    uint2 u;
    u.x = pack_half2(v.x, v.y);
    u.y = pack_half2(v.z, v.w);
    *reinterpret_cast<uint2 *>(dst + row * kCaLd + c4 * 4) = u;
  }
}

__global__ void __launch_bounds__(128) k_codec_attn_tc(const float *q, const float *k, const float *v, int T, int nh,
                                                       int nkv, float scale, __half *out) {
  __shared__ __align__(16) __half Qs[kCaRows * kCaLd], Ks[kCaRows * kCaLd], Vs[kCaRows * kCaLd];
  const int b = blockIdx.z, h = blockIdx.y, q0 = blockIdx.x * kCaRows;
  const int hk = h / (nh / nkv);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const float *qb = q + ((size_t)b * nh + h) * T * 64;
  const float *kb = k + ((size_t)b * nkv + hk) * T * 64;
  const float *vb = v + ((size_t)b * nkv + hk) * T * 64;
  ca_load_tile(Qs, qb, q0, T);
  __syncthreads();
  uint32_t qa[4][4];  // A fragments of this warp's 16 query rows, 4 k-steps of 16 dims
#pragma unroll
  for (int ks = 0; ks < 4; ks++)
    ldmatrix_x4(qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3],
                Qs + (warp * 16 + (lane & 15)) * kCaLd + ks * 16 + (lane >> 4) * 8);
  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;  // rows g and g + 8
  for (int j0 = 0; j0 < T; j0 += kCaRows) {
    __syncthreads();  // the previous tile is consumed
    ca_load_tile(Ks, kb, j0, T);
    ca_load_tile(Vs, vb, j0, T);
    __syncthreads();
    float s[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; nt++) {
      s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < 4; ks++) {
        uint32_t b0, b1;
        ldmatrix_x2(b0, b1, Ks + (nt * 8 + (lane & 7)) * kCaLd + ks * 16 + ((lane >> 3) & 1) * 8);
        mma_f16(s[nt], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b0, b1);
      }
    }
    float mx0 = m0, mx1 = m1;
#pragma unroll
    for (int nt = 0; nt < 8; nt++)
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const int key = j0 + nt * 8 + 2 * t + (e & 1);
        s[nt][e] = key < T ? s[nt][e] * scale : -INFINITY;
        if (e < 2)
          mx0 = fmaxf(mx0, s[nt][e]);
        else
          mx1 = fmaxf(mx1, s[nt][e]);
      }
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
    }
    const float c0 = expf(m0 - mx0), c1 = expf(m1 - mx1);  // the first tile has a valid key: mx finite
    m0 = mx0;
    m1 = mx1;
    float r0 = 0.f, r1 = 0.f;
#pragma unroll
    for (int nt = 0; nt < 8; nt++) {
      s[nt][0] = expf(s[nt][0] - m0);
      s[nt][1] = expf(s[nt][1] - m0);
      s[nt][2] = expf(s[nt][2] - m1);
      s[nt][3] = expf(s[nt][3] - m1);
      r0 += s[nt][0] + s[nt][1];
      r1 += s[nt][2] + s[nt][3];
    }
    l0 = l0 * c0 + r0;  // this lane's share; the quad sums it at the end
    l1 = l1 * c1 + r1;
#pragma unroll
    for (int dt = 0; dt < 8; dt++) {
      o[dt][0] *= c0;
      o[dt][1] *= c0;
      o[dt][2] *= c1;
      o[dt][3] *= c1;
    }
#pragma unroll
    for (int kk = 0; kk < 4; kk++) {
      const uint32_t pa0 = pack_half2(s[2 * kk][0], s[2 * kk][1]), pa1 = pack_half2(s[2 * kk][2], s[2 * kk][3]);
      const uint32_t pa2 = pack_half2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      const uint32_t pa3 = pack_half2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int dt = 0; dt < 8; dt++) {
        uint32_t b0, b1;
        ldmatrix_x2_trans(b0, b1, Vs + (kk * 16 + (lane & 15)) * kCaLd + dt * 8);
        mma_f16(o[dt], pa0, pa1, pa2, pa3, b0, b1);
      }
    }
  }
#pragma unroll
  for (int off = 1; off < 4; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
  const int ra = q0 + warp * 16 + g, rb = ra + 8;
#pragma unroll
  for (int dt = 0; dt < 8; dt++) {
    const int d = dt * 8 + 2 * t;
    if (ra < T)
      *reinterpret_cast<__half2 *>(out + ((size_t)b * T + ra) * nh * 64 + h * 64 + d) =
          __floats2half2_rn(o[dt][0] / l0, o[dt][1] / l0);
    if (rb < T)
      *reinterpret_cast<__half2 *>(out + ((size_t)b * T + rb) * nh * 64 + h * 64 + d) =
          __floats2half2_rn(o[dt][2] / l1, o[dt][3] / l1);
  }
}

__global__ void k_silu_mul_h(const float *gu, int I, __half *out) {
  const size_t row = blockIdx.x;
  for (int i = threadIdx.x; i < I; i += blockDim.x) {
    const float g = gu[row * 2 * I + i], u = gu[row * 2 * I + I + i];
    out[row * I + i] = __float2half_rn(g / (1.f + expf(-g)) * u);
  }
}

// ConvNeXt depthwise causal conv k7 + LayerNorm (wave.rs:96-108, eps 1e-6)
__global__ void __launch_bounds__(256) k_dwconv_ln(const float *y, int L, int C, const float *w, const float *bias,
                                                   const float *ln_w, const float *ln_b, __half *out) {
  __shared__ float red[33];
  extern __shared__ float dv[];
  const int bt = blockIdx.x, b = bt / L, t = bt - b * L;
  float s = 0.f;
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    float a = bias[c];
#pragma unroll
    for (int j = 0; j < 7; j++) {
      const int tt = t - 6 + j;
      if (tt >= 0) a += w[c * 7 + j] * y[((size_t)b * L + tt) * C + c];
    }
    dv[c] = a;
    s += a;
  }
  const float mean = block_sum(s, red) / (float)C;
  float vs = 0.f;
  for (int c = threadIdx.x; c < C; c += blockDim.x) vs += (dv[c] - mean) * (dv[c] - mean);
  const float var = block_sum(vs, red) / (float)C;
  const float den = sqrtf(var + 1e-6f);
  for (int c = threadIdx.x; c < C; c += blockDim.x)
    out[(size_t)bt * C + c] = __float2half_rn((dv[c] - mean) / den * ln_w[c] + ln_b[c]);
}

// output conv C -> 1, k7, causal, + clamp (decoder.rs:273-276) and PCM
// (codec/infer/mod.rs:80-90).  y[t] = bias + sum_j p_j[t - 6 + j] with
// p_j[u] = a[u] . w[j]: each thread reads one input row of the tile's rows
// [t0 - 6, t0 + kOutTile) once, 8 channels at a time, and forms its 7 tap
// products against weights broadcast from shared memory (4 FMAs per shared
// load); the partial sums meet in shared memory.
constexpr int kOutTile = 128;
__global__ void __launch_bounds__(kOutTile) k_out_conv(const __half *a, int L, int C, const float *w, float bias,
                                                       float *wave, int16_t *pcm) {
  __shared__ __align__(16) float ws[7 * 192];
  __shared__ float ps[7][kOutTile + 6];
  const int b = blockIdx.y, t0 = blockIdx.x * kOutTile;
  for (int e = threadIdx.x; e < 7 * C; e += blockDim.x) ws[e] = w[e];
  __syncthreads();
  for (int r = threadIdx.x; r < kOutTile + 6; r += blockDim.x) {
    const int u = t0 - 6 + r;
    float p[7] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (u >= 0 && u < L) {
      const uint4 *row = reinterpret_cast<const uint4 *>(a + ((size_t)b * L + u) * C);
      for (int c8 = 0; c8 < C / 8; c8++) {
        const uint4 v = row[c8];
        const __half2 *h = reinterpret_cast<const __half2 *>(&v);
        float x[8];
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const float2 f = __half22float2(h[i]);
          x[2 * i] = f.x;
          x[2 * i + 1] = f.y;
        }
#pragma unroll
        for (int j = 0; j < 7; j++) {
          const float4 w0 = *reinterpret_cast<const float4 *>(ws + j * C + 8 * c8);
          const float4 w1 = *reinterpret_cast<const float4 *>(ws + j * C + 8 * c8 + 4);
          p[j] += x[0] * w0.x + x[1] * w0.y + x[2] * w0.z + x[3] * w0.w + x[4] * w1.x + x[5] * w1.y + x[6] * w1.z +
                  x[7] * w1.w;
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 7; j++) ps[j][r] = p[j];
  }
  __syncthreads();
  const int t = t0 + threadIdx.x;
  if (t >= L) return;
  float acc = bias;
#pragma unroll
  for (int j = 0; j < 7; j++) acc += ps[j][threadIdx.x + j];
  const float y = fminf(fmaxf(acc, -1.f), 1.f);
  if (wave) wave[(size_t)b * L + t] = y;
  if (pcm) {
    int v = (int)roundf(y * 32768.0f);
    v = v < -32768 ? -32768 : (v > 32767 ? 32767 : v);
    pcm[(size_t)b * L + t] = (int16_t)v;
  }
}

// ---------------------------------------------------------------------------
// model
// ---------------------------------------------------------------------------
struct ConvW {
  __half *w = nullptr;  // [phases][taps][Cout][Cin]
  float *bias = nullptr;
  int phases = 1, taps = 1, cout = 0, cin = 0;
};
struct SnakeP {
  float *ea = nullptr, *ib = nullptr;
};
struct CodecLayerW {
  float *in_norm, *post_norm, *attn_scale, *mlp_scale;
  ConvW qkv, o, gu, down;
};
struct UpW {
  ConvW convt;
  float *dw_w, *dw_b, *ln_w, *ln_b, *gamma;
  ConvW pw1, pw2;
  int r;
};
struct ResW {
  SnakeP a1, a2;
  ConvW c1, c2;
};
struct StageW {
  SnakeP s0;
  ConvW convt;
  ResW ru[3];
  int r, cin, cout;
};

struct CodecModel {
  q3t_codec_config c{};
  DevArena ar;
  float *cent = nullptr;  // [nq][cb][half]
  ConvW qproj, pre_conv, in_proj, out_proj, in_conv;
  std::vector<CodecLayerW> layers;
  float *final_norm = nullptr, *rope_th = nullptr;
  std::vector<UpW> up;
  std::vector<StageW> stages;
  SnakeP out_snake;
  float *out_w = nullptr;  // [7][C]
  float out_b = 0.f;
};

// The tensor `name` (or its other checkpoint spelling, checkpoint_alias) with
// `shape`'s element count, f32 or bf16.
static const q3t_tensor *find(const q3t_model_desc *d, const std::string &name, std::vector<int64_t> shape) {
  const std::string alt = checkpoint_alias(name);
  for (int pass = 0; pass < 2; pass++) {
    const std::string &want = pass == 0 ? name : alt;
    if (want.empty()) break;
    for (int i = 0; i < d->num_tensors; i++) {
      const q3t_tensor *t = &d->tensors[i];
      if (!t->name || want != t->name) continue;
      int64_t n1 = 1, n2 = 1;
      for (int k = 0; k < t->ndim; k++) n1 *= t->shape[k];
      for (auto s : shape) n2 *= s;
      if (n1 != n2 || !t->data || (t->dtype != Q3T_F32 && t->dtype != Q3T_BF16))
        FAIL(Q3T_RUNTIME_LOAD, "codec tensor %s: unexpected size or dtype (f32 or bf16 expected)", want.c_str());
      return t;
    }
  }
  FAIL(Q3T_RUNTIME_LOAD, "missing tensor %s", name.c_str());
}

// f32 host copy of an f32 or bf16 tensor
static std::vector<float> host(const q3t_tensor *t) {
  int64_t n = 1;
  for (int k = 0; k < t->ndim; k++) n *= t->shape[k];
  if (t->dtype == Q3T_F32) {
    const float *p = reinterpret_cast<const float *>(t->data);
    return std::vector<float>(p, p + n);
  }
  std::vector<float> f((size_t)n);
  const uint16_t *p = reinterpret_cast<const uint16_t *>(t->data);
  for (int64_t i = 0; i < n; i++) {
    const uint32_t u = (uint32_t)p[i] << 16;
    memcpy(&f[i], &u, 4);
  }
  return f;
}

template <typename T>
static T *to_dev(DevArena &ar, const std::vector<T> &h, cudaStream_t st) {
  T *d = ar.alloc<T>(h.size());
  CK(cudaMemcpyAsync(d, h.data(), h.size() * sizeof(T), cudaMemcpyHostToDevice, st));
  CK(cudaStreamSynchronize(st));
  return d;
}

static std::vector<__half> to_half(const std::vector<float> &f) {
  std::vector<__half> h(f.size());
  for (size_t i = 0; i < f.size(); i++) h[i] = __float2half_rn(f[i]);
  return h;
}

// Linear [out][in] -> ConvW (1 phase, 1 tap)
static ConvW linear_w(CodecModel *c, const q3t_model_desc *d, const std::string &name, int out, int in,
                      const std::string &bias, cudaStream_t st) {
  ConvW w;
  w.cout = out;
  w.cin = in;
  w.w = to_dev(c->ar, to_half(host(find(d, name, {out, in}))), st);
  if (!bias.empty()) w.bias = to_dev(c->ar, host(find(d, bias, {out})), st);
  return w;
}

// Conv1d [out][in][k] -> [k taps][out][in]
static ConvW conv_w(CodecModel *c, const q3t_model_desc *d, const std::string &name, int out, int in, int k,
                    bool bias, cudaStream_t st) {
  std::vector<float> src = host(find(d, name + ".weight", {out, in, k}));
  std::vector<float> dst((size_t)k * out * in);
  for (int o = 0; o < out; o++)
    for (int i = 0; i < in; i++)
      for (int j = 0; j < k; j++) dst[((size_t)j * out + o) * in + i] = src[((size_t)o * in + i) * k + j];
  ConvW w;
  w.cout = out;
  w.cin = in;
  w.taps = k;
  w.w = to_dev(c->ar, to_half(dst), st);
  if (bias) w.bias = to_dev(c->ar, host(find(d, name + ".bias", {out})), st);
  return w;
}

// ConvTranspose1d [in][out][k], stride r.  k == r: r phases x 1 tap (w[.,.,p]);
// k == 2r (trimmed by r): r phases x 2 taps {w[.,.,p+r], w[.,.,p]}.
static ConvW convt_w(CodecModel *c, const q3t_model_desc *d, const std::string &name, int in, int out, int k,
                     int r, cudaStream_t st) {
  std::vector<float> src = host(find(d, name + ".weight", {in, out, k}));
  const int taps = k / r;
  std::vector<float> dst((size_t)r * taps * out * in);
  for (int p = 0; p < r; p++)
    for (int tp = 0; tp < taps; tp++) {
      const int j = taps == 1 ? p : (tp == 0 ? p + r : p);
      for (int o = 0; o < out; o++)
        for (int i = 0; i < in; i++)
          dst[(((size_t)p * taps + tp) * out + o) * in + i] = src[((size_t)i * out + o) * k + j];
    }
  ConvW w;
  w.cout = out;
  w.cin = in;
  w.taps = taps;
  w.phases = r;
  w.w = to_dev(c->ar, to_half(dst), st);
  w.bias = to_dev(c->ar, host(find(d, name + ".bias", {out})), st);
  return w;
}

static SnakeP snake_w(CodecModel *c, const q3t_model_desc *d, const std::string &prefix, int C, cudaStream_t st) {
  std::vector<float> al = host(find(d, prefix + ".alpha", {C})), be = host(find(d, prefix + ".beta", {C}));
  std::vector<float> ea(C), ib(C);
  for (int i = 0; i < C; i++) {
    ea[i] = expf(al[i]);
    ib[i] = 1.0f / (expf(be[i]) + 1e-9f);
  }
  return SnakeP{to_dev(c->ar, ea, st), to_dev(c->ar, ib, st)};
}

CodecModel *codec_load(q3t_model *m, const q3t_model_desc *d, cudaStream_t st) {
  auto *c = new CodecModel();
  try {
    const q3t_codec_config &k = d->codec;
    c->c = k;
    const int half = k.codebook_dim / 2, D = k.codebook_dim, LAT = k.latent_dim, H = k.hidden_size;
    if (k.codebook_dim % 64 || k.latent_dim % 128 || k.decoder_dim % 128 || k.hidden_size % 128)
      FAIL(Q3T_INVALID_INPUT, "codec widths must be multiples of 64/128");
    if (k.head_dim != 64) FAIL(Q3T_INVALID_INPUT, "codec head_dim %d unsupported (64 expected)", k.head_dim);
    if (k.num_quantizers < 1 || k.num_semantic_quantizers < 1 || k.num_semantic_quantizers > k.num_quantizers)
      FAIL(Q3T_INVALID_INPUT, "codec quantizer counts invalid");
    if (k.num_upsample_rates < 1 || k.num_upsample_rates > 8 || k.num_upsampling_ratios > 4)
      FAIL(Q3T_INVALID_INPUT, "codec upsampling config invalid");
    // codebooks: centroids = embedding_sum / clamp_min(cluster_usage, 1e-6)
    std::vector<float> cent((size_t)k.num_quantizers * k.codebook_size * half);
    for (int q = 0; q < k.num_quantizers; q++) {
      const bool sem = q < k.num_semantic_quantizers;
      const std::string p = std::string("decoder.quantizer.") + (sem ? "rvq_first" : "rvq_rest") + ".vq.layers." +
                            std::to_string(sem ? q : q - k.num_semantic_quantizers) + "._codebook";
      std::vector<float> es = host(find(d, p + ".embedding_sum", {k.codebook_size, half}));
      std::vector<float> us = host(find(d, p + ".cluster_usage", {k.codebook_size}));
      for (int i = 0; i < k.codebook_size; i++) {
        const float u = us[i] < 1e-6f ? 1e-6f : us[i];
        for (int j = 0; j < half; j++) cent[((size_t)q * k.codebook_size + i) * half + j] = es[(size_t)i * half + j] / u;
      }
    }
    c->cent = to_dev(c->ar, cent, st);
    // output projections of both RVQ groups as one K = 2*half GEMM
    {
      std::vector<float> f = host(find(d, "decoder.quantizer.rvq_first.output_proj.weight", {D, half, 1}));
      std::vector<float> r = host(find(d, "decoder.quantizer.rvq_rest.output_proj.weight", {D, half, 1}));
      std::vector<float> w((size_t)D * 2 * half);
      for (int o = 0; o < D; o++)
        for (int i = 0; i < half; i++) {
          w[(size_t)o * 2 * half + i] = f[(size_t)o * half + i];
          w[(size_t)o * 2 * half + half + i] = r[(size_t)o * half + i];
        }
      c->qproj.cout = D;
      c->qproj.cin = 2 * half;
      c->qproj.w = to_dev(c->ar, to_half(w), st);
    }
    c->pre_conv = conv_w(c, d, "decoder.pre_conv.conv", LAT, D, 3, true, st);
    const std::string pt = "decoder.pre_transformer";
    c->in_proj = linear_w(c, d, pt + ".input_proj.weight", H, LAT, pt + ".input_proj.bias", st);
    c->out_proj = linear_w(c, d, pt + ".output_proj.weight", LAT, H, pt + ".output_proj.bias", st);
    c->final_norm = to_dev(c->ar, host(find(d, pt + ".norm.weight", {H})), st);
    const int qd = k.num_attention_heads * 64, kd = k.num_key_value_heads * 64;
    for (int l = 0; l < k.num_hidden_layers; l++) {
      const std::string p = pt + ".layers." + std::to_string(l);
      CodecLayerW L;
      L.in_norm = to_dev(c->ar, host(find(d, p + ".input_layernorm.weight", {H})), st);
      L.post_norm = to_dev(c->ar, host(find(d, p + ".post_attention_layernorm.weight", {H})), st);
      L.attn_scale = to_dev(c->ar, host(find(d, p + ".self_attn_layer_scale.scale", {H})), st);
      L.mlp_scale = to_dev(c->ar, host(find(d, p + ".mlp_layer_scale.scale", {H})), st);
      std::vector<float> qkv;
      for (const char *n : {"q", "k", "v"}) {
        const int rows = n[0] == 'q' ? qd : kd;
        std::vector<float> t = host(find(d, p + ".self_attn." + n + "_proj.weight", {rows, H}));
        qkv.insert(qkv.end(), t.begin(), t.end());
      }
      L.qkv.cout = qd + 2 * kd;
      L.qkv.cin = H;
      L.qkv.w = to_dev(c->ar, to_half(qkv), st);
      L.o = linear_w(c, d, p + ".self_attn.o_proj.weight", H, qd, "", st);
      std::vector<float> gu = host(find(d, p + ".mlp.gate_proj.weight", {k.intermediate_size, H}));
      std::vector<float> up = host(find(d, p + ".mlp.up_proj.weight", {k.intermediate_size, H}));
      gu.insert(gu.end(), up.begin(), up.end());
      L.gu.cout = 2 * k.intermediate_size;
      L.gu.cin = H;
      L.gu.w = to_dev(c->ar, to_half(gu), st);
      L.down = linear_w(c, d, p + ".mlp.down_proj.weight", H, k.intermediate_size, "", st);
      c->layers.push_back(L);
    }
    {  // burn::nn::RotaryEncoding: theta_i = 1 / theta^(2i / d), via exp(ln(theta) * 2i / d)
      std::vector<float> th(32);
      for (int i = 0; i < 32; i++) th[i] = 1.0f / expf((float)(2 * i) / 64.0f * logf(k.rope_theta));
      c->rope_th = to_dev(c->ar, th, st);
    }
    for (int u = 0; u < k.num_upsampling_ratios; u++) {
      const std::string p = "decoder.upsample." + std::to_string(u);
      const int r = k.upsampling_ratios[u];
      UpW U;
      U.r = r;
      U.convt = convt_w(c, d, p + ".0.conv", LAT, LAT, r, r, st);
      U.dw_w = to_dev(c->ar, host(find(d, p + ".1.dwconv.conv.weight", {LAT, 1, 7})), st);
      U.dw_b = to_dev(c->ar, host(find(d, p + ".1.dwconv.conv.bias", {LAT})), st);
      U.ln_w = to_dev(c->ar, host(find(d, p + ".1.norm.weight", {LAT})), st);
      U.ln_b = to_dev(c->ar, host(find(d, p + ".1.norm.bias", {LAT})), st);
      U.pw1 = linear_w(c, d, p + ".1.pwconv1.weight", 4 * LAT, LAT, p + ".1.pwconv1.bias", st);
      U.pw2 = linear_w(c, d, p + ".1.pwconv2.weight", LAT, 4 * LAT, p + ".1.pwconv2.bias", st);
      U.gamma = to_dev(c->ar, host(find(d, p + ".1.gamma", {LAT})), st);
      c->up.push_back(U);
    }
    int C = k.decoder_dim;
    c->in_conv = conv_w(c, d, "decoder.decoder.0.conv", C, LAT, 7, true, st);
    for (int i = 0; i < k.num_upsample_rates; i++) {
      const std::string p = "decoder.decoder." + std::to_string(i + 1) + ".block";
      const int r = k.upsample_rates[i], Co = C / 2;
      StageW S;
      S.r = r;
      S.cin = C;
      S.cout = Co;
      S.s0 = snake_w(c, d, p + ".0", C, st);
      S.convt = convt_w(c, d, p + ".1.conv", C, Co, 2 * r, r, st);
      for (int j = 0; j < 3; j++) {
        const std::string q = p + "." + std::to_string(j + 2);
        S.ru[j].a1 = snake_w(c, d, q + ".act1", Co, st);
        S.ru[j].a2 = snake_w(c, d, q + ".act2", Co, st);
        S.ru[j].c1 = conv_w(c, d, q + ".conv1.conv", Co, Co, 7, true, st);
        S.ru[j].c2 = conv_w(c, d, q + ".conv2.conv", Co, Co, 1, true, st);
      }
      c->stages.push_back(S);
      C = Co;
    }
    if (C > 192 || C % 2) FAIL(Q3T_INVALID_INPUT, "codec output channels %d unsupported", C);
    const int n = k.num_upsample_rates;
    c->out_snake = snake_w(c, d, "decoder.decoder." + std::to_string(n + 1), C, st);
    {
      std::vector<float> w = host(find(d, "decoder.decoder." + std::to_string(n + 2) + ".conv.weight", {1, C, 7}));
      std::vector<float> wt((size_t)7 * C);
      for (int i = 0; i < C; i++)
        for (int j = 0; j < 7; j++) wt[(size_t)j * C + i] = w[(size_t)i * 7 + j];
      c->out_w = to_dev(c->ar, wt, st);
      c->out_b = host(find(d, "decoder.decoder." + std::to_string(n + 2) + ".conv.bias", {1}))[0];
    }
    static uint64_t attrs = 0;
    if (first_on_device(attrs)) {
      CK(cudaFuncSetAttribute(k_conv<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)conv_smem(128)));
      CK(cudaFuncSetAttribute(k_conv<96>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)conv_smem(96)));
    }
  } catch (...) {
    delete c;
    throw;
  }
  (void)m;
  return c;
}

void codec_free(CodecModel *c) { delete c; }

void codec_out_len(const CodecModel *c, int T, int64_t *n) {
  int64_t L = T;
  for (int i = 0; i < c->c.num_upsampling_ratios; i++) L *= c->c.upsampling_ratios[i];
  for (int i = 0; i < c->c.num_upsample_rates; i++) L = L > 0 ? (L - 1) * c->c.upsample_rates[i] : 0;
  *n = L;
}

// ---------------------------------------------------------------------------
// decode
// ---------------------------------------------------------------------------
static ConvArgs conv_args(const ConvW &w, const __half *X, int B, int Lin, int in_off, int dil, int Lq, int ostride,
                          int Lout) {
  ConvArgs a{};
  a.X = X;
  a.Lin = Lin;
  a.Cin = w.cin;
  a.B = B;
  a.W = w.w;
  a.Cout = w.cout;
  a.taps = w.taps;
  a.w_phase_stride = (long long)w.taps * w.cout * w.cin;
  a.bias = w.bias;
  a.in_off = in_off;
  a.dil = dil;
  a.Lq = Lq;
  a.ostride = ostride;
  a.Lout = Lout;
  return a;
}

// Decodes codes [B][nq][T] (device) into wave / pcm [B][n] (device, nullable).
// Intermediate buffers of one decode of B x T frames and their sizes in bytes.
struct CodecScratch {
  enum { X32, A0, A1, HH, F1, G, Q, K, V, HRES, N };
  int64_t bytes[N];
  void *p[N];
};

static CodecScratch codec_scratch(const CodecModel *c, int B, int T) {
  const auto &k = c->c;
  const int half = k.codebook_dim / 2, LAT = k.latent_dim, H = k.hidden_size;
  const int nh = k.num_attention_heads, nkv = k.num_key_value_heads, qd = nh * 64, kd = nkv * 64;
  const int M0 = B * T;
  int64_t Lmax = T;
  for (int i = 0; i < k.num_upsampling_ratios; i++) Lmax *= k.upsampling_ratios[i];
  const int64_t Lup = Lmax;
  int64_t big = Lup * k.decoder_dim, L = Lup;
  for (int i = 0; i < k.num_upsample_rates; i++) {
    L = (L - 1) * k.upsample_rates[i];
    big = std::max<int64_t>(big, L * (k.decoder_dim >> (i + 1)));
  }
  big *= B;
  const int64_t pre = (int64_t)M0 * std::max(std::max(qd + 2 * kd, 2 * k.intermediate_size), LAT);
  const int64_t upn = B * Lup * 4 * (int64_t)LAT;
  CodecScratch s{};
  s.bytes[CodecScratch::X32] = std::max(big, (int64_t)B * Lup * LAT) * 4;
  s.bytes[CodecScratch::A0] = std::max(big, upn) * 2;
  s.bytes[CodecScratch::A1] = std::max(big, (int64_t)B * Lup * LAT) * 2;
  s.bytes[CodecScratch::HH] = std::max(big, (int64_t)M0 * 2 * half) * 2;
  s.bytes[CodecScratch::F1] = std::max(pre, (int64_t)M0 * H) * 4;
  s.bytes[CodecScratch::G] = std::max(pre, (int64_t)M0 * qd) * 2;
  s.bytes[CodecScratch::Q] = (int64_t)M0 * qd * 4;
  s.bytes[CodecScratch::K] = (int64_t)M0 * kd * 4;
  s.bytes[CodecScratch::V] = (int64_t)M0 * kd * 4;
  s.bytes[CodecScratch::HRES] = (int64_t)M0 * H * 4;  // pre-transformer residual [M0][H]
  return s;
}

static void decode_with(CodecModel *c, const CodecScratch &ws, const int64_t *d_codes, int B, int T,
                        float *d_wave, int16_t *d_pcm, cudaStream_t st);

static void decode_device(CodecModel *c, const int64_t *d_codes, int B, int T, float *d_wave, int16_t *d_pcm,
                          cudaStream_t st) {
  CodecScratch ws = codec_scratch(c, B, T);
  for (int i = 0; i < CodecScratch::N; i++) CK(cudaMallocAsync(&ws.p[i], ws.bytes[i], st));
  decode_with(c, ws, d_codes, B, T, d_wave, d_pcm, st);
  for (int i = 0; i < CodecScratch::N; i++) CK(cudaFreeAsync(ws.p[i], st));
}

static void decode_with(CodecModel *c, const CodecScratch &ws, const int64_t *d_codes, int B, int T,
                        float *d_wave, int16_t *d_pcm, cudaStream_t st) {
  const auto &k = c->c;
  const int half = k.codebook_dim / 2, LAT = k.latent_dim, H = k.hidden_size;
  const int nh = k.num_attention_heads, nkv = k.num_key_value_heads;
  const int M0 = B * T;
  float *X32 = (float *)ws.p[CodecScratch::X32], *F1 = (float *)ws.p[CodecScratch::F1];
  float *Q = (float *)ws.p[CodecScratch::Q], *K = (float *)ws.p[CodecScratch::K];
  float *V = (float *)ws.p[CodecScratch::V], *hres = (float *)ws.p[CodecScratch::HRES];
  __half *A0 = (__half *)ws.p[CodecScratch::A0], *A1 = (__half *)ws.p[CodecScratch::A1];
  __half *Hh = (__half *)ws.p[CodecScratch::HH], *G = (__half *)ws.p[CodecScratch::G];

  // quantizer: gather-sum + both output projections in one GEMM
  k_gather<<<M0, 256, 0, st>>>(d_codes, k.num_quantizers, k.num_semantic_quantizers, T, c->cent, k.codebook_size,
                                half, Hh);
  CK(cudaGetLastError());
  {
    ConvArgs a = conv_args(c->qproj, Hh, B, T, 0, 1, T, 1, T);
    a.Yh = A1;  // [B][T][D]
    launch_conv(a, 1, st);
  }
  // pre_conv causal k3 (decoder.rs:261)
  {
    ConvArgs a = conv_args(c->pre_conv, A1, B, T, -2, 1, T, 1, T);
    a.Yh = A0;  // [B][T][LAT]
    launch_conv(a, 1, st);
  }
  // pre-transformer (decoder.rs:175-194)
  {
    ConvArgs a = conv_args(c->in_proj, A0, B, T, 0, 1, T, 1, T);
    a.Yf = hres;
    launch_conv(a, 1, st);
  }
  for (const auto &Lw : c->layers) {
    k_rmsnorm_h<<<M0, 128, 0, st>>>(hres, Lw.in_norm, H, k.rms_norm_eps, G);
    ConvArgs a = conv_args(Lw.qkv, G, B, T, 0, 1, T, 1, T);
    a.Yf = F1;
    launch_conv(a, 1, st);
    k_codec_rope<<<M0, 256, 0, st>>>(F1, T, nh, nkv, 64, c->rope_th, Q, K, V);
    if (getenv("Q3T_CODEC_ATTN_F32"))
      k_codec_attn<<<dim3((T + 127) / 128, nh, B), 128, 0, st>>>(Q, K, V, T, nh, nkv, 0.125f, G);
    else
      k_codec_attn_tc<<<dim3((T + kCaRows - 1) / kCaRows, nh, B), 128, 0, st>>>(Q, K, V, T, nh, nkv, 0.125f, G);
    CK(cudaGetLastError());
    a = conv_args(Lw.o, G, B, T, 0, 1, T, 1, T);
    a.Yf = hres;
    a.R = hres;
    a.scale = Lw.attn_scale;
    launch_conv(a, 1, st);
    k_rmsnorm_h<<<M0, 128, 0, st>>>(hres, Lw.post_norm, H, k.rms_norm_eps, G);
    a = conv_args(Lw.gu, G, B, T, 0, 1, T, 1, T);
    a.Yf = F1;
    launch_conv(a, 1, st);
    k_silu_mul_h<<<M0, 256, 0, st>>>(F1, k.intermediate_size, G);
    a = conv_args(Lw.down, G, B, T, 0, 1, T, 1, T);
    a.Yf = hres;
    a.R = hres;
    a.scale = Lw.mlp_scale;
    launch_conv(a, 1, st);
    g_launches += 5;
  }
  k_rmsnorm_h<<<M0, 128, 0, st>>>(hres, c->final_norm, H, k.rms_norm_eps, G);
  g_launches += 2;
  {
    ConvArgs a = conv_args(c->out_proj, G, B, T, 0, 1, T, 1, T);
    a.Yh = A1;  // [B][T][LAT]
    launch_conv(a, 1, st);
  }
  // upsample: ConvT(k = r, s = r) + ConvNeXt (decoder.rs:268-271)
  int Lc = T;
  const __half *cur = A1;
  for (const auto &U : c->up) {
    const int Lo = Lc * U.r;
    ConvArgs a = conv_args(U.convt, cur, B, Lc, 0, 1, Lc, U.r, Lo);
    a.Yf = X32;
    launch_conv(a, U.r, st);
    k_dwconv_ln<<<B * Lo, 256, LAT * sizeof(float), st>>>(X32, Lo, LAT, U.dw_w, U.dw_b, U.ln_w, U.ln_b, Hh);
    CK(cudaGetLastError());
    g_launches++;
    a = conv_args(U.pw1, Hh, B, Lo, 0, 1, Lo, 1, Lo);
    a.Yh = A0;
    a.act = ACT_GELU;
    launch_conv(a, 1, st);
    a = conv_args(U.pw2, A0, B, Lo, 0, 1, Lo, 1, Lo);
    a.Yf = X32;
    a.R = X32;
    a.scale = U.gamma;
    a.Yh = A1;
    launch_conv(a, 1, st);
    cur = A1;
    Lc = Lo;
  }
  // wave decoder (wave.rs:12-94)
  {
    ConvArgs a = conv_args(c->in_conv, cur, B, Lc, -6, 1, Lc, 1, Lc);
    a.Yf = X32;
    a.Yh = A0;
    a.act = ACT_SNAKE;
    a.act_a = c->stages[0].s0.ea;
    a.act_b = c->stages[0].s0.ib;
    launch_conv(a, 1, st);
  }
  __half *act = A0, *other = A1;
  for (size_t s = 0; s < c->stages.size(); s++) {
    const StageW &S = c->stages[s];
    const int Lo = (Lc - 1) * S.r;
    ConvArgs a = conv_args(S.convt, act, B, Lc, 0, 1, Lc - 1, S.r, Lo);
    a.Yf = X32;
    a.Yh = other;
    a.act = ACT_SNAKE;
    a.act_a = S.ru[0].a1.ea;
    a.act_b = S.ru[0].a1.ib;
    launch_conv(a, S.r, st);
    std::swap(act, other);
    Lc = Lo;
    static const int dil[3] = {1, 3, 9};
    for (int j = 0; j < 3; j++) {
      const ResW &R = S.ru[j];
      const SnakeP &nx = j < 2 ? S.ru[j + 1].a1 : (s + 1 < c->stages.size() ? c->stages[s + 1].s0 : c->out_snake);
      if (fused_unit_ok(R.c1.cout)) {
        // one launch; its fp16 output goes to the spare buffer because the
        // k7 taps read rows of `act` that neighbouring tiles own
        ConvArgs u = conv_args(R.c1, act, B, Lc, -6 * dil[j], dil[j], Lc, 1, Lc);
        u.bias = R.c2.bias;
        u.Yf = X32;
        u.R = X32;
        u.Yh = other;
        u.act = ACT_SNAKE;
        u.act_a = nx.ea;
        u.act_b = nx.ib;
        const ConvFuse fu{R.c2.w, R.c1.bias, R.a2.ea, R.a2.ib};
        launch_unit(u, fu, st);
        std::swap(act, other);
        continue;
      }
      ConvArgs c1 = conv_args(R.c1, act, B, Lc, -6 * dil[j], dil[j], Lc, 1, Lc);
      c1.Yh = Hh;
      c1.act = ACT_SNAKE;
      c1.act_a = R.a2.ea;
      c1.act_b = R.a2.ib;
      launch_conv(c1, 1, st);
      ConvArgs c2 = conv_args(R.c2, Hh, B, Lc, 0, 1, Lc, 1, Lc);
      c2.Yf = X32;
      c2.R = X32;
      c2.Yh = act;  // overwrites snake1(x), consumed by c1 above
      c2.act = ACT_SNAKE;
      c2.act_a = nx.ea;
      c2.act_b = nx.ib;
      launch_conv(c2, 1, st);
    }
  }
  const int C = c->stages.back().cout;
  if (C % 8 || C > 192) FAIL(Q3T_INVALID_INPUT, "codec output conv: %d channels (multiple of 8, <= 192 supported)", C);
  {
    dim3 grid((Lc + kOutTile - 1) / kOutTile, B);
    k_out_conv<<<grid, kOutTile, 0, st>>>(act, Lc, C, c->out_w, c->out_b, d_wave, d_pcm);
    CK(cudaGetLastError());
    g_launches++;
  }
}

static void check_codes(const CodecModel *c, const int64_t *codes, int64_t n) {
  for (int64_t i = 0; i < n; i++)
    if (codes[i] < 0 || codes[i] >= c->c.codebook_size)
      FAIL(Q3T_INVALID_INPUT, "codec code %lld at %lld outside [0, %d)", (long long)codes[i], (long long)i,
           c->c.codebook_size);
}

// device time of the calling thread's last q3t_codec_decode (codes on the
// device -> samples on the device)
static thread_local float g_codec_ms = 0.f;

void codec_decode_host_codes(q3t_model *m, const int64_t *codes, int B, int T, float *wave, int16_t *pcm,
                             cudaStream_t st) {
  CodecModel *c = m->codec;
  if (!c) FAIL(Q3T_INVALID_INPUT, "model has no codec");
  if (B <= 0 || T <= 0) FAIL(Q3T_INVALID_INPUT, "codec decode needs B > 0 and T > 0");
  const int64_t ncodes = (int64_t)B * c->c.num_quantizers * T;
  check_codes(c, codes, ncodes);
  int64_t n = 0;
  codec_out_len(c, T, &n);
  if (n <= 0) FAIL(Q3T_INVALID_INPUT, "T = %d frames decode to no samples", T);
  int64_t *dc;
  float *dw = nullptr;
  int16_t *dp = nullptr;
  int *derr = nullptr, herr = 0;  // this call's convolution timeout word
  CK(cudaMallocAsync((void **)&dc, ncodes * 8, st));
  CK(cudaMallocAsync((void **)&derr, sizeof(int), st));
  CK(cudaMemsetAsync(derr, 0, sizeof(int), st));
  CK(cudaMemcpyAsync(dc, codes, ncodes * 8, cudaMemcpyHostToDevice, st));
  if (wave) CK(cudaMallocAsync((void **)&dw, (size_t)B * n * 4, st));
  if (pcm) CK(cudaMallocAsync((void **)&dp, (size_t)B * n * 2, st));
  cudaEvent_t e0, e1;
  CK(cudaEventCreate(&e0));
  CK(cudaEventCreate(&e1));
  CK(cudaEventRecord(e0, st));
  {
    ConvErrScope scope(derr);
    decode_device(c, dc, B, T, dw, dp, st);
  }
  CK(cudaEventRecord(e1, st));
  if (wave) CK(cudaMemcpyAsync(wave, dw, (size_t)B * n * 4, cudaMemcpyDeviceToHost, st));
  if (pcm) CK(cudaMemcpyAsync(pcm, dp, (size_t)B * n * 2, cudaMemcpyDeviceToHost, st));
  CK(cudaMemcpyAsync(&herr, derr, sizeof(int), cudaMemcpyDeviceToHost, st));
  CK(cudaFreeAsync(dc, st));
  CK(cudaFreeAsync(derr, st));
  if (dw) CK(cudaFreeAsync(dw, st));
  if (dp) CK(cudaFreeAsync(dp, st));
  CK(cudaStreamSynchronize(st));
  CK(cudaEventElapsedTime(&g_codec_ms, e0, e1));
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  conv_check_err(herr, "codec decode");
}

extern "C" q3t_status q3t_codec_last_ms(float *ms) {
  if (!ms) return Q3T_INVALID_INPUT;
  *ms = g_codec_ms;
  return Q3T_OK;
}

// ---------------------------------------------------------------------------
// decode without allocation: the call's convolution timeout word, the codes,
// every intermediate buffer and the output samples are carved out of one
// file-scope device array.  Only the timeout word must start at zero (it is
// cleared on the caller's stream before the kernels); every other buffer is
// written by a kernel before a later kernel reads it.  Calls that overlap in
// time on one device (from any thread or stream) share the array and race.
// ---------------------------------------------------------------------------
constexpr int64_t kStaticScratchBytes = 48ll << 20;  // one 24-frame window at B = 1 needs 42.7 MiB
constexpr int kStaticMaxDevices = 64;
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];
static void *g_static_addr[kStaticMaxDevices];
static std::mutex g_static_mu;

// Device address of g_static_scratch on `dev` (the current device): looked up
// once per device, on the first call.
static unsigned char *static_scratch(int dev) {
  if (dev < 0 || dev >= kStaticMaxDevices) FAIL(Q3T_INVALID_INPUT, "device %d beyond %d", dev, kStaticMaxDevices);
  std::lock_guard<std::mutex> lk(g_static_mu);
  if (!g_static_addr[dev]) CK(cudaGetSymbolAddress(&g_static_addr[dev], g_static_scratch));
  return (unsigned char *)g_static_addr[dev];
}

static void codec_decode_static(q3t_model *m, const int64_t *codes, int B, int T, float *wave, int16_t *pcm,
                                cudaStream_t st) {
  CodecModel *c = m->codec;
  if (!c) FAIL(Q3T_INVALID_INPUT, "model has no codec");
  if (B <= 0 || T <= 0) FAIL(Q3T_INVALID_INPUT, "codec decode needs B > 0 and T > 0");
  const int64_t ncodes = (int64_t)B * c->c.num_quantizers * T;
  check_codes(c, codes, ncodes);
  int64_t n = 0;
  codec_out_len(c, T, &n);
  if (n <= 0) FAIL(Q3T_INVALID_INPUT, "T = %d frames decode to no samples", T);
  CodecScratch ws = codec_scratch(c, B, T);
  auto up = [](int64_t b) { return (b + 255) & ~(int64_t)255; };
  const int64_t err_b = 256, codes_b = up(ncodes * 8), wave_b = wave ? up(B * n * 4) : 0,
                pcm_b = pcm ? up(B * n * 2) : 0;
  int64_t need = err_b + codes_b + wave_b + pcm_b;
  for (int i = 0; i < CodecScratch::N; i++) need += up(ws.bytes[i]);
  if (need > kStaticScratchBytes)
    FAIL(Q3T_INVALID_INPUT,
         "static codec decode of B = %d x T = %d frames needs %lld bytes of scratch; the static array holds %lld "
         "(about 26 frames in total)",
         B, T, (long long)need, (long long)kStaticScratchBytes);
  unsigned char *base = static_scratch(m->device);
  int *derr = (int *)base;
  int64_t off = err_b;
  int64_t *dc = (int64_t *)(base + off);
  off += codes_b;
  float *dw = wave ? (float *)(base + off) : nullptr;
  off += wave_b;
  int16_t *dp = pcm ? (int16_t *)(base + off) : nullptr;
  off += pcm_b;
  for (int i = 0; i < CodecScratch::N; i++) {
    ws.p[i] = base + off;
    off += up(ws.bytes[i]);
  }
  int herr = 0;
  CK(cudaMemsetAsync(derr, 0, sizeof(int), st));
  CK(cudaMemcpyAsync(dc, codes, ncodes * 8, cudaMemcpyHostToDevice, st));
  {
    ConvErrScope scope(derr);
    decode_with(c, ws, dc, B, T, dw, dp, st);
  }
  if (wave) CK(cudaMemcpyAsync(wave, dw, (size_t)B * n * 4, cudaMemcpyDeviceToHost, st));
  if (pcm) CK(cudaMemcpyAsync(pcm, dp, (size_t)B * n * 2, cudaMemcpyDeviceToHost, st));
  CK(cudaMemcpyAsync(&herr, derr, sizeof(int), cudaMemcpyDeviceToHost, st));
  CK(cudaStreamSynchronize(st));
  conv_check_err(herr, "static codec decode");
}

// ---------------------------------------------------------------------------
// chunked streaming inside a batch (codec_mode 2): every chunk_frames frames a
// window of up to left_context + chunk_frames frames of the request's codes
// is decoded and the samples of its newest chunk are emitted.  With the
// reference's non-causal pre-transformer this is an approximation of the
// full-sequence decode (no reference counterpart; new mode).
//
// The windows of step n decode on a second, lowest-priority stream while the
// (highest-priority) batch stream runs step n + 1's talker / predictor
// kernels, which are latency bound and leave most of the GPU idle.  The
// window codes are gathered on the batch stream at the end of step n (so a
// slot that a later step reuses cannot change them); the decode is launched
// right after step n + 1's frame is enqueued, so the host issues those
// launches while the frame runs; samples go to a pinned staging buffer, and
// the codec call at the end of step n + 1 joins the work: host wait, a
// device-side wait of the batch stream, copies into the requests' sample
// vectors and the sample counts.  A step in which a request finishes
// launches and joins at once, so a retired request's output is complete.
// ---------------------------------------------------------------------------
struct StreamOut {
  Req *r;
  int64_t src, dst, n;  // staging offset, offset in r->wave, samples
};
struct StreamState {
  std::map<int64_t, int> emitted;  // request id -> frames emitted
  int64_t *d_codes = nullptr;      // gathered windows of one step, back to back
  float *d_wave = nullptr;         // their samples, back to back
  float *h_wave = nullptr;         // pinned staging of the emitted samples
  size_t codes_cap = 0, wave_cap = 0;
  cudaStream_t cst = nullptr;
  cudaEvent_t ev_codes = nullptr, ev_done = nullptr;
  std::vector<StreamOut> out;      // emitted by the work in flight
  bool inflight = false;
  struct PendWin {
    Req *r;
    int64_t s0, n, dst;             // samples [s0, s0 + n) of the window's decode, offset in r->wave
  };
  struct PendGroup {
    int Tw, Bw;
    int64_t nout;
    int64_t *dc;
    float *dw;
    std::vector<PendWin> w;
  };
  std::vector<PendGroup> pend;     // gathered windows whose decode is not launched yet
  int *d_err = nullptr;            // the batch's convolution timeout word
  int *h_err = nullptr;            // its pinned copy, taken with the work
};
static std::map<q3t_batch *, StreamState> g_streams;

static void stream_capacity(StreamState &S, size_t codes, size_t wave) {
  if (S.codes_cap < codes) {
    if (S.d_codes) CK(cudaFree(S.d_codes));
    S.codes_cap = codes;
    CK(cudaMalloc(&S.d_codes, S.codes_cap * 8));
  }
  if (S.wave_cap < wave) {
    if (S.d_wave) CK(cudaFree(S.d_wave));
    if (S.h_wave) CK(cudaFreeHost(S.h_wave));
    S.wave_cap = wave;
    CK(cudaMalloc(&S.d_wave, S.wave_cap * 4));
    CK(cudaHostAlloc(&S.h_wave, S.wave_cap * 4, cudaHostAllocDefault));
  }
}

// Sizes the buffers for max_active windows of left_context + chunk_frames
// frames and runs one decode of each window length the stream uses
// (chunk_frames for a request's first window, left_context + chunk_frames
// after) on the codec stream, so its workspace pool and the kernels are set
// up before the first chunk is due rather than inside a step.
void codec_stream_init(q3t_model *m, q3t_batch *b) {
  StreamState S;
  CodecModel *c = m->codec;
  const int chunk = std::max(1, b->desc.chunk_frames), ctx = std::max(0, b->desc.left_context);
  const int Bw = std::max(1, b->A), nq = c->c.num_quantizers;
  int least = 0, greatest = 0;
  CK(cudaDeviceGetStreamPriorityRange(&least, &greatest));
  CK(cudaStreamCreateWithPriority(&S.cst, cudaStreamNonBlocking, least));
  CK(cudaEventCreateWithFlags(&S.ev_codes, cudaEventDisableTiming));
  CK(cudaEventCreateWithFlags(&S.ev_done, cudaEventDisableTiming));
  int64_t nmax = 0;
  codec_out_len(c, chunk + ctx, &nmax);
  stream_capacity(S, (size_t)Bw * nq * (chunk + ctx), (size_t)Bw * std::max<int64_t>(nmax, 1));
  CK(cudaMalloc(&S.d_err, sizeof(int)));
  CK(cudaMemsetAsync(S.d_err, 0, sizeof(int), S.cst));
  CK(cudaHostAlloc(&S.h_err, sizeof(int), cudaHostAllocDefault));
  *S.h_err = 0;
  g_streams[b] = S;  // codec_stream_free releases it if the warm-up below fails
  {
    ConvErrScope scope(S.d_err);
    for (int Tw : {chunk, chunk + ctx}) {
      int64_t nout = 0;
      codec_out_len(c, Tw, &nout);
      if (nout <= 0) continue;
      CK(cudaMemsetAsync(S.d_codes, 0, (size_t)Bw * nq * Tw * 8, S.cst));
      decode_device(c, S.d_codes, Bw, Tw, S.d_wave, nullptr, S.cst);
    }
  }
  CK(cudaMemcpyAsync(S.h_err, S.d_err, sizeof(int), cudaMemcpyDeviceToHost, S.cst));
  CK(cudaStreamSynchronize(S.cst));
  const int e = *S.h_err;
  *S.h_err = 0;
  CK(cudaMemsetAsync(S.d_err, 0, sizeof(int), S.cst));
  conv_check_err(e, "streaming codec warm-up");
}

// Completes the codec work in flight (see above); samples (nullable) counts
// the samples it emitted.
// Launches the decode of the windows gathered by the last codec_stream_step
// on the codec stream (after their gather on the batch stream).
void codec_stream_launch(q3t_batch *b) {
  auto it = g_streams.find(b);
  if (it == g_streams.end() || it->second.pend.empty()) return;
  StreamState &S = it->second;
  CodecModel *c = b->m->codec;
  CK(cudaStreamWaitEvent(S.cst, S.ev_codes, 0));
  size_t hoff = 0;
  ConvErrScope scope(S.d_err);
  for (const auto &g : S.pend) {
    if (g.nout > 0) decode_device(c, g.dc, g.Bw, g.Tw, g.dw, nullptr, S.cst);
    for (int i = 0; i < (int)g.w.size(); i++) {
      const auto &w = g.w[i];
      if (w.n <= 0) continue;
      if (b->desc.keep_output) {
        CK(cudaMemcpyAsync(S.h_wave + hoff, g.dw + (size_t)i * g.nout + w.s0, w.n * 4, cudaMemcpyDeviceToHost,
                           S.cst));
        b->d2h += w.n * 4;
      }
      S.out.push_back(StreamOut{w.r, (int64_t)hoff, w.dst, w.n});
      if (b->desc.keep_output) hoff += w.n;
    }
  }
  S.pend.clear();
  CK(cudaMemcpyAsync(S.h_err, S.d_err, sizeof(int), cudaMemcpyDeviceToHost, S.cst));
  CK(cudaEventRecord(S.ev_done, S.cst));
  S.inflight = true;
}

void codec_stream_join(q3t_batch *b, int64_t *samples) {
  codec_stream_launch(b);
  auto it = g_streams.find(b);
  if (it == g_streams.end() || !it->second.inflight) return;
  StreamState &S = it->second;
  CK(cudaEventSynchronize(S.ev_done));
  CK(cudaStreamWaitEvent(b->st, S.ev_done, 0));
  if (*S.h_err) {
    const int e = *S.h_err;
    *S.h_err = 0;
    S.out.clear();
    S.inflight = false;
    CK(cudaMemsetAsync(S.d_err, 0, sizeof(int), S.cst));
    conv_check_err(e, "streaming codec");
  }
  for (const StreamOut &o : S.out) {
    if (b->desc.keep_output) memcpy(o.r->wave.data() + o.dst, S.h_wave + o.src, (size_t)o.n * 4);
    o.r->samples += o.n;
    if (samples) *samples += o.n;
  }
  S.out.clear();
  S.inflight = false;
}

void codec_stream_free(q3t_batch *b) {
  auto it = g_streams.find(b);
  if (it == g_streams.end()) return;
  StreamState &S = it->second;
  S.pend.clear();  // gathered but never decoded: the batch is going away
  if (S.inflight) cudaEventSynchronize(S.ev_done);
  if (S.cst) cudaStreamSynchronize(S.cst);
  if (S.d_codes) cudaFree(S.d_codes);
  if (S.d_wave) cudaFree(S.d_wave);
  if (S.h_wave) cudaFreeHost(S.h_wave);
  if (S.h_err) cudaFreeHost(S.h_err);
  if (S.d_err) cudaFree(S.d_err);
  if (S.ev_codes) cudaEventDestroy(S.ev_codes);
  if (S.ev_done) cudaEventDestroy(S.ev_done);
  if (S.cst) cudaStreamDestroy(S.cst);
  g_streams.erase(it);
}

__global__ void k_window_codes(const int64_t *hist, int maxF, int G, int nq, int slot, int f0, int Tw, int64_t *out) {
  // hist [slot][frame][G] -> out [nq][Tw]
  for (int e = threadIdx.x + blockIdx.x * blockDim.x; e < nq * Tw; e += gridDim.x * blockDim.x) {
    const int q = e / Tw, t = e - q * Tw;
    out[e] = hist[((size_t)slot * maxF + f0 + t) * G + q];
  }
}

void codec_stream_step(q3t_model *m, q3t_batch *b, const std::vector<Req *> &act, int64_t *samples) {
  CodecModel *c = m->codec;
  codec_stream_join(b, samples);  // the previous step's windows
  auto &S = g_streams[b];
  const int chunk = std::max(1, b->desc.chunk_frames), ctx = std::max(0, b->desc.left_context);
  const int nq = c->c.num_quantizers;
  int64_t spf = 1;  // samples per frame (1920 at the default rates)
  for (int i = 0; i < c->c.num_upsampling_ratios; i++) spf *= c->c.upsampling_ratios[i];
  for (int i = 0; i < c->c.num_upsample_rates; i++) spf *= c->c.upsample_rates[i];
  struct Win {
    Req *r;
    int e, n, f0;
    int64_t s0, s1, dst;  // emitted samples [s0, s1) of the window's decode, offset in r->wave
  };
  std::vector<Win> wins;
  auto add = [&](Req *r, int e, int n) {
    const int f0 = std::max(0, e - ctx), Tw = e + n - f0;
    int64_t nout = 0;
    codec_out_len(c, Tw, &nout);
    // window-relative frames [e - f0, e - f0 + n) map to samples shifted by
    // the trim deficit (555 at the default rates), so consecutive chunks tile
    // the full-length output
    const int64_t deficit = spf * Tw - nout, a0 = e - f0;
    const int64_t s0 = a0 > 0 ? std::min<int64_t>(nout, a0 * spf - deficit) : 0;
    const int64_t s1 = std::min<int64_t>(nout, (a0 + n) * spf - deficit);
    wins.push_back(Win{r, e, n, f0, s0, s1, 0});
  };
  // every request emits each chunk as soon as its frames exist; a finished
  // request emits the frames it still owes
  for (Req *r : act) {
    int e = S.emitted[r->id];
    const int avail = r->step_idx;
    while (avail - e >= chunk || (r->finished && avail > e)) {
      const int n = std::min(chunk, avail - e);
      add(r, e, n);
      e += n;
    }
  }
  for (Req *r : act)
    if (r->finished) S.emitted.erase(r->id);
  if (wins.empty()) return;
  for (Win &w : wins) {  // a request's windows were added in time order
    if (!w.r->finished) S.emitted[w.r->id] = w.e + w.n;
    if (w.s1 > w.s0 && b->desc.keep_output) {
      w.dst = (int64_t)w.r->wave.size();
      w.r->wave.resize(w.r->wave.size() + (w.s1 - w.s0));
    }
  }
  std::map<int, std::vector<int>> groups;  // window length -> windows
  for (int i = 0; i < (int)wins.size(); i++) groups[wins[i].e + wins[i].n - wins[i].f0].push_back(i);
  size_t need_codes = 0, need_wave = 0;
  for (auto &kv : groups) {
    int64_t nout = 0;
    codec_out_len(c, kv.first, &nout);
    need_codes += kv.second.size() * (size_t)nq * kv.first;
    need_wave += kv.second.size() * (size_t)std::max<int64_t>(nout, 1);
  }
  stream_capacity(S, need_codes, need_wave);  // nothing is in flight here
  size_t coff = 0, woff = 0;
  for (auto &kv : groups) {
    const int Tw = kv.first, Bw = (int)kv.second.size();
    int64_t nout = 0;
    codec_out_len(c, Tw, &nout);
    StreamState::PendGroup g{Tw, Bw, nout, S.d_codes + coff, S.d_wave + woff, {}};
    for (int i = 0; i < Bw; i++) {
      const Win &w = wins[kv.second[i]];
      k_window_codes<<<8, 256, 0, b->st>>>(b->d_hist_codes, b->maxF, b->G, nq, w.r->slot, w.f0, Tw,
                                           g.dc + (size_t)i * nq * Tw);
      CK(cudaGetLastError());
      g_launches++;
      g.w.push_back(StreamState::PendWin{w.r, w.s0, std::max<int64_t>(0, w.s1 - w.s0), w.dst});
    }
    S.pend.push_back(std::move(g));
    coff += (size_t)Bw * nq * Tw;
    woff += (size_t)Bw * std::max<int64_t>(nout, 1);
  }
  CK(cudaEventRecord(S.ev_codes, b->st));
  // The decode is launched by the next step right after its frame is
  // enqueued (codec_stream_launch), so these launches overlap that frame on
  // the device instead of delaying it; a step in which a request finishes
  // decodes and joins now.
  static const bool serial = getenv("Q3T_CODEC_SERIAL") != nullptr;  // no overlap (A/B measurements)
  bool join = serial;
  for (Req *r : act) join |= r->finished;  // retired after this call: its last samples must be in place
  if (join) codec_stream_join(b, samples);  // launches, then waits
}

}  // namespace q3t

using namespace q3t;

extern "C" q3t_status q3t_codec_out_len(const q3t_model *m, int T, int64_t *n) {
  if (!m || !n || T <= 0 || !m->has_codec || !m->codec) {
    set_error("q3t_codec_out_len: model has no codec or T <= 0");
    return Q3T_INVALID_INPUT;
  }
  codec_out_len(m->codec, T, n);
  return Q3T_OK;
}

extern "C" q3t_status q3t_codec_decode(q3t_model *m, const int64_t *codes, int B, int T, float *wave, int16_t *pcm,
                                       int64_t *n) {
  if (!m || !codes) {
    set_error("q3t_codec_decode: null argument");
    return Q3T_INVALID_INPUT;
  }
  try {
    CK(cudaSetDevice(m->device));
    if (!m->has_codec || !m->codec) FAIL(Q3T_INVALID_INPUT, "model has no codec");
    int64_t len = 0;
    codec_out_len(m->codec, T > 0 ? T : 1, &len);
    if (n) *n = len;
    cudaStream_t st;
    CK(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    try {
      codec_decode_host_codes(m, codes, B, T, wave, pcm, st);
    } catch (...) {
      cudaStreamDestroy(st);
      throw;
    }
    CK(cudaStreamDestroy(st));
    return Q3T_OK;
  } catch (const Status &s) {
    return s.code;
  } catch (const CudaFail &c) {
    set_error("CUDA error %s (%s) in %s", cudaGetErrorName(c.err), cudaGetErrorString(c.err), c.what.c_str());
    return Q3T_CUDA_ERROR;
  }
}

extern "C" q3t_status q3t_codec_decode_static(q3t_model *m, const int64_t *codes, int B, int T, float *wave,
                                              int16_t *pcm, int64_t *n, void *stream) {
  if (!m || !codes) {
    set_error("q3t_codec_decode_static: null argument");
    return Q3T_INVALID_INPUT;
  }
  // the calling thread's current device is put back on every return
  struct DeviceRestore {
    int dev = -1;
    DeviceRestore() {
      if (cudaGetDevice(&dev) != cudaSuccess) dev = -1;
    }
    ~DeviceRestore() {
      if (dev >= 0) cudaSetDevice(dev);
    }
  } restore;
  try {
    CK(cudaSetDevice(m->device));
    if (!m->has_codec || !m->codec) FAIL(Q3T_INVALID_INPUT, "model has no codec");
    int64_t len = 0;
    codec_out_len(m->codec, T > 0 ? T : 1, &len);
    if (n) *n = len;
    codec_decode_static(m, codes, B, T, wave, pcm, (cudaStream_t)stream);
    return Q3T_OK;
  } catch (const Status &s) {
    return s.code;
  } catch (const CudaFail &c) {
    set_error("CUDA error %s (%s) in %s", cudaGetErrorName(c.err), cudaGetErrorString(c.err), c.what.c_str());
    return Q3T_CUDA_ERROR;
  }
}

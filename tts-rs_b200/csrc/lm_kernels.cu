// Talker / code-predictor kernels for sm_100a.
//
// One decoder layer of tts_qwen3_tts/src/model/talker/network/layer.rs:23-44
// runs as five kernels:
//   gemm(Wqkv)  X = RMSNorm(x) (from the previous layer's sum-of-squares
//               partials); epilogue q/k RMSNorm + RoPE, q -> bf16, K/V
//               appended to the paged cache
//   attention   split-K flash-decoding over the pages
//   gemm(Wo)    epilogue x += o, sum-of-squares partials of x
//   gemm(Wgu)   X = RMSNorm(x); epilogue silu(gate) * up -> bf16
//   gemm(Wdown) epilogue x += down, sum-of-squares partials of x
// Every kernel is PDL-aware: a GEMM's weight stream is issued before
// griddepcontrol.wait, and each kernel lets its dependent launch early.
// Sums run in a fixed order, so results are deterministic.
#include <cstdlib>
#include <utility>

#include <cudaTypedefs.h>

#include "lm_device.cuh"
#include "umma.cuh"

namespace q3t {

bool g_use_pdl = true;
int64_t g_launches = 0;
cudaError_t g_launch_err = cudaSuccess;
const char *g_launch_err_kernel = "";

cudaError_t take_launch_error(const char **kernel) {
  cudaError_t e = g_launch_err;
  if (kernel) *kernel = g_launch_err_kernel;
  g_launch_err = cudaSuccess;
  return e;
}

static void note(cudaError_t e, const char *what) {
  if (e != cudaSuccess && g_launch_err == cudaSuccess) {
    g_launch_err = e;
    g_launch_err_kernel = what;
  }
}

void note_launch(cudaError_t e, const char *what) { note(e, what); }

// ---------------------------------------------------------------------------
// Launch trace (see lm_kernels.cuh)
// ---------------------------------------------------------------------------
__device__ TraceRec *g_trace = nullptr;
__device__ unsigned g_trace_n = 0;
__device__ unsigned g_trace_cap = 0;
static TraceRec *h_trace_buf = nullptr;

Q3T_DEV unsigned long long gclock() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// thread 0 of a CTA: append the record (no-op when tracing is off)
Q3T_DEV void trace_put(TraceRec *buf, int kind, const unsigned long long *t, int n, int k) {
  if (!buf) return;
  const unsigned i = atomicAdd(&g_trace_n, 1u);
  if (i >= g_trace_cap) return;
  TraceRec r;
  asm volatile("mov.u64 %0, %%gridid;" : "=l"(r.grid));
#pragma unroll
  for (int j = 0; j < 7; j++) r.t[j] = t[j];
  r.kind = kind;
  r.cta = (int)(blockIdx.x + blockIdx.y * gridDim.x);
  r.n = n;
  r.k = k;
  buf[i] = r;
}

bool trace_start(size_t cap, cudaStream_t st) {
  if (h_trace_buf) return false;
  if (cudaMalloc(&h_trace_buf, cap * sizeof(TraceRec)) != cudaSuccess) {
    h_trace_buf = nullptr;
    return false;
  }
  const unsigned zero = 0, c = (unsigned)cap;
  cudaMemcpyToSymbolAsync(g_trace_n, &zero, 4, 0, cudaMemcpyHostToDevice, st);
  cudaMemcpyToSymbolAsync(g_trace_cap, &c, 4, 0, cudaMemcpyHostToDevice, st);
  cudaMemcpyToSymbolAsync(g_trace, &h_trace_buf, sizeof(void *), 0, cudaMemcpyHostToDevice, st);
  return cudaStreamSynchronize(st) == cudaSuccess;
}

void trace_stop(std::vector<TraceRec> &out, cudaStream_t st) {
  if (!h_trace_buf) return;
  TraceRec *none = nullptr;
  unsigned n = 0, cap = 0;
  cudaMemcpyToSymbolAsync(g_trace, &none, sizeof(void *), 0, cudaMemcpyHostToDevice, st);
  cudaMemcpyFromSymbolAsync(&n, g_trace_n, 4, 0, cudaMemcpyDeviceToHost, st);
  cudaMemcpyFromSymbolAsync(&cap, g_trace_cap, 4, 0, cudaMemcpyDeviceToHost, st);
  cudaStreamSynchronize(st);
  out.resize(n < cap ? n : cap);
  cudaMemcpy(out.data(), h_trace_buf, out.size() * sizeof(TraceRec), cudaMemcpyDeviceToHost);
  cudaFree(h_trace_buf);
  h_trace_buf = nullptr;
}

template <typename... KArgs, typename... Args>
static void launch(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = g_use_pdl ? 1 : 0;
  note(cudaLaunchKernelEx(&cfg, k, std::forward<Args>(args)...), "kernel launch");
  g_launches++;
}

// ---------------------------------------------------------------------------
// Weight packing: W [N][K] row-major -> one 512-byte m16n8k16 A fragment per
// (16-row block rb, 16-column block kb), tiles ordered rb-major so a K-range
// of one row block is one contiguous stream.  Lane l of the warp finds its 4
// A registers at bytes [16 l, 16 l + 16) of the tile (PTX ISA fragment
// layout for mma.m16n8k16 .bf16 A: rows g, g+8, columns 2t..2t+1, +8).
// ---------------------------------------------------------------------------
__global__ void k_pack(const uint16_t *__restrict__ src, uint16_t *__restrict__ dst, int N, int K) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int kbs = K / 16;
  const int64_t ntiles = (int64_t)(N / 16) * kbs;
  if (idx >= ntiles * 32) return;
  const int lane = (int)(idx & 31);
  const int64_t tile = idx >> 5;
  const int rb = (int)(tile / kbs), kb = (int)(tile % kbs);
  const int g = lane >> 2, t = lane & 3;
  const uint16_t *r0 = src + (size_t)(rb * 16 + g) * K + kb * 16;
  const uint16_t *r1 = r0 + (size_t)8 * K;
  uint16_t *d = dst + tile * 256 + lane * 8;
  d[0] = r0[2 * t];
  d[1] = r0[2 * t + 1];
  d[2] = r1[2 * t];
  d[3] = r1[2 * t + 1];
  d[4] = r0[2 * t + 8];
  d[5] = r0[2 * t + 9];
  d[6] = r1[2 * t + 8];
  d[7] = r1[2 * t + 9];
}

void pack_weight(const uint16_t *src, uint16_t *dst, int N, int K, cudaStream_t st) {
  int64_t n = (int64_t)(N / 16) * (K / 16) * 32;
  k_pack<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(src, dst, N, K);
  note(cudaGetLastError(), "k_pack");
  g_launches++;
}

__global__ void k_f32_to_bf16(const float *__restrict__ s, uint16_t *__restrict__ d, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    d[i] = f2bf(s[i]);
}

void f32_to_bf16(const float *src, uint16_t *dst, int64_t n, cudaStream_t st) {
  k_f32_to_bf16<<<1184, 256, 0, st>>>(src, dst, n);
  note(cudaGetLastError(), "k_f32_to_bf16");
  g_launches++;
}

// ---------------------------------------------------------------------------
// standalone kernels
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_rmsnorm(RmsArgs a) {
  __shared__ float red[33];
  TraceRec *trb = threadIdx.x == 0 ? g_trace : nullptr;
  unsigned long long tst[7] = {0, 0, 0, 0, 0, 0, 0};
  if (trb) tst[0] = gclock();
  pdl_wait();
  pdl_launch();
  if (trb) tst[1] = gclock();
  d_rmsnorm(a, blockIdx.x, red);
  if (trb) {
    tst[6] = gclock();
    trace_put(trb, 1, tst, 0, 0);
  }
}

RmsArgs rms_args(float *x, int ldx, int row_mul, int row_add, Part add, const float *gamma, uint16_t *out, int ldo,
                 int H, float eps, const int *ntok, float *out_f32, const int *slot) {
  RmsArgs a{};
  a.x = x;
  a.ldx = ldx;
  a.row_mul = row_mul;
  a.row_add = row_add;
  a.add = add;
  a.gamma = gamma;
  a.out = out;
  a.ldo = ldo;
  a.H = H;
  a.eps = eps;
  a.ntok = ntok;
  a.out_f32 = out_f32;
  a.slot = slot;
  return a;
}

void rmsnorm(const RmsArgs &a, int grid_rows, cudaStream_t st) {
  launch(k_rmsnorm, dim3(grid_rows), dim3(256), 0, st, a);
}

void rmsnorm(float *x, int ldx, int row_mul, int row_add, Part add, const float *gamma, uint16_t *out, int ldo, int H,
             float eps, const int *ntok, int grid_rows, float *out_f32, const int *slot, cudaStream_t st) {
  rmsnorm(rms_args(x, ldx, row_mul, row_add, add, gamma, out, ldo, H, eps, ntok, out_f32, slot), grid_rows, st);
}

// ---------------------------------------------------------------------------
// Cluster split-K GEMM on the 5th-generation tensor cores (GemmArgs in
// lm_kernels.cuh).  A CTA owns one 128-row output block and the cluster
// rank's K range (KA atoms of 64) for up to N = 8*NT tokens:
//   - one thread issues the TMA loads of its weight tile (K-major,
//     SWIZZLE_128B) before griddepcontrol.wait, so the weight stream overlaps
//     the end of the previous kernel;
//   - X arrives by TMA (bf16 rows) or is staged by all threads from the f32
//     residual rows, RMS-normalised and rounded to bf16, straight into the
//     swizzled operand layout;
//   - the same thread issues KA*4 tcgen05.mma (M = 128, N, K = 16) into a
//     TMEM accumulator and commits them to an mbarrier;
//   - warps 0..3 read the accumulator back (tcgen05.ld, one row per thread)
//     into an f32 tile [token][row] over the consumed weight tile; after a
//     cluster barrier CTA rank c sums token slice c of all ranks' tiles
//     through distributed shared memory (rank order) and runs the epilogue,
//     one warp per token, lane = 4 consecutive rows.
// Every mbarrier wait is bounded; a timeout sets a bit in *err and the kernel
// still runs to completion with the same barriers, so a cluster never hangs.
// ---------------------------------------------------------------------------
constexpr int kTileLd = 132;  // f32 pitch of the reduction tile
constexpr int kMaxNss = 16;   // sum-of-squares partials per row (hidden <= 2048)

template <int NT, int KA>
struct GemmSmem {
  static constexpr int N = NT * 8;
  static constexpr int kW = KA * 16384;   // weight tile: KA atoms of 128 rows x 128 B
  static constexpr int kXAtom = N * 128;  // one X atom: N rows x 128 B
  static constexpr int kTile = N * kTileLd * 4;
  static constexpr int kR0 = kW > kTile ? kW : (kTile + 1023) / 1024 * 1024;
  static constexpr int kX = KA * kXAtom;
  static constexpr int kMisc = 1024;       // mbarriers, TMEM slot, rms, token metadata
  static constexpr size_t kBytes = (size_t)kR0 + kX + kMisc + 1024;  // + alignment slack
};

Q3T_DEV void store_bf16x4(uint16_t *dst, float a, float b, float c, float d) {
  uint2 p;
  p.x = pack_bf16x2(a, b);
  p.y = pack_bf16x2(c, d);
  *reinterpret_cast<uint2 *>(dst) = p;
}

// rows rg*128 + 4*lane .. +3 of token t (warp-wide: the norms reduce over the
// warp); tm = {position, page} of t for GE_QKV; xpre = the residual rows
// already loaded for GE_RESID when have_pre
Q3T_DEV void gemm_epilogue(const GemmArgs &a, int t, int rg, int lane, float4 v, const int *tm, float4 xpre,
                           bool have_pre, float4 gqk, float4 fr) {
  const int n = rg * 128 + lane * 4;
  if (a.epi == GE_F32) {
    *reinterpret_cast<float4 *>(a.y + (size_t)t * a.ldy + n) = v;
  } else if (a.epi == GE_RESID) {
    float4 *xp = reinterpret_cast<float4 *>(a.y + (size_t)t * a.ldy + n);
    float4 x = have_pre ? xpre : *xp;
    x.x += v.x;
    x.y += v.y;
    x.z += v.z;
    x.w += v.w;
    *xp = x;
    if (a.xg_out)  // gqk holds this lane's xg_gamma
      store_bf16x4(a.xg_out + (size_t)t * a.ldy + n, x.x * gqk.x, x.y * gqk.y, x.z * gqk.z, x.w * gqk.w);
    const float ss = warp_sum(x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w);
    if (lane == 0) a.ss_out[(size_t)rg * a.ss_ld + t] = ss;
  } else if (a.epi == GE_BIAS_SILU || a.epi == GE_BIAS_BF16) {
    const float4 b = *reinterpret_cast<const float4 *>(a.bias + n);
    const float y0 = v.x + b.x, y1 = v.y + b.y, y2 = v.z + b.z, y3 = v.w + b.w;
    if (a.epi == GE_BIAS_SILU)
      store_bf16x4(a.h + (size_t)t * a.ldh + n, silu(y0), silu(y1), silu(y2), silu(y3));
    else
      *reinterpret_cast<float4 *>(a.y + (size_t)t * a.ldy + n) =
          make_float4(bf16_round(y0), bf16_round(y1), bf16_round(y2), bf16_round(y3));
  } else if (a.epi == GE_SILU) {
    const float ux = __shfl_xor_sync(0xffffffffu, v.x, 16), uy = __shfl_xor_sync(0xffffffffu, v.y, 16);
    const float uz = __shfl_xor_sync(0xffffffffu, v.z, 16), uw = __shfl_xor_sync(0xffffffffu, v.w, 16);
    if (lane < 16)
      store_bf16x4(a.h + (size_t)t * a.ldh + rg * 64 + lane * 4, silu(v.x) * ux, silu(v.y) * uy, silu(v.z) * uz,
                   silu(v.w) * uw);
  } else {  // GE_QKV: row block rg = q head rg | k head rg - nh | v head rg - nh - nkv
    const int pos = tm[0];
    float o[4];
    if (rg < a.nh) {
      norm_rope_reg(v, gqk, fr, a.eps, lane, pos, o);
      store_bf16x4(a.q + (size_t)t * a.nh * 128 + rg * 128 + lane * 4, o[0], o[1], o[2], o[3]);
      return;
    }
    const int h = rg < a.nh + a.nkv ? rg - a.nh : rg - a.nh - a.nkv;
    const size_t e = a.layer * a.kv.layer_stride + (((size_t)tm[1] * a.kv.n_kv + h) * 16 + (pos & 15)) * 128 + lane * 4;
    if (rg < a.nh + a.nkv) {
      norm_rope_reg(v, gqk, fr, a.eps, lane, pos, o);
      store_bf16x4(a.kv.k + e, o[0], o[1], o[2], o[3]);
    } else {
      store_bf16x4(a.kv.v + e, v.x, v.y, v.z, v.w);
    }
  }
}

template <int NT, int KA>
__global__ void __launch_bounds__(256, KA > 4 ? 1 : 2) k_gemm(const __grid_constant__ GemmArgs a) {
  using L = GemmSmem<NT, KA>;
  constexpr int N = L::N, KC = KA * 64;
  constexpr uint32_t kCols = N < 32 ? 32 : N;
  extern __shared__ unsigned char gsm_raw[];
  unsigned char *gsm = gsm_raw + ((1024 - (smem_addr(gsm_raw) & 1023)) & 1023);
  unsigned char *wsm = gsm, *xsm = gsm + L::kR0;
  float *tile = reinterpret_cast<float *>(gsm);  // after the MMA, over the weights
  uint64_t *bars = reinterpret_cast<uint64_t *>(xsm + L::kX);  // weights, X, MMA done
  uint32_t *tslot = reinterpret_cast<uint32_t *>(bars + 3);
  float *rms = reinterpret_cast<float *>(bars + 4);             // [64]
  int *meta = reinterpret_cast<int *>(rms + 64);                // [128]
  const int cs = a.cs, ks = blockIdx.x % cs, rg = blockIdx.x / cs;
  const int tok0 = blockIdx.y * N, k0 = ks * KC;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    mbar_init(&bars[2], 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(tslot, kCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  TraceRec *trb = threadIdx.x == 0 ? g_trace : nullptr;
  unsigned long long tst[7] = {0, 0, 0, 0, 0, 0, 0};
  if (trb) tst[0] = gclock();
  if (threadIdx.x == 0) {  // weights: independent of earlier kernels
    mbar_expect_tx(&bars[0], L::kW);
#pragma unroll
    for (int i = 0; i < KA; i++) tma_load_2d(wsm + i * 16384, &a.tw, k0 + 64 * i, rg * 128, &bars[0]);
  }
  // GX_NORM staging layout: a thread keeps one 8-column chunk (its gamma in
  // registers, loaded before the dependency wait: weights are never written)
  // and rows r0, r0 + rstep, ...
  constexpr int c8n = KC / 8, rstep = 256 / c8n, NR = (N + rstep - 1) / rstep;
  const int c8 = threadIdx.x % c8n, r0 = threadIdx.x / c8n;
  float4 g0 = make_float4(0.f, 0.f, 0.f, 0.f), g1 = g0;
  // GE_QKV: this lane's q_norm / k_norm gamma (by the row block's head) and
  // RoPE inverse frequencies, for the epilogue
  float4 gqk = g0, fr = g0;
  if (a.epi == GE_QKV && rg < a.nh + a.nkv) {
    gqk = *reinterpret_cast<const float4 *>((rg < a.nh ? a.q_norm : a.k_norm) + lane * 4);
    fr = *reinterpret_cast<const float4 *>(a.inv_freq + ((lane * 4) & 63));
  }
  if (a.epi == GE_RESID && a.xg_out) gqk = *reinterpret_cast<const float4 *>(a.xg_gamma + rg * 128 + lane * 4);
  if constexpr (KA <= 4) {
    if (a.xmode == GX_NORM && r0 < rstep) {
      g0 = *reinterpret_cast<const float4 *>(a.gamma + k0 + c8 * 8);
      g1 = *reinterpret_cast<const float4 *>(a.gamma + k0 + c8 * 8 + 4);
    }
  }
  // The token count, and for GE_QKV the position and page of this CTA's
  // epilogue tokens, come from host-written metadata and page tables, so
  // they load before the dependency wait.
  const int ts = (N + cs - 1) / cs, t_lo = ks * ts;
  int ntok = *a.ntok - tok0;
  ntok = ntok < 0 ? 0 : (ntok > N ? N : ntok);
  const int t_hi = min(t_lo + ts, ntok);
  if (a.epi == GE_QKV && (int)threadIdx.x < t_hi - t_lo) {
    const int t = tok0 + t_lo + threadIdx.x;
    const int pos = a.tv.pos[t] + a.tv.pos_add;
    meta[2 * threadIdx.x] = pos;
    meta[2 * threadIdx.x + 1] = a.kv.page_table[(size_t)a.tv.seq[t] * a.kv.pt_stride + (pos >> 4)];
  }
  pdl_wait();
  pdl_launch();
  if (trb) tst[1] = gclock();
  // Loads that do not wait for the token count: rows tok0 .. tok0 + N - 1 of
  // every activation buffer exist (buffers hold >= tok0 + N rows); rows at or
  // beyond the count are read but never used.
  // GE_RESID: the residual rows of this warp's first two epilogue tokens
  // (final once the previous kernel completed)
  float4 xres[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
  if (a.epi == GE_RESID) {
#pragma unroll
    for (int i = 0; i < 2; i++) {
      const int tt = t_lo + warp + 8 * i;
      if (tt < t_lo + ts && tt < N)
        xres[i] = *reinterpret_cast<const float4 *>(a.y + (size_t)(tok0 + tt) * a.ldy + rg * 128 + lane * 4);
    }
  }
  // GX_NORM: this thread's x rows and (thread r < N) row r's sum-of-squares partials
  float4 xv[KA <= 4 ? NR : 1][2];
  float ssp[kMaxNss];
  if constexpr (KA <= 4) {
    if (a.xmode == GX_NORM) {
#pragma unroll
      for (int i = 0; i < NR; i++) {
        const int r = r0 + i * rstep;
        xv[i][0] = xv[i][1] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (r0 < rstep && r < N) {
          const float *xr = a.x + (size_t)((tok0 + r) * a.xrow_mul + a.xrow_add) * a.ldx + k0 + c8 * 8;
          xv[i][0] = *reinterpret_cast<const float4 *>(xr);
          xv[i][1] = *reinterpret_cast<const float4 *>(xr + 4);
        }
      }
      if ((int)threadIdx.x < N) {
        const float *sp = a.ss + (size_t)(tok0 + threadIdx.x) * a.xrow_mul + a.xrow_add;
#pragma unroll
        for (int i = 0; i < kMaxNss; i++) ssp[i] = i < a.nss ? sp[(size_t)i * a.ss_ld] : 0.f;
      }
    }
  }
  if (a.xmode != GX_NORM) {
    if (threadIdx.x == 0) {
      mbar_expect_tx(&bars[1], L::kX);
#pragma unroll
      for (int i = 0; i < KA; i++) tma_load_2d(xsm + i * L::kXAtom, &a.tx, k0 + 64 * i, tok0, &bars[1]);
    }
    // GX_SCALED: 1 / rms of this CTA's epilogue tokens (partials summed in
    // index order, as GX_NORM does), for the epilogue; the barriers before
    // the MMA order these stores before their reads
    if (a.xmode == GX_SCALED && (int)threadIdx.x < t_hi - t_lo) {
      const float *sp = a.ss + (size_t)(tok0 + t_lo + threadIdx.x) * a.xrow_mul + a.xrow_add;
      float p[kMaxNss];
#pragma unroll
      for (int i = 0; i < kMaxNss; i++) p[i] = i < a.nss ? sp[(size_t)i * a.ss_ld] : 0.f;
      float sum = p[0];
#pragma unroll
      for (int i = 1; i < kMaxNss; i++) sum += p[i];
      rms[threadIdx.x] = 1.f / sqrtf(sum / (float)a.K + a.eps);
    }
  } else if constexpr (KA <= 4) {
    // the scale of each row, then x * (1 / rms) * gamma -> bf16 at chunk
    // (c ^ (row & 7)) of the row's 128-byte atom line
    if ((int)threadIdx.x < ntok) {
      float sum = ssp[0];
#pragma unroll
      for (int i = 1; i < kMaxNss; i++) sum += ssp[i];
      rms[threadIdx.x] = 1.f / sqrtf(sum / (float)a.K + a.eps);
    }
    __syncthreads();
    if (r0 < rstep) {
#pragma unroll
      for (int i = 0; i < NR; i++) {
        const int r = r0 + i * rstep;
        if (r >= N) break;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (r < ntok) {
          const float d = rms[r];
          v.x = pack_bf16x2(xv[i][0].x * d * g0.x, xv[i][0].y * d * g0.y);
          v.y = pack_bf16x2(xv[i][0].z * d * g0.z, xv[i][0].w * d * g0.w);
          v.z = pack_bf16x2(xv[i][1].x * d * g1.x, xv[i][1].y * d * g1.y);
          v.w = pack_bf16x2(xv[i][1].z * d * g1.z, xv[i][1].w * d * g1.w);
        }
        *reinterpret_cast<uint4 *>(xsm + (c8 >> 3) * L::kXAtom + r * 128 + (((c8 & 7) ^ (r & 7)) << 4)) = v;
      }
    }
    fence_proxy_async();
  }
  __syncthreads();
  if (trb) tst[2] = gclock();
  uint32_t err = 0;
  if (threadIdx.x == 0) {
    if (!mbar_wait(&bars[0], 0)) err |= 1u;
    if (a.xmode != GX_NORM && !mbar_wait(&bars[1], 0)) err |= 2u;
    tc_fence_after();
    constexpr uint32_t idesc = umma_idesc_bf16(128, N);
#pragma unroll
    for (int s = 0; s < KA * 4; s++) {
      const int at = s >> 2, off = (s & 3) * 32;
      umma_kf16(tmem, sw128_desc(wsm + at * 16384 + off), sw128_desc(xsm + at * L::kXAtom + off), idesc,
                s > 0 ? 1u : 0u);
    }
    umma_commit(&bars[2]);
    if (!mbar_wait(&bars[2], 0)) err |= 4u;  // the other threads block in the barrier below, not polling
    if (trb) tst[3] = gclock();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp < 4) {  // accumulator lane = output row, column = token
    const uint32_t tq = tmem + ((uint32_t)(32 * warp) << 16);
    const int row = 32 * warp + lane;
#pragma unroll
    for (int c0 = 0; c0 < N; c0 += 8) {
      float v[8];
      tmem_ld8(tq + c0, v);
#pragma unroll
      for (int j = 0; j < 8; j++) tile[(c0 + j) * kTileLd + row] = v[j];
    }
  }
  if (err && a.err) atomicOr(a.err, (int)err);
  tc_fence_before();
  if (cs > 1)
    cluster_sync();
  else
    __syncthreads();
  if (trb) tst[4] = gclock();
  for (int tt = t_lo + warp; tt < t_hi; tt += 8) {
    const float *src = tile + tt * kTileLd + 4 * lane;
    float4 v;
    if (cs == 1) {
      v = *reinterpret_cast<const float4 *>(src);
    } else {  // all remote loads in flight, then the sum in rank order
      float4 p[8];
#pragma unroll
      for (int c = 0; c < 8; c++)
        if (c < cs) p[c] = ld_cluster_f4(src, (uint32_t)c);
      v = p[0];
#pragma unroll
      for (int c = 1; c < 8; c++)
        if (c < cs) {
          v.x += p[c].x;
          v.y += p[c].y;
          v.z += p[c].z;
          v.w += p[c].w;
        }
    }
    if (a.xmode == GX_SCALED) {
      const float d = rms[tt - t_lo];
      v.x *= d;
      v.y *= d;
      v.z *= d;
      v.w *= d;
    }
    const int i = (tt - t_lo - warp) >> 3;
    gemm_epilogue(a, tok0 + tt, rg, lane, v, meta + 2 * (tt - t_lo), i == 0 ? xres[0] : xres[1], i < 2, gqk, fr);
  }
  if (trb) tst[5] = gclock();
  if (cs > 1) cluster_sync();  // no CTA leaves while another still reads its tile
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kCols);
  if (trb) {
    tst[6] = gclock();
    trace_put(trb, 2, tst, a.N, a.K);
  }
}

GemmArgs gemm_args(const Linear &W, const int *ntok, int max_tok) {
  GemmArgs a;
  memset(&a, 0, sizeof a);
  a.tw = W.tm;
  a.N = W.N;
  a.K = W.K;
  a.ntok = ntok;
  const int per = max_tok < 64 ? max_tok : 64;
  a.nt = per <= 8 ? 1 : (per <= 16 ? 2 : (per <= 32 ? 4 : 8));
  // smallest cluster that gives >= 128 CTAs (at most 8) whose K range is a
  // whole number of 64-wide atoms, then enough splits for <= 6 atoms per CTA
  const int groups = W.N / 128, atoms = W.K / 64;
  int cs = 1;
  while (cs < 8 && groups * cs < 128 && atoms % (2 * cs) == 0) cs *= 2;
  while (cs < 8 && atoms / cs > 6 && atoms % (2 * cs) == 0) cs *= 2;
  a.cs = cs;
  a.ldx = W.K;
  a.xrow_mul = 1;
  return a;
}

template <int NT, int KA>
static void gemm_launch(const GemmArgs &a, dim3 grid, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = GemmSmem<NT, KA>::kBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = a.cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = g_use_pdl ? 2 : 1;
  note(cudaLaunchKernelEx(&cfg, k_gemm<NT, KA>, a), "k_gemm");
  g_launches++;
}

template <int NT>
static void gemm_nt(const GemmArgs &a, dim3 grid, cudaStream_t st) {
  switch ((a.K / 64) / a.cs) {
    case 2: gemm_launch<NT, 2>(a, grid, st); break;
    case 4: gemm_launch<NT, 4>(a, grid, st); break;
    case 6: gemm_launch<NT, 6>(a, grid, st); break;
    default: note(cudaErrorInvalidValue, "k_gemm (K range per CTA must be 2, 4 or 6 atoms of 64)"); break;
  }
}

void gemm(const GemmArgs &a, int max_tok, cudaStream_t st) {
  const int atoms = a.K / 64;
  if (a.N % 128 || a.K % 64 || a.cs < 1 || a.cs > 8 || atoms % a.cs || max_tok < 1 ||
      (a.epi == GE_SILU && a.h == nullptr) || (a.xmode == GX_NORM && (a.x == nullptr || a.ss == nullptr)) ||
      ((a.epi == GE_BIAS_SILU || a.epi == GE_BIAS_BF16) && a.bias == nullptr) ||
      (a.epi == GE_BIAS_SILU && a.h == nullptr) || (a.epi == GE_BIAS_BF16 && a.y == nullptr) ||
      a.nss > kMaxNss || (a.epi == GE_RESID && (a.ss_out == nullptr || a.y == nullptr)) ||
      (a.xmode == GX_NORM && atoms / a.cs > 4) || (a.xmode == GX_SCALED && a.ss == nullptr) ||
      (a.epi == GE_RESID && a.xg_out && a.xg_gamma == nullptr)) {
    note(cudaErrorInvalidValue, "k_gemm (shape / arguments)");
    return;
  }
  const dim3 grid((a.N / 128) * a.cs, (max_tok + a.nt * 8 - 1) / (a.nt * 8));
  switch (a.nt) {
    case 1: gemm_nt<1>(a, grid, st); break;
    case 2: gemm_nt<2>(a, grid, st); break;
    case 4: gemm_nt<4>(a, grid, st); break;
    default: gemm_nt<8>(a, grid, st); break;
  }
}

template <int NT, int KA>
static void gemm_attr() {
  cudaFuncSetAttribute(k_gemm<NT, KA>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)GemmSmem<NT, KA>::kBytes);
}
template <int NT>
static void gemm_attrs() {
  gemm_attr<NT, 2>();
  gemm_attr<NT, 4>();
  gemm_attr<NT, 6>();
}

static PFN_cuTensorMapEncodeTiled_v12000 g_encode_tiled = nullptr;

bool make_tmap(CUtensorMap *m, CUtensorMapDataType type, int rank, const void *base, const uint64_t *dims,
               const uint64_t *strides, const uint32_t *box, CUtensorMapSwizzle swizzle) {
  if (!g_encode_tiled) {
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", reinterpret_cast<void **>(&g_encode_tiled),
                                cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return false;
  }
  cuuint64_t d[5], st[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; i++) {
    d[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
    if (i + 1 < rank) st[i] = strides[i];
  }
  return g_encode_tiled(m, type, rank, const_cast<void *>(base), d, st, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_tmap_bf16(CUtensorMap *m, const void *base, uint64_t inner, uint64_t rows, uint64_t row_bytes,
                    uint32_t box_inner, uint32_t box_rows) {
  const uint64_t dims[2] = {inner, rows}, strides[1] = {row_bytes};
  const uint32_t box[2] = {box_inner, box_rows};
  return make_tmap(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

struct BlockSync {
  __device__ void operator()() const { __syncthreads(); }
};

__global__ void __launch_bounds__(128, 3) k_attn(AttnArgs a) {
  __shared__ AttnSmem S;
  extern __shared__ __align__(16) uint16_t attn_ring[];
  TraceRec *trb = threadIdx.x == 0 ? g_trace : nullptr;
  unsigned long long tst[7] = {0, 0, 0, 0, 0, 0, 0};
  if (trb) tst[0] = gclock();
  d_attn_number(a, threadIdx.x, S, BlockSync{});  // host-written metadata only
  pdl_wait();
  pdl_launch();
  if (trb) tst[1] = gclock();
  d_attn_run(a, threadIdx.x, blockIdx.x * kAttnWarps, gridDim.x * kAttnWarps, S, attn_ring, BlockSync{});
  if (trb) {
    tst[6] = gclock();
    trace_put(trb, 3, tst, 0, 0);
  }
}

static int g_attn_grid = 0;

// grid of k_attn: enough CTAs for max_tok * n_kv * max_units units, at most
// the resident CTAs of the whole GPU (the warps loop over the units)
static int attn_grid(const AttnArgs &a, int max_tok) {
  if (g_attn_grid == 0) {
    int dev = 0, sms = 0, occ = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k_attn, 128, kAttnDynSmem);
    g_attn_grid = sms * (occ < 1 ? 1 : occ);
  }
  const long long units = (long long)max_tok * a.kv.n_kv * a.max_units;
  const long long need = (units + kAttnWarps - 1) / kAttnWarps;
  return (int)(need < g_attn_grid ? (need < 1 ? 1 : need) : g_attn_grid);
}

static void attention_launch(const AttnArgs &a, int max_tok, cudaStream_t st) {
  if (max_tok > kAttnMaxTok || a.pw < 1 || a.max_units < 1 || a.max_units > kAttnMaxUnits) {
    note(cudaErrorInvalidValue, "k_attn (max_tok / pw / max_units out of range)");
    return;
  }
  launch(k_attn, dim3(attn_grid(a, max_tok)), dim3(128), kAttnDynSmem, st, a);
}

void attention(const uint16_t *q, KVView kv, int layer, TokView tv, int max_tok, int nh, int pw, int max_units,
               AttnWork ws, uint16_t *out, cudaStream_t st) {
  AttnArgs a{};
  a.q = q;
  a.kv = kv;
  a.layer = layer;
  a.tv = tv;
  a.nh = nh;
  a.pw = pw;
  a.max_units = max_units;
  a.scale = 1.0f / sqrtf(128.0f);
  a.ws = ws;
  a.out = out;
  attention_launch(a, max_tok, st);
}

constexpr int kSampleThreads = 512;
constexpr size_t kSampleSmem = (size_t)kSampleMaxV * 12;

// One token per CTA: the sampler, then (has_tail) the next input row of the
// same token built from the code just sampled and normalised, so the two
// steps of a code-predictor position share one launch.
__global__ void __launch_bounds__(kSampleThreads) k_sample(SampleArgs a, RmsArgs tail, int has_tail) {
  extern __shared__ __align__(16) float smem_f[];
  __shared__ float rv[32];
  __shared__ int ri[32];
  __shared__ float red[33];
  TraceRec *trb = threadIdx.x == 0 ? g_trace : nullptr;
  unsigned long long tst[7] = {0, 0, 0, 0, 0, 0, 0};
  if (trb) tst[0] = gclock();
  pdl_wait();
  pdl_launch();
  if (trb) tst[1] = gclock();
  d_sample(a, blockIdx.x, smem_f, smem_f + kSampleMaxV, reinterpret_cast<int *>(smem_f + 2 * kSampleMaxV), rv, ri);
  if (has_tail) d_rmsnorm(tail, blockIdx.x, red);  // d_sample ended with a block barrier: its codes are visible
  if (trb) {
    tst[6] = gclock();
    trace_put(trb, 4, tst, 0, 0);
  }
}

void sample(const SampleArgs &a, int max_tok, cudaStream_t st, const RmsArgs *tail) {
  RmsArgs t{};
  if (tail) t = *tail;
  launch(k_sample, dim3(max_tok), dim3(kSampleThreads), kSampleSmem, st, a, t, tail ? 1 : 0);
}

// out[i] = table[ids[i]] for i < n, rows of `width` bf16 (width % 8 == 0).
__global__ void k_gather_rows(const uint16_t *__restrict__ table, const int *__restrict__ ids, int width,
                              uint16_t *__restrict__ out) {
  const uint4 *src = reinterpret_cast<const uint4 *>(table + (size_t)ids[blockIdx.x] * width);
  uint4 *dst = reinterpret_cast<uint4 *>(out + (size_t)blockIdx.x * width);
  for (int i = threadIdx.x; i < width / 8; i += blockDim.x) dst[i] = src[i];
}

void gather_rows_bf16(const uint16_t *table, const int *ids, int n, int width, uint16_t *out, cudaStream_t st) {
  if (n <= 0) return;
  if (width % 8) {
    note(cudaErrorInvalidValue, "k_gather_rows (width)");
    return;
  }
  k_gather_rows<<<n, 128, 0, st>>>(table, ids, width, out);
  note(cudaGetLastError(), "k_gather_rows");
  g_launches++;
}

// Prompt seed rows (session_seed.rs:151-215): out[s] = bf16(P[text_row[s]] +
// codec_emb[codec_id[s]]), either term absent when its index is negative.
__global__ void k_seed_rows(const float *P, const uint16_t *codec_emb, const int *text_row, const int *codec_id,
                            const float *X, const int *x_row, int H, float *out) {
  const int s = blockIdx.x, tr = text_row[s], ci = codec_id[s], xr = x_row ? x_row[s] : -1;
  for (int h = threadIdx.x; h < H; h += blockDim.x) {
    float v = tr >= 0 ? P[(size_t)tr * H + h] : 0.f;
    if (ci >= 0)
      v += __uint_as_float((uint32_t)codec_emb[(size_t)ci * H + h] << 16);
    else if (xr >= 0)
      v += X[(size_t)xr * H + h];
    out[(size_t)s * H + h] = __bfloat162float(__float2bfloat16_rn(v));
  }
}

void seed_rows(const float *P, const uint16_t *codec_emb, const int *text_row, const int *codec_id, int S, int H,
               float *out, cudaStream_t st, const float *X, const int *x_row) {
  if (S <= 0) return;
  k_seed_rows<<<S, 256, 0, st>>>(P, codec_emb, text_row, codec_id, X, x_row, H, out);
  note(cudaGetLastError(), "k_seed_rows");
  g_launches++;
}

// Row 0: bf16(spk); row 1 + t: frame t of the reference codes [G][T], the
// talker codec embedding of group 0 plus the predictor embedding g - 1 of
// every group g >= 1, each partial sum rounded to bf16 in group order.
__global__ void k_clone_rows(const float *spk, const int64_t *codes, int G, int T, const uint16_t *emb0,
                             const uint16_t *const *embs, int H, float *X) {
  const int r = blockIdx.x;
  for (int h = threadIdx.x; h < H; h += blockDim.x) {
    float v;
    if (r == 0) {
      v = __bfloat162float(__float2bfloat16_rn(spk[h]));
    } else {
      const int t = r - 1;
      v = __uint_as_float((uint32_t)emb0[(size_t)codes[t] * H + h] << 16);
      for (int g = 1; g < G; g++)
        v = __bfloat162float(__float2bfloat16_rn(
            v + __uint_as_float((uint32_t)embs[g - 1][(size_t)codes[(size_t)g * T + t] * H + h] << 16)));
    }
    X[(size_t)r * H + h] = v;
  }
}

void clone_rows(const float *spk, const int64_t *codes, int G, int T, const uint16_t *emb0,
                const uint16_t *const *embs, int H, float *X, cudaStream_t st) {
  k_clone_rows<<<1 + T, 256, 0, st>>>(spk, codes, G, T, emb0, embs, H, X);
  note(cudaGetLastError(), "k_clone_rows");
  g_launches++;
}

__global__ void k_kv_import(const uint16_t *k, const uint16_t *v, int len, KVView kv, int seq) {
  const int l = blockIdx.z, h = blockIdx.y, j = blockIdx.x;
  const size_t src = (((size_t)l * kv.n_kv + h) * len + j) * 128;
  const size_t dst = l * kv.layer_stride + page_elem(kv, seq, j, h);
  for (int d = threadIdx.x; d < 128; d += blockDim.x) {
    kv.k[dst + d] = k[src + d];
    kv.v[dst + d] = v[src + d];
  }
}

void kv_import(const uint16_t *k, const uint16_t *v, int layers, int len, KVView kv, int seq, cudaStream_t st) {
  if (len <= 0) return;
  k_kv_import<<<dim3(len, kv.n_kv, layers), 128, 0, st>>>(k, v, len, kv, seq);
  note(cudaGetLastError(), "k_kv_import");
  g_launches++;
}

void run_phases(const Phase *ph, int n, cudaStream_t st) {
  for (int i = 0; i < n; i++) {
    const Phase &p = ph[i];
    switch (p.type) {
      case PH_NORM: rmsnorm(p.norm, p.max_tok, st); break;
      case PH_GEMM: gemm(p.gemm, p.max_tok, st); break;
      case PH_ATTN: attention_launch(p.attn, p.max_tok, st); break;
      case PH_SAMPLE: sample(p.smp, p.max_tok, st, p.has_tail ? &p.tail : nullptr); break;
      default: note(cudaErrorInvalidValue, "run_phases: unknown phase"); break;
    }
  }
}

void init_kernel_attributes() {
  cudaFuncSetAttribute(k_sample, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSampleSmem);
  cudaFuncSetAttribute(k_attn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kAttnDynSmem);
  gemm_attrs<1>();
  gemm_attrs<2>();
  gemm_attrs<4>();
  gemm_attrs<8>();
  const char *e = getenv("Q3T_PDL");
  if (e && e[0] == '0') g_use_pdl = false;
}

}  // namespace q3t

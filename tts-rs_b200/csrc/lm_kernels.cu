// Talker / code-predictor decode kernels for sm_100a.
//
// One decoder layer of tts_qwen3_tts/src/model/talker/network/layer.rs:23-44
// runs as:  rmsnorm(+zero qkv) -> linear(Wqkv) -> [qkv_post] -> attention ->
// linear(Wo, += residual) -> rmsnorm(+zero gate|up) -> linear(Wgu) ->
// linear(Wdown, silu(gate)*up prologue, += residual).
// Every kernel is PDL-aware: the weight stream of a linear starts before
// griddepcontrol.wait, so it overlaps the tail of the previous kernel.
#include <cfloat>
#include <cstdlib>
#include <utility>

#include "common.cuh"
#include "lm_kernels.cuh"

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

template <typename... KArgs, typename... Args>
static void launch(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                   Args &&...args) {
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
// (16-row block rb, 16-column block kb), tiles ordered rb-major so a CTA's
// K-range of one row block is one contiguous stream.  Lane l of the warp
// finds its 4 A registers at bytes [16 l, 16 l + 16) of the tile.
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
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    d[i] = f2bf(s[i]);
}

void f32_to_bf16(const float *src, uint16_t *dst, int64_t n, cudaStream_t st) {
  k_f32_to_bf16<<<1184, 256, 0, st>>>(src, dst, n);
  note(cudaGetLastError(), "k_f32_to_bf16");
  g_launches++;
}

// ---------------------------------------------------------------------------
// RMSNorm (burn::nn::RmsNorm: x / sqrt(mean(x^2) + eps) * gamma) -> bf16
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_rmsnorm(const float *x, int ldx, int row_mul,
                                                 int row_add, const float *__restrict__ gamma,
                                                 uint16_t *out, int ldo, int H,
                                                 float eps, const int *ntok,
                                                 float *zero, int ldz, int zero_cols,
                                                 float *out_f32,
                                                 const int *slot) {
  __shared__ float red[33];
  pdl_wait();
  const int t = blockIdx.x;
  if (t < *ntok) {
    const float *xr = x + (size_t)(t * row_mul + row_add) * ldx;
    float ss = 0.f;
    for (int i = threadIdx.x * 4; i < H; i += blockDim.x * 4) {
      float4 v = *reinterpret_cast<const float4 *>(xr + i);
      ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    ss = block_sum(ss, red);
    const float rms = sqrtf(ss / (float)H + eps);
    for (int i = threadIdx.x * 4; i < H; i += blockDim.x * 4) {
      float4 v = *reinterpret_cast<const float4 *>(xr + i);
      float4 gm = *reinterpret_cast<const float4 *>(gamma + i);
      float4 y = make_float4(v.x / rms * gm.x, v.y / rms * gm.y, v.z / rms * gm.z, v.w / rms * gm.w);
      uint2 p;
      p.x = pack_bf16x2(y.x, y.y);
      p.y = pack_bf16x2(y.z, y.w);
      *reinterpret_cast<uint2 *>(out + (size_t)t * ldo + i) = p;
      if (out_f32) *reinterpret_cast<float4 *>(out_f32 + (size_t)slot[t] * H + i) = y;
    }
    if (zero)
      for (int i = threadIdx.x * 4; i < zero_cols; i += blockDim.x * 4)
        *reinterpret_cast<float4 *>(zero + (size_t)t * ldz + i) = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  pdl_launch();
}

void rmsnorm(const float *x, int ldx, int row_mul, int row_add, const float *gamma, uint16_t *out,
             int ldo, int H, float eps, const int *ntok, int grid_rows, float *zero, int ldz,
             int zero_cols, float *out_f32, const int *slot, cudaStream_t st) {
  launch(k_rmsnorm, dim3(grid_rows), dim3(256), 0, st, x, ldx, row_mul, row_add, gamma, out, ldo,
         H, eps, ntok, zero, ldz, zero_cols, out_f32, slot);
}

// ---------------------------------------------------------------------------
// Skinny GEMM Y[t][n] += W[n][:] . X[t][:] on the tensor cores (m16n8k16).
// CTA = 4 warps = 4 row blocks (64 output rows) x one K chunk of kc <= 256.
// Each warp first issues all of its weight-fragment loads (16 B per lane,
// fully coalesced, L1 no-allocate), then waits for the previous kernel,
// stages the X chunk of up to 64 tokens in shared memory and runs NT
// n-tiles of 8 tokens per fragment.  Split-K partials go out as f32 atomics.
// ---------------------------------------------------------------------------
template <int NT, int XMODE>
__global__ void __launch_bounds__(128) k_linear(const uint4 *__restrict__ W, int N, int K, int kc,
                                                const void *X, int ldx,
                                                float *Y, int ldy,
                                                const int *ntok_p, int tok_base) {
  constexpr int FR = 16;
  extern __shared__ __align__(16) uint16_t xs[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rb = blockIdx.x * 4 + warp;
  const int k0 = blockIdx.y * kc;
  const int nkb = kc >> 4;
  uint4 a[FR];
  const uint4 *wp = W + ((size_t)rb * (K >> 4) + (k0 >> 4)) * 32 + lane;
#pragma unroll
  for (int i = 0; i < FR; i++)
    if (i < nkb) a[i] = ldg_stream(wp + i * 32);
  pdl_wait();
  int ntok = *ntok_p - tok_base;
  ntok = ntok < 0 ? 0 : (ntok > NT * 8 ? NT * 8 : ntok);
  const int ldsx = kc + 8;
  const int c8n = kc >> 3;
  for (int idx = threadIdx.x; idx < NT * 8 * c8n; idx += 128) {
    const int r = idx / c8n, c8 = (idx - r * c8n) * 8;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (r < ntok) {
      if (XMODE == 0) {
        v = *reinterpret_cast<const uint4 *>(reinterpret_cast<const uint16_t *>(X) +
                                             (size_t)(tok_base + r) * ldx + k0 + c8);
      } else {
        const float *g = reinterpret_cast<const float *>(X) + (size_t)(tok_base + r) * ldx + k0 + c8;
        const float *u = g + K;
        float4 g0 = *reinterpret_cast<const float4 *>(g), g1 = *reinterpret_cast<const float4 *>(g + 4);
        float4 u0 = *reinterpret_cast<const float4 *>(u), u1 = *reinterpret_cast<const float4 *>(u + 4);
        v.x = pack_bf16x2(silu(g0.x) * u0.x, silu(g0.y) * u0.y);
        v.y = pack_bf16x2(silu(g0.z) * u0.z, silu(g0.w) * u0.w);
        v.z = pack_bf16x2(silu(g1.x) * u1.x, silu(g1.y) * u1.y);
        v.w = pack_bf16x2(silu(g1.z) * u1.z, silu(g1.w) * u1.w);
      }
    }
    *reinterpret_cast<uint4 *>(xs + r * ldsx + c8) = v;
  }
  __syncthreads();
  pdl_launch();
  float acc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; j++) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int i = 0; i < FR; i++) {
    if (i < nkb) {
#pragma unroll
      for (int j = 0; j < NT; j++) {
        const uint16_t *xr = xs + (j * 8 + g) * ldsx + i * 16 + 2 * t;
        const uint32_t b0 = *reinterpret_cast<const uint32_t *>(xr);
        const uint32_t b1 = *reinterpret_cast<const uint32_t *>(xr + 8);
        mma_16816(acc[j], a[i].x, a[i].y, a[i].z, a[i].w, b0, b1);
      }
    }
  }
  const int row = rb * 16 + g;
#pragma unroll
  for (int j = 0; j < NT; j++) {
    const int tk = j * 8 + 2 * t;
    if (tk < ntok) {
      float *y = Y + (size_t)(tok_base + tk) * ldy + row;
      atomicAdd(y, acc[j][0]);
      atomicAdd(y + 8, acc[j][2]);
    }
    if (tk + 1 < ntok) {
      float *y = Y + (size_t)(tok_base + tk + 1) * ldy + row;
      atomicAdd(y, acc[j][1]);
      atomicAdd(y + 8, acc[j][3]);
    }
  }
}

template <int NT>
static void linear_nt(const uint16_t *Wp, int N, int K, int kc, const void *X, int ldx, int xmode,
                      float *Y, int ldy, const int *ntok, int tok_base, cudaStream_t st) {
  dim3 grid(N / 64, K / kc);
  size_t smem = (size_t)NT * 8 * (kc + 8) * 2;
  const uint4 *W = reinterpret_cast<const uint4 *>(Wp);
  if (xmode == 0)
    launch(k_linear<NT, 0>, grid, dim3(128), smem, st, W, N, K, kc, X, ldx, Y, ldy, ntok, tok_base);
  else
    launch(k_linear<NT, 1>, grid, dim3(128), smem, st, W, N, K, kc, X, ldx, Y, ldy, ntok, tok_base);
}

void linear(const uint16_t *Wp, int N, int K, const void *X, int ldx, int xmode, float *Y, int ldy,
            const int *ntok, int max_tok, cudaStream_t st) {
  const int kc = (K % 256 == 0) ? 256 : (K % 128 == 0 ? 128 : 64);
  for (int base = 0; base < max_tok; base += 64) {
    const int n = max_tok - base < 64 ? max_tok - base : 64;
    if (n <= 8)
      linear_nt<1>(Wp, N, K, kc, X, ldx, xmode, Y, ldy, ntok, base, st);
    else if (n <= 16)
      linear_nt<2>(Wp, N, K, kc, X, ldx, xmode, Y, ldy, ntok, base, st);
    else if (n <= 32)
      linear_nt<4>(Wp, N, K, kc, X, ldx, xmode, Y, ldy, ntok, base, st);
    else
      linear_nt<8>(Wp, N, K, kc, X, ldx, xmode, Y, ldy, ntok, base, st);
  }
}

// ---------------------------------------------------------------------------
// q_norm / k_norm + RoPE (attention.rs:49-69): one warp per head, lane l
// holds dims [4l, 4l+4); the rotate-half partner of dim d is d +- 64, i.e.
// lane l ^ 16.
// ---------------------------------------------------------------------------
Q3T_DEV void norm_rope_lane(float4 v, const float *gm, float eps, int lane, int pos,
                            const float *__restrict__ inv_freq, float out[4]) {
  const float ss = warp_sum(v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w);
  const float rms = sqrtf(ss / 128.f + eps);
  float e[4] = {v.x / rms * gm[lane * 4 + 0], v.y / rms * gm[lane * 4 + 1],
                v.z / rms * gm[lane * 4 + 2], v.w / rms * gm[lane * 4 + 3]};
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const float p = __shfl_xor_sync(0xffffffffu, e[i], 16);
    const int d = lane * 4 + i;
    float s, c;
    sincosf((float)pos * inv_freq[d & 63], &s, &c);
    out[i] = d < 64 ? e[i] * c - p * s : e[i] * c + p * s;
  }
}

Q3T_DEV size_t page_elem(const KVView &kv, int seq, int pos, int h) {
  const int page = kv.page_table[(size_t)seq * kv.pt_stride + (pos >> 4)];
  return (((size_t)page * kv.n_kv + h) * 16 + (pos & 15)) * 128;
}

__global__ void __launch_bounds__(1024) k_qkv_post(const float *qkv, int ldqkv,
                                                   const float *__restrict__ q_norm,
                                                   const float *__restrict__ k_norm,
                                                   const float *__restrict__ inv_freq, float eps,
                                                   int nh, int nkv, TokView tv,
                                                   uint16_t *qout, KVView kv,
                                                   int layer) {
  pdl_wait();
  const int t = blockIdx.x;
  if (t < *tv.ntok) {
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pos = tv.pos[t] + tv.pos_add, seq = tv.seq[t];
    const float *row = qkv + (size_t)t * ldqkv;
    if (w < nh + nkv) {
      const bool isq = w < nh;
      const int h = isq ? w : w - nh;
      const float4 v = *reinterpret_cast<const float4 *>(row + (isq ? h : nh + h) * 128 + lane * 4);
      float o[4];
      norm_rope_lane(v, isq ? q_norm : k_norm, eps, lane, pos, inv_freq, o);
      uint2 p;
      p.x = pack_bf16x2(o[0], o[1]);
      p.y = pack_bf16x2(o[2], o[3]);
      if (isq)
        *reinterpret_cast<uint2 *>(qout + (size_t)t * nh * 128 + h * 128 + lane * 4) = p;
      else
        *reinterpret_cast<uint2 *>(kv.k + layer * kv.layer_stride + page_elem(kv, seq, pos, h) + lane * 4) = p;
    } else if (w < nh + 2 * nkv) {
      const int h = w - nh - nkv;
      const float4 v = *reinterpret_cast<const float4 *>(row + (nh + nkv + h) * 128 + lane * 4);
      uint2 p;
      p.x = pack_bf16x2(v.x, v.y);
      p.y = pack_bf16x2(v.z, v.w);
      *reinterpret_cast<uint2 *>(kv.v + layer * kv.layer_stride + page_elem(kv, seq, pos, h) + lane * 4) = p;
    }
  }
  pdl_launch();
}

void qkv_post(const float *qkv, int ldqkv, const float *q_norm, const float *k_norm,
              const float *inv_freq, float eps, int nh, int nkv, TokView tv, int max_tok,
              uint16_t *qout, KVView kv, int layer, cudaStream_t st) {
  launch(k_qkv_post, dim3(max_tok), dim3(32 * (nh + 2 * nkv)), 0, st, qkv, ldqkv, q_norm, k_norm,
         inv_freq, eps, nh, nkv, tv, qout, kv, layer);
}

// ---------------------------------------------------------------------------
// Split-K flash-decoding GQA attention (attention.rs:88-123 with the f32
// softmax of nn/attention.rs:13-26).  CTA = (split, kv head g, token t):
// both query heads 2g, 2g+1 of the group share every K/V row read.  Splits
// of `chunk` keys write (o, m, l) partials; the last CTA of (t, g) to finish
// merges them (counter reset by the merger).
// ---------------------------------------------------------------------------
constexpr int kPart = 132;

template <bool FUSED>
__global__ void __launch_bounds__(128) k_attn(const float *qkv, int ldqkv,
                                              const float *__restrict__ q_norm,
                                              const float *__restrict__ k_norm,
                                              const float *__restrict__ inv_freq, float eps,
                                              const uint16_t *qin, KVView kv,
                                              int layer, TokView tv, int nh, int chunk,
                                              float scale, AttnWork ws, uint16_t *out) {
  __shared__ float qs[2][128];
  __shared__ float sc[2][256];
  __shared__ float red[2][4];
  __shared__ float opart[2][2][128];
  __shared__ int s_last;
  const int sp = blockIdx.x, g = blockIdx.y, t = blockIdx.z;
  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
  pdl_wait();
  if (t >= *tv.ntok) return;
  const int pos = tv.pos[t] + tv.pos_add, L = pos + 1, seq = tv.seq[t];
  const int nsplit = (L + chunk - 1) / chunk;
  if (sp >= nsplit) return;
  const int j0 = sp * chunk;
  const int n = min(L - j0, chunk);
  uint16_t *kb = kv.k + layer * kv.layer_stride;
  uint16_t *vb = kv.v + layer * kv.layer_stride;
  if (FUSED) {
    const float *row = qkv + (size_t)t * ldqkv;
    if (w < 2) {
      const int h = 2 * g + w;
      const float4 v = *reinterpret_cast<const float4 *>(row + h * 128 + lane * 4);
      float o[4];
      norm_rope_lane(v, q_norm, eps, lane, pos, inv_freq, o);
#pragma unroll
      for (int i = 0; i < 4; i++) qs[w][lane * 4 + i] = bf16_round(o[i]);
    } else if (sp == nsplit - 1) {
      const size_t e = page_elem(kv, seq, pos, g) + lane * 4;
      if (w == 2) {
        const float4 v = *reinterpret_cast<const float4 *>(row + (nh + g) * 128 + lane * 4);
        float o[4];
        norm_rope_lane(v, k_norm, eps, lane, pos, inv_freq, o);
        uint2 p;
        p.x = pack_bf16x2(o[0], o[1]);
        p.y = pack_bf16x2(o[2], o[3]);
        *reinterpret_cast<uint2 *>(kb + e) = p;
      } else {
        const float4 v =
            *reinterpret_cast<const float4 *>(row + (nh + kv.n_kv + g) * 128 + lane * 4);
        uint2 p;
        p.x = pack_bf16x2(v.x, v.y);
        p.y = pack_bf16x2(v.z, v.w);
        *reinterpret_cast<uint2 *>(vb + e) = p;
      }
    }
  } else {
    for (int e = tid; e < 256; e += 128)
      qs[e >> 7][e & 127] = bf2f(qin[(size_t)t * nh * 128 + (2 * g + (e >> 7)) * 128 + (e & 127)]);
  }
  __syncthreads();
  // scores: one key row (256 B) per thread
  for (int jj = tid; jj < n; jj += 128) {
    const int j = j0 + jj;
    const uint4 *kr = reinterpret_cast<const uint4 *>(kb + page_elem(kv, seq, j, g));
    float s0 = 0.f, s1 = 0.f;
#pragma unroll 4
    for (int c = 0; c < 16; c++) {
      const uint4 u = kr[c];
      const uint32_t wv[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const float k0v = bf2f(wv[e] & 0xffffu), k1v = bf2f(wv[e] >> 16);
        s0 += qs[0][c * 8 + 2 * e] * k0v + qs[0][c * 8 + 2 * e + 1] * k1v;
        s1 += qs[1][c * 8 + 2 * e] * k0v + qs[1][c * 8 + 2 * e + 1] * k1v;
      }
    }
    sc[0][jj] = s0 * scale;
    sc[1][jj] = s1 * scale;
  }
  __syncthreads();
  float m0 = -FLT_MAX, m1 = -FLT_MAX;
  for (int jj = tid; jj < n; jj += 128) {
    m0 = fmaxf(m0, sc[0][jj]);
    m1 = fmaxf(m1, sc[1][jj]);
  }
  m0 = warp_max(m0);
  m1 = warp_max(m1);
  if (lane == 0) {
    red[0][w] = m0;
    red[1][w] = m1;
  }
  __syncthreads();
  m0 = fmaxf(fmaxf(red[0][0], red[0][1]), fmaxf(red[0][2], red[0][3]));
  m1 = fmaxf(fmaxf(red[1][0], red[1][1]), fmaxf(red[1][2], red[1][3]));
  __syncthreads();
  float l0 = 0.f, l1 = 0.f;
  for (int jj = tid; jj < n; jj += 128) {
    const float p0 = expf(sc[0][jj] - m0), p1 = expf(sc[1][jj] - m1);
    sc[0][jj] = p0;
    sc[1][jj] = p1;
    l0 += p0;
    l1 += p1;
  }
  l0 = warp_sum(l0);
  l1 = warp_sum(l1);
  if (lane == 0) {
    red[0][w] = l0;
    red[1][w] = l1;
  }
  __syncthreads();
  l0 = red[0][0] + red[0][1] + red[0][2] + red[0][3];
  l1 = red[1][0] + red[1][1] + red[1][2] + red[1][3];
  // P.V: thread = (key parity kh, dim pair dp)
  {
    const int dp = tid & 63, kh = tid >> 6, d = dp * 2;
    float o00 = 0.f, o01 = 0.f, o10 = 0.f, o11 = 0.f;
    for (int jj = kh; jj < n; jj += 2) {
      const uint32_t vv = *reinterpret_cast<const uint32_t *>(vb + page_elem(kv, seq, j0 + jj, g) + d);
      const float v0 = bf2f(vv & 0xffffu), v1 = bf2f(vv >> 16);
      const float p0 = sc[0][jj], p1 = sc[1][jj];
      o00 += p0 * v0;
      o01 += p0 * v1;
      o10 += p1 * v0;
      o11 += p1 * v1;
    }
    opart[kh][0][d] = o00;
    opart[kh][0][d + 1] = o01;
    opart[kh][1][d] = o10;
    opart[kh][1][d + 1] = o11;
  }
  __syncthreads();
  const int out_ld = nh * 128;
  if (nsplit == 1) {
    for (int e = tid; e < 256; e += 128) {
      const int h = e >> 7, d = e & 127;
      const float o = opart[0][h][d] + opart[1][h][d];
      out[(size_t)t * out_ld + (2 * g + h) * 128 + d] = f2bf(o / (h ? l1 : l0));
    }
  } else {
    float *P = ws.part + (((size_t)t * kv.n_kv + g) * ws.max_split + sp) * 2 * kPart;
    for (int e = tid; e < 256; e += 128) {
      const int h = e >> 7, d = e & 127;
      P[h * kPart + d] = opart[0][h][d] + opart[1][h][d];
    }
    if (tid == 0) {
      P[128] = m0;
      P[129] = l0;
      P[kPart + 128] = m1;
      P[kPart + 129] = l1;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
      const int prev = atomicAdd(&ws.counters[t * kv.n_kv + g], 1);
      s_last = prev == nsplit - 1;
    }
    __syncthreads();
    if (s_last) {
      __threadfence();
      const float *P0 = ws.part + ((size_t)t * kv.n_kv + g) * ws.max_split * 2 * kPart;
      for (int e = tid; e < 256; e += 128) {
        const int h = e >> 7, d = e & 127;
        float M = -FLT_MAX;
        for (int s = 0; s < nsplit; s++) M = fmaxf(M, __ldcg(P0 + (size_t)s * 2 * kPart + h * kPart + 128));
        float Ls = 0.f, acc = 0.f;
        for (int s = 0; s < nsplit; s++) {
          const float *Ps = P0 + (size_t)s * 2 * kPart + h * kPart;
          const float f = expf(__ldcg(Ps + 128) - M);
          Ls += __ldcg(Ps + 129) * f;
          acc += __ldcg(Ps + d) * f;
        }
        out[(size_t)t * out_ld + (2 * g + h) * 128 + d] = f2bf(acc / Ls);
      }
      if (tid == 0) ws.counters[t * kv.n_kv + g] = 0;
    }
  }
  pdl_launch();
}

void attention(int fused, const float *qkv, int ldqkv, const float *q_norm, const float *k_norm,
               const float *inv_freq, float eps, const uint16_t *qin, KVView kv, int layer,
               TokView tv, int max_tok, int nh, int chunk, int max_split, AttnWork ws,
               uint16_t *out, cudaStream_t st) {
  dim3 grid(max_split, kv.n_kv, max_tok);
  const float scale = 1.0f / sqrtf(128.0f);
  if (fused)
    launch(k_attn<true>, grid, dim3(128), 0, st, qkv, ldqkv, q_norm, k_norm, inv_freq, eps, qin, kv,
           layer, tv, nh, chunk, scale, ws, out);
  else
    launch(k_attn<false>, grid, dim3(128), 0, st, qkv, ldqkv, q_norm, k_norm, inv_freq, eps, qin,
           kv, layer, tv, nh, chunk, scale, ws, out);
}

// ---------------------------------------------------------------------------
// Codec-group context embedding (infer/mod.rs:343-383)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_embed(const uint16_t *__restrict__ emb0,
                                               const uint16_t *const *__restrict__ embs, int G,
                                               int H, const int64_t *codes,
                                               const int *slot,
                                               const float *const *extra,
                                               const int *frame,
                                               int64_t *hist, int hist_frames,
                                               const int *ntok, float *x) {
  pdl_wait();
  const int t = blockIdx.x;
  if (t < *ntok) {
    const int s = slot[t];
    const int64_t *c = codes + (size_t)s * G;
    const float *ex = extra ? extra[t] : nullptr;
    for (int i = threadIdx.x * 4; i < H; i += blockDim.x * 4) {
      const uint2 e0 = *reinterpret_cast<const uint2 *>(emb0 + (size_t)c[0] * H + i);
      float a0 = bf2f(e0.x & 0xffffu), a1 = bf2f(e0.x >> 16), a2 = bf2f(e0.y & 0xffffu),
            a3 = bf2f(e0.y >> 16);
      for (int q = 1; q < G; q++) {
        const uint2 e = *reinterpret_cast<const uint2 *>(embs[q - 1] + (size_t)c[q] * H + i);
        a0 += bf2f(e.x & 0xffffu);
        a1 += bf2f(e.x >> 16);
        a2 += bf2f(e.y & 0xffffu);
        a3 += bf2f(e.y >> 16);
      }
      if (ex) {
        const float4 v = *reinterpret_cast<const float4 *>(ex + i);
        a0 += v.x;
        a1 += v.y;
        a2 += v.z;
        a3 += v.w;
      }
      *reinterpret_cast<float4 *>(x + (size_t)t * H + i) = make_float4(a0, a1, a2, a3);
    }
    if (hist && threadIdx.x < G) hist[((size_t)s * hist_frames + frame[t]) * G + threadIdx.x] = c[threadIdx.x];
  }
  pdl_launch();
}

void embed_codes(const uint16_t *emb0, const uint16_t *const *embs, int G, int H,
                 const int64_t *codes, const int *slot, const float *const *extra,
                 const int *frame, int64_t *hist, int hist_frames, const int *ntok, int max_tok,
                 float *x, cudaStream_t st) {
  launch(k_embed, dim3(max_tok), dim3(256), 0, st, emb0, embs, G, H, codes, slot, extra, frame,
         hist, hist_frames, ntok, x);
}

__global__ void __launch_bounds__(256) k_pred_input0(const float *hidden,
                                                     const uint16_t *__restrict__ emb0,
                                                     const int64_t *codes, int G,
                                                     const int *slot,
                                                     const int *ntok, int H,
                                                     float *x) {
  pdl_wait();
  const int b = blockIdx.x;
  if (b < *ntok) {
    const int s = slot[b];
    const int64_t c0 = codes[(size_t)s * G];
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
      x[(size_t)(2 * b) * H + i] = hidden[(size_t)s * H + i];
      x[(size_t)(2 * b + 1) * H + i] = bf2f(emb0[(size_t)c0 * H + i]);
    }
  }
  pdl_launch();
}

void pred_input0(const float *hidden, const uint16_t *emb0, const int64_t *codes, int G,
                 const int *slot, const int *ntok, int max_tok, int H, float *x, cudaStream_t st) {
  launch(k_pred_input0, dim3(max_tok), dim3(256), 0, st, hidden, emb0, codes, G, slot, ntok, H, x);
}

__global__ void __launch_bounds__(256) k_pred_input(const uint16_t *__restrict__ emb,
                                                    const int64_t *codes, int G,
                                                    int col, const int *slot,
                                                    const int *ntok, int H,
                                                    float *x) {
  pdl_wait();
  const int b = blockIdx.x;
  if (b < *ntok) {
    const int64_t c = codes[(size_t)slot[b] * G + col];
    for (int i = threadIdx.x; i < H; i += blockDim.x)
      x[(size_t)b * H + i] = bf2f(emb[(size_t)c * H + i]);
  }
  pdl_launch();
}

void pred_input(const uint16_t *emb, const int64_t *codes, int G, int col, const int *slot,
                const int *ntok, int max_tok, int H, float *x, cudaStream_t st) {
  launch(k_pred_input, dim3(max_tok), dim3(256), 0, st, emb, codes, G, col, slot, ntok, H, x);
}

// ---------------------------------------------------------------------------
// Sampling (sampling.rs:33-150) — one CTA per token row, V <= 4096.
// ---------------------------------------------------------------------------
Q3T_DEV uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

constexpr int kSampleThreads = 512;
constexpr int kSampleMaxV = 4096;

// bitonic sort of (value desc, index asc) pairs in shared memory
Q3T_DEV void bitonic_desc(float *v, int *ix, int n) {
  for (int k = 2; k <= n; k <<= 1)
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int l = i ^ j;
        if (l > i) {
          const bool up = (i & k) == 0;  // up: descending segment
          const float a = v[i], b = v[l];
          const int ia = ix[i], ib = ix[l];
          const bool a_first = a > b || (a == b && ia < ib);
          if (up ? !a_first : a_first) {
            v[i] = b;
            v[l] = a;
            ix[i] = ib;
            ix[l] = ia;
          }
        }
      }
      __syncthreads();
    }
}

constexpr size_t kSampleSmem = (size_t)kSampleMaxV * 12;

__global__ void __launch_bounds__(kSampleThreads) k_sample(SampleArgs a) {
  extern __shared__ __align__(16) float smem_f[];
  float *lg = smem_f;
  float *sv = smem_f + kSampleMaxV;
  int *si = reinterpret_cast<int *>(smem_f + 2 * kSampleMaxV);
  __shared__ float rv[32];
  __shared__ int ri[32];
  pdl_wait();
  const int t = blockIdx.x;
  if (t >= *a.ntok) return;
  const int s = a.slot[t];
  const SampleParams P = a.params[s * 2 + a.use_pred_params];
  const int V = a.V, tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  float *row = a.logits + (size_t)t * a.ldl;
  for (int i = tid; i < V; i += blockDim.x) lg[i] = row[i];
  __syncthreads();
  // repetition penalty: gather the ORIGINAL logits, scatter-add (duplicates accumulate)
  if (P.rep_penalty > 0.f && a.hist_mode != 0) {
    const float scale = 1.0f / P.rep_penalty - 1.0f;
    if (a.hist_mode == 1) {
      const int n = a.hist_len[s];
      const int32_t *hs = a.hist + (size_t)s * a.hist_cap;
      for (int i = tid; i < n; i += blockDim.x) atomicAdd(&lg[hs[i]], row[hs[i]] * scale);
    } else {
      for (int i = 1 + tid; i < a.col; i += blockDim.x) {
        const int id = (int)a.codes[(size_t)s * a.G + i];
        atomicAdd(&lg[id], row[id] * scale);
      }
    }
    __syncthreads();
    for (int i = tid; i < V; i += blockDim.x) row[i] = lg[i];
    __syncthreads();
  }
  if (a.suppress && a.sup_on && a.sup_on[s]) {
    for (int i = tid; i < a.n_suppress; i += blockDim.x) {
      const int64_t id = a.suppress[i];
      if (id >= 0 && id < V) lg[id] = -INFINITY;
    }
    __syncthreads();
  }
  int tok = 0;
  if (!P.do_sample) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = tid; i < V; i += blockDim.x)
      if (lg[i] > bv || (lg[i] == bv && i < bi)) {
        bv = lg[i];
        bi = i;
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (lane == 0) {
      rv[w] = bv;
      ri[w] = bi;
    }
    __syncthreads();
    if (tid == 0) {
      for (int k = 1; k < (int)(blockDim.x >> 5); k++)
        if (rv[k] > bv || (rv[k] == bv && ri[k] < bi)) {
          bv = rv[k];
          bi = ri[k];
        }
      // all -inf (fully suppressed row): Burn's argmax returns index 0
      tok = bi == 0x7fffffff ? 0 : bi;
    }
  } else {
    // temperature -> top-k threshold -> top-p -> softmax -> categorical
    const float temp = P.temperature > 1e-5f ? P.temperature : 1e-5f;
    int n = 1;
    while (n < V) n <<= 1;
    for (int i = tid; i < n; i += blockDim.x) {
      if (i < V) lg[i] = lg[i] / temp;
      sv[i] = i < V ? lg[i] : -INFINITY;
      si[i] = i;
    }
    __syncthreads();
    bitonic_desc(sv, si, n);
    if (P.top_k > 0 && P.top_k < V) {
      const float kth = sv[P.top_k - 1];
      for (int i = tid; i < V; i += blockDim.x)
        if (lg[i] < kth) lg[i] = -INFINITY;
      for (int i = tid; i < n; i += blockDim.x)
        if (sv[i] < kth) sv[i] = -INFINITY;
      __syncthreads();
    }
    if (isfinite(P.top_p) && P.top_p > 0.f && P.top_p < 1.f) {
      if (tid == 0) {
        const float mx = sv[0];
        float sum = 0.f;
        for (int i = 0; i < V; i++) sum += expf(sv[i] - mx);
        float cum = 0.f;
        for (int i = 0; i < V; i++) {
          const float p = expf(sv[i] - mx) / sum;
          cum += p;
          if (!((cum - p) < P.top_p)) lg[si[i]] = -INFINITY;
        }
      }
      __syncthreads();
    }
    if (tid == 0) {
      float mx = -INFINITY;
      for (int i = 0; i < V; i++) mx = fmaxf(mx, lg[i]);
      double sum = 0.0;
      for (int i = 0; i < V; i++) sum += expf(lg[i] - mx);
      const uint64_t r = mix64(P.seed ^ mix64((uint64_t)a.step_seed * 131ull + (uint64_t)a.col) ^
                               ((uint64_t)s << 40));
      const double u = (double)(r >> 11) * (1.0 / 9007199254740992.0);
      const double target = u * sum;
      double cum = 0.0;
      tok = V - 1;
      for (int i = 0; i < V; i++) {
        const double p = expf(lg[i] - mx);
        if (p <= 0.0) continue;
        cum += p;
        if (cum > target) {
          tok = i;
          break;
        }
      }
    }
  }
  if (tid == 0) {
    if (a.raw) {  // the sampled token before any teacher forcing (parity checks)
      const int f = a.frame[t] + a.fadd;
      if (f < a.max_frames) a.raw[((size_t)s * a.max_frames + f) * a.G + a.col] = tok;
    }
    if (a.forced && a.force_on) {  // force_on[slot] = number of teacher-forced frames
      const int f = a.frame[t] + a.fadd;
      if (f < a.force_on[s] && f < a.max_frames)
        tok = (int)a.forced[((size_t)s * a.max_frames + f) * a.G + a.col];
    }
    a.codes[(size_t)s * a.G + a.col] = tok;
    if (a.hist_mode == 1) {
      const int n = a.hist_len[s];
      if (n < a.hist_cap) {
        a.hist[(size_t)s * a.hist_cap + n] = tok;
        a.hist_len[s] = n + 1;
      }
    }
    if (a.eos_flag) a.eos_flag[t] = (a.eos[s] >= 0 && (int64_t)tok == a.eos[s]) ? 1 : 0;
    if (a.sup_on) a.sup_on[s] = 0;
  }
  pdl_launch();
}

void sample(const SampleArgs &a, int max_tok, cudaStream_t st) {
  launch(k_sample, dim3(max_tok), dim3(kSampleThreads), kSampleSmem, st, a);
}

void init_kernel_attributes() {
  cudaFuncSetAttribute(k_sample, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSampleSmem);
  const char *e = getenv("Q3T_PDL");
  if (e && e[0] == '0') g_use_pdl = false;
}

// ---------------------------------------------------------------------------
__global__ void k_kv_import(const uint16_t *k, const uint16_t *v,
                            int len, KVView kv, int seq) {
  const int l = blockIdx.z, h = blockIdx.y, j = blockIdx.x;
  const size_t src = (((size_t)l * kv.n_kv + h) * len + j) * 128;
  const size_t dst = l * kv.layer_stride + page_elem(kv, seq, j, h);
  for (int d = threadIdx.x; d < 128; d += blockDim.x) {
    kv.k[dst + d] = k[src + d];
    kv.v[dst + d] = v[src + d];
  }
}

void kv_import(const uint16_t *k, const uint16_t *v, int layers, int len, KVView kv, int seq,
               cudaStream_t st) {
  if (len <= 0) return;
  k_kv_import<<<dim3(len, kv.n_kv, layers), 128, 0, st>>>(k, v, len, kv, seq);
  note(cudaGetLastError(), "k_kv_import");
  g_launches++;
}

}  // namespace q3t

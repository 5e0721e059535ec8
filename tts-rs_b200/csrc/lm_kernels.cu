// Talker / code-predictor kernels for sm_100a.
//
// One decoder layer of tts_qwen3_tts/src/model/talker/network/layer.rs:23-44
// runs as:  rmsnorm -> linear(Wqkv) -> [qkv_post] -> attention -> linear(Wo)
// -> rmsnorm (folds the o_proj partials into the residual) -> linear(Wgu) ->
// silu_mul -> linear(Wdown) (folded by the next rmsnorm).  Linears write
// split-K partial sums with plain stores; the consumer reduces them in a
// fixed order, so results are deterministic.
//
// Two execution forms share the device code of lm_device.cuh:
//   - standalone kernels (prefill, the isolated decode step), PDL-aware: the
//     weight stream of a linear starts before griddepcontrol.wait;
//   - the persistent frame kernel: one cooperative launch per decode frame
//     runs every phase (15 code-predictor passes + the talker + sampling),
//     separated by grid barriers; each GEMM phase issues its weight loads
//     before the barrier that precedes it.
#include <cstdlib>
#include <utility>

#include "lm_device.cuh"

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
  pdl_wait();
  d_rmsnorm(a, blockIdx.x, red);
  pdl_launch();
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

template <int NT, int FR>
__global__ void __launch_bounds__(kLinWarps * 32, 2) k_linear(LinArgs a) {
  extern __shared__ __align__(16) uint16_t xs[];
  uint4 frag[FR];
  const int item = blockIdx.x;
  d_linear_load<FR>(a, item, frag);
  pdl_wait();
  d_linear_compute<NT, FR>(a, item, frag, xs);
  pdl_launch();
}

static size_t lin_smem(int nt, int fr) { return (size_t)nt * 8 * (16 * fr + 8) * 2; }

__host__ __device__ int linear_items(const LinArgs &a) {
  return (a.N / (16 * kLinWarps)) * (a.K / (16 * a.fr)) * a.ntc;
}

LinArgs linear_plan(const uint16_t *Wp, int N, int K, const void *X, int ldx, float *ws, long long ws_elems,
                    int rows_cap, const int *ntok, int max_tok, int target_items, Part *out) {
  LinArgs a{};
  a.W = reinterpret_cast<const uint4 *>(Wp);
  a.N = N;
  a.K = K;
  a.X = reinterpret_cast<const uint16_t *>(X);
  a.ldx = ldx;
  a.ntok = ntok;
  const int per = max_tok < 64 ? max_tok : 64;
  a.nt = per <= 8 ? 1 : (per <= 16 ? 2 : (per <= 32 ? 4 : 8));
  a.ntc = (max_tok + 63) / 64;
  // the largest K chunk whose item count still reaches the target
  const int rows = N / (16 * kLinWarps);
  int fr = 16;
  while (fr > 4 && (K % (16 * fr) != 0 || (long)rows * (K / (16 * fr)) < target_items)) fr >>= 1;
  a.fr = fr;
  a.P = ws;
  a.pstride = (long long)rows_cap * N;
  a.ldy = N;
  Part P{ws, K / (16 * fr), a.pstride, N};
  if (N % (16 * kLinWarps) || K % 64 || (long long)P.splits * P.stride > ws_elems || max_tok > rows_cap)
    note(cudaErrorInvalidValue, "linear: shape or workspace");
  if (out) *out = P;
  return a;
}

template <int NT>
static void linear_nt(const LinArgs &a, cudaStream_t st) {
  const dim3 grid(linear_items(a));
  const size_t sm = lin_smem(NT, a.fr);
  if (a.fr == 16)
    launch(k_linear<NT, 16>, grid, dim3(kLinWarps * 32), sm, st, a);
  else if (a.fr == 8)
    launch(k_linear<NT, 8>, grid, dim3(kLinWarps * 32), sm, st, a);
  else
    launch(k_linear<NT, 4>, grid, dim3(kLinWarps * 32), sm, st, a);
}

Part linear(const uint16_t *Wp, int N, int K, const void *X, int ldx, float *ws, long long ws_elems, int rows_cap,
            const int *ntok, int max_tok, cudaStream_t st) {
  Part P;
  const LinArgs a = linear_plan(Wp, N, K, X, ldx, ws, ws_elems, rows_cap, ntok, max_tok, 148, &P);
  switch (a.nt) {
    case 1: linear_nt<1>(a, st); break;
    case 2: linear_nt<2>(a, st); break;
    case 4: linear_nt<4>(a, st); break;
    default: linear_nt<8>(a, st); break;
  }
  return P;
}

__global__ void __launch_bounds__(256) k_reduce_rows(Part P, int N, const int *ntok, float *out) {
  pdl_wait();
  const int t = blockIdx.y;
  if (t < *ntok)
    for (int n = (blockIdx.x * blockDim.x + threadIdx.x) * 4; n < N; n += gridDim.x * blockDim.x * 4)
      *reinterpret_cast<float4 *>(out + (size_t)t * N + n) = part4(P, t, n);
  pdl_launch();
}

void reduce_rows(Part P, int N, const int *ntok, int max_tok, float *out, cudaStream_t st) {
  launch(k_reduce_rows, dim3((N / 4 + 255) / 256, max_tok), dim3(256), 0, st, P, N, ntok, out);
}

__global__ void __launch_bounds__(256) k_silu_mul(SiluArgs a) {
  pdl_wait();
  d_silu(a, blockIdx.y, (blockIdx.x * blockDim.x + threadIdx.x) * 4);
  pdl_launch();
}

void silu_mul(Part gu, int I, const int *ntok, int max_tok, uint16_t *out, cudaStream_t st) {
  SiluArgs a{gu, I, ntok, out};
  launch(k_silu_mul, dim3((I / 4 + 255) / 256, max_tok), dim3(256), 0, st, a);
}

__global__ void __launch_bounds__(1024) k_qkv_post(QkvArgs a) {
  pdl_wait();
  d_qkv_post(a, blockIdx.x);
  pdl_launch();
}

void qkv_post(Part qkv, const float *q_norm, const float *k_norm, const float *inv_freq, float eps, int nh, int nkv,
              TokView tv, int max_tok, uint16_t *qout, KVView kv, int layer, cudaStream_t st) {
  QkvArgs a{qkv, q_norm, k_norm, inv_freq, eps, nh, nkv, tv, qout, kv, layer};
  launch(k_qkv_post, dim3(max_tok), dim3(32 * (nh + 2 * nkv)), 0, st, a);
}

struct BlockSync {
  __device__ void operator()() const { __syncthreads(); }
};

__global__ void __launch_bounds__(128) k_attn(AttnArgs a) {
  __shared__ AttnSmem S;
  pdl_wait();
  d_attn(a, blockIdx.x, blockIdx.y, blockIdx.z, threadIdx.x, S, BlockSync{});
  pdl_launch();
}

static AttnArgs attn_args(int fused, Part qkv, const float *q_norm, const float *k_norm, const float *inv_freq,
                          float eps, const uint16_t *qin, KVView kv, int layer, TokView tv, int nh, int chunk,
                          int max_split, AttnWork ws, uint16_t *out) {
  AttnArgs a{};
  a.qkv = qkv;
  a.q_norm = q_norm;
  a.k_norm = k_norm;
  a.inv_freq = inv_freq;
  a.eps = eps;
  a.qin = qin;
  a.kv = kv;
  a.layer = layer;
  a.tv = tv;
  a.nh = nh;
  a.chunk = chunk;
  a.max_split = max_split;
  a.fused = fused;
  a.scale = 1.0f / sqrtf(128.0f);
  a.ws = ws;
  a.out = out;
  return a;
}

void attention(int fused, Part qkv, const float *q_norm, const float *k_norm, const float *inv_freq, float eps,
               const uint16_t *qin, KVView kv, int layer, TokView tv, int max_tok, int nh, int chunk, int max_split,
               AttnWork ws, uint16_t *out, cudaStream_t st) {
  const AttnArgs a =
      attn_args(fused, qkv, q_norm, k_norm, inv_freq, eps, qin, kv, layer, tv, nh, chunk, max_split, ws, out);
  launch(k_attn, dim3(max_split, kv.n_kv, max_tok), dim3(128), 0, st, a);
}

constexpr int kSampleThreads = 512;
constexpr size_t kSampleSmem = (size_t)kSampleMaxV * 12;

__global__ void __launch_bounds__(kSampleThreads) k_sample(SampleArgs a) {
  extern __shared__ __align__(16) float smem_f[];
  __shared__ float rv[32];
  __shared__ int ri[32];
  pdl_wait();
  d_sample(a, blockIdx.x, smem_f, smem_f + kSampleMaxV, reinterpret_cast<int *>(smem_f + 2 * kSampleMaxV), rv, ri);
  pdl_launch();
}

void sample(const SampleArgs &a, int max_tok, cudaStream_t st) {
  launch(k_sample, dim3(max_tok), dim3(kSampleThreads), kSampleSmem, st, a);
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

// ---------------------------------------------------------------------------
// persistent frame kernel
// ---------------------------------------------------------------------------
constexpr int kFrameThreads = 256;
constexpr int kBarrierGroups = 16;
constexpr unsigned kSpinLimit = 1u << 22;  // ~2-3 s of polling (each poll is an L2 round trip)
// dynamic shared memory: the sampler's arrays (48 KB) cover the GEMM X tile
// (<= 64 x 264 bf16 = 33.8 KB) and two attention groups
constexpr size_t kFrameSmem = kSampleSmem;

struct FrameShared {
  Phase ph;
  float red[33];
  float rv[32];
  int ri[32];
  int abort;
};

// Grid barrier k (1-based) over all CTAs: arrival on one of 16 group
// counters (128 B apart), the last arrival of a group bumps the top counter;
// CTAs wait for top == k * 16.  Every wait is bounded: after kSpinLimit polls
// the CTA sets *err, and all CTAs leave at the next phase boundary.
__device__ bool grid_barrier(const FrameCtl &c, unsigned k, FrameShared &sh) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned grp = blockIdx.x % kBarrierGroups;
    const unsigned gsize = gridDim.x / kBarrierGroups + (grp < gridDim.x % kBarrierGroups ? 1u : 0u);
    const unsigned old = atomicAdd(&c.ctr[(1 + grp) * 32], 1u);
    if (old + 1 == k * gsize) atomicAdd(&c.ctr[0], 1u);
    unsigned spins = 0;
    int abort = 0;
    while (true) {
      unsigned v;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(c.ctr) : "memory");
      if (v >= k * kBarrierGroups) break;
      if (*(volatile int *)c.err) {
        abort = 1;
        break;
      }
      if (++spins > kSpinLimit) {
        atomicExch(c.err, 1);
        abort = 1;
        break;
      }
      __nanosleep(32);
    }
    __threadfence();
    sh.abort = abort;
  }
  __syncthreads();
  return sh.abort == 0;
}

template <int FR>
__device__ __forceinline__ void frame_gemm(const LinArgs &a, uint4 (&pre)[16], bool have_pre, uint16_t *xs) {
  const int n = linear_items(a);
  for (int item = blockIdx.x; item < n; item += gridDim.x) {
    if (!(item == (int)blockIdx.x && have_pre)) d_linear_load<FR>(a, item, pre);
    switch (a.nt) {
      case 1: d_linear_compute<1, FR>(a, item, pre, xs); break;
      case 2: d_linear_compute<2, FR>(a, item, pre, xs); break;
      case 4: d_linear_compute<4, FR>(a, item, pre, xs); break;
      default: d_linear_compute<8, FR>(a, item, pre, xs); break;
    }
  }
}

struct HalfSync {
  int id;
  __device__ void operator()() const { asm volatile("bar.sync %0, 128;" ::"r"(id) : "memory"); }
};

__global__ void __launch_bounds__(kFrameThreads, 2) k_frame(const Phase *phases, int n_phases, FrameCtl ctl) {
  extern __shared__ __align__(16) float fsm[];
  __shared__ FrameShared sh;
  uint4 pre[16];
  for (int i = 0; i < n_phases; i++) {
    // load the phase descriptor
    for (int w = threadIdx.x; w < (int)(sizeof(Phase) / 4); w += blockDim.x)
      reinterpret_cast<int *>(&sh.ph)[w] = reinterpret_cast<const int *>(&phases[i])[w];
    __syncthreads();
    const Phase &ph = sh.ph;
    // a GEMM phase streams its first item's weights before the barrier
    bool have_pre = false;
    if (ph.type == PH_GEMM && (int)blockIdx.x < linear_items(ph.lin)) {
      if (ph.lin.fr == 16)
        d_linear_load<16>(ph.lin, blockIdx.x, pre);
      else if (ph.lin.fr == 8)
        d_linear_load<8>(ph.lin, blockIdx.x, pre);
      else
        d_linear_load<4>(ph.lin, blockIdx.x, pre);
      have_pre = true;
    }
    if (i > 0 && !grid_barrier(ctl, (unsigned)i, sh)) return;
    if (ctl.t && blockIdx.x == 0 && threadIdx.x == 0) {
      unsigned long long now;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
      ctl.t[i] = now;
    }
    switch (ph.type) {
      case PH_NORM:
        for (int t = blockIdx.x; t < ph.max_tok; t += gridDim.x) d_rmsnorm(ph.norm, t, sh.red);
        break;
      case PH_GEMM: {
        uint16_t *xs = reinterpret_cast<uint16_t *>(fsm);
        if (ph.lin.fr == 16)
          frame_gemm<16>(ph.lin, pre, have_pre, xs);
        else if (ph.lin.fr == 8)
          frame_gemm<8>(ph.lin, pre, have_pre, xs);
        else
          frame_gemm<4>(ph.lin, pre, have_pre, xs);
        break;
      }
      case PH_QKV:
        for (int t = blockIdx.x; t < ph.max_tok; t += gridDim.x) d_qkv_post(ph.qkv, t);
        break;
      case PH_ATTN: {
        // two independent 128-thread groups per CTA, one item each
        const int half = threadIdx.x >> 7;
        AttnSmem *S = reinterpret_cast<AttnSmem *>(fsm) + half;
        const int nkv = ph.attn.kv.n_kv, ms = ph.attn.max_split;
        const int n_items = ph.max_tok * nkv * ms;
        for (int base = 2 * blockIdx.x; base < n_items; base += 2 * gridDim.x) {
          const int item = base + half;
          if (item < n_items) {
            const int sp = item % ms, g = (item / ms) % nkv, t = item / (ms * nkv);
            d_attn(ph.attn, sp, g, t, threadIdx.x & 127, *S, HalfSync{1 + half});
          }
        }
        break;
      }
      case PH_SILU: {
        const int chunks = (ph.silu.I / 4 + kFrameThreads - 1) / kFrameThreads;
        for (int item = blockIdx.x; item < ph.max_tok * chunks; item += gridDim.x)
          d_silu(ph.silu, item / chunks, ((item % chunks) * kFrameThreads + threadIdx.x) * 4);
        break;
      }
      case PH_SAMPLE:
        for (int t = blockIdx.x; t < ph.max_tok; t += gridDim.x) {
          d_sample(ph.smp, t, fsm, fsm + kSampleMaxV, reinterpret_cast<int *>(fsm + 2 * kSampleMaxV), sh.rv, sh.ri);
          if (ph.has_tail) d_rmsnorm(ph.tail, t, sh.red);
        }
        break;
      default:
        break;
    }
    __syncthreads();
  }
  if (ctl.t && grid_barrier(ctl, (unsigned)n_phases, sh) && blockIdx.x == 0 && threadIdx.x == 0) {
    unsigned long long now;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
    ctl.t[n_phases] = now;
  }
}

static int g_frame_grid = 0;

int frame_grid() {
  if (g_frame_grid == 0) {
    int dev = 0, sms = 0, occ = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k_frame, kFrameThreads, kFrameSmem);
    g_frame_grid = sms * (occ < 2 ? (occ < 1 ? 1 : occ) : 2);
  }
  return g_frame_grid;
}

int frame_target_items() { return frame_grid(); }

void frame_launch(const Phase *d_phases, int n_phases, FrameCtl ctl, cudaStream_t st) {
  note(cudaMemsetAsync(ctl.ctr, 0, kFrameCtrWords * sizeof(unsigned), st), "frame barrier reset");
  const int grid = frame_grid();
  void *args[] = {(void *)&d_phases, (void *)&n_phases, (void *)&ctl};
  note(cudaLaunchCooperativeKernel((const void *)k_frame, dim3(grid), dim3(kFrameThreads), args, kFrameSmem, st),
       "k_frame (cooperative)");
  g_launches++;
}

void run_phases(const Phase *ph, int n, cudaStream_t st) {
  for (int i = 0; i < n; i++) {
    const Phase &p = ph[i];
    switch (p.type) {
      case PH_NORM: rmsnorm(p.norm, p.max_tok, st); break;
      case PH_GEMM:
        switch (p.lin.nt) {
          case 1: linear_nt<1>(p.lin, st); break;
          case 2: linear_nt<2>(p.lin, st); break;
          case 4: linear_nt<4>(p.lin, st); break;
          default: linear_nt<8>(p.lin, st); break;
        }
        break;
      case PH_QKV:
        launch(k_qkv_post, dim3(p.max_tok), dim3(32 * (p.qkv.nh + 2 * p.qkv.nkv)), 0, st, p.qkv);
        break;
      case PH_ATTN:
        launch(k_attn, dim3(p.attn.max_split, p.attn.kv.n_kv, p.max_tok), dim3(128), 0, st, p.attn);
        break;
      case PH_SILU:
        launch(k_silu_mul, dim3((p.silu.I / 4 + 255) / 256, p.max_tok), dim3(256), 0, st, p.silu);
        break;
      case PH_SAMPLE:
        sample(p.smp, p.max_tok, st);
        if (p.has_tail) rmsnorm(p.tail, p.max_tok, st);
        break;
      default: break;
    }
  }
}

void init_kernel_attributes() {
  cudaFuncSetAttribute(k_sample, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSampleSmem);
  cudaFuncSetAttribute(k_frame, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kFrameSmem);
  const char *e = getenv("Q3T_PDL");
  if (e && e[0] == '0') g_use_pdl = false;
}

}  // namespace q3t

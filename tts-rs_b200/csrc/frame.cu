// Persistent frame kernel (k_frame): one cooperative, clustered launch runs a
// whole list of decode-frame phases (the same Phase records the per-phase
// kernels take: cluster split-K tcgen05 GEMMs with their epilogues, paged
// attention, RMSNorm rows, samplers with their next-input tails), with a grid
// barrier between phases instead of a kernel boundary.
//
// Why: the code-predictor loop of one frame (infer/mod.rs:434-535) is ~400
// dependent phases (15 codebooks x 5 layers x 5 kernels + heads + samplers)
// whose weight streams take ~1 us each at the HBM rate, while a kernel
// boundary (grid drain, launch, dependent-launch wait, TMEM allocation,
// barrier setup) costs several microseconds.  Here every CTA stays resident:
// TMEM is allocated once, the mbarriers are initialised once and reused by
// phase parity, and a phase starts as soon as the slowest CTA has finished
// the previous one.
//
// Work mapping.  A GEMM phase has (N / 128) row groups x token tiles virtual
// clusters of cs CTAs each (cs = the phase's K split, a divisor of the
// hardware cluster size HC); every hardware cluster hosts HC / cs of them per
// round, and the cs CTAs of a virtual cluster reduce their partial tiles
// through distributed shared memory exactly as the per-phase kernel does (rank
// order, deterministic).  Every CTA of a hardware cluster takes part in the
// cluster barriers of every round, with or without a virtual cluster.  Norm
// and sampler rows go round-robin over the CTAs; attention work units over
// the warps of the first four warps of every CTA.
//
// Every wait is bounded: an mbarrier or grid-barrier wait that gives up sets
// a bit in *err, later grid-barrier waits are skipped, and the kernel still
// runs its cluster barriers, so a launch always ends.
#include <cstdio>

#include "frame.cuh"
#include "lm_device.cuh"
#include "umma.cuh"

namespace q3t {

namespace {

constexpr int kFThreads = 256;
constexpr int kFMaxKA = 6;   // K atoms of 64 per CTA
constexpr int kFMaxN = 64;   // tokens per GEMM tile (NT = 8)
constexpr int kFW = kFMaxKA * 16384;            // weight tile: KA atoms x 128 rows x 128 B
constexpr int kFX = kFMaxKA * kFMaxN * 128;     // X tile: KA atoms x 64 rows x 128 B
constexpr int kFTileLd = 132;
constexpr int kFT = kFMaxN * kFTileLd * 4;       // f32 reduction tile [token][row]
constexpr int kFOverlay = kFX + kFT;             // attention ring / sampler arrays reuse X + tile
constexpr int kGridPolls = 1 << 22;              // ~0.5 s of 100 ns sleeps

static_assert((size_t)kAttnWarps * kAttnStages * 2 * kPageElems * 2 <= (size_t)kFOverlay, "attention ring");
static_assert((size_t)kSampleMaxV * 12 <= (size_t)kFOverlay, "sampler arrays");
static_assert(sizeof(Phase) % 16 == 0 && sizeof(Phase) / 16 <= kFThreads, "phase record copy");

struct FMisc {
  Phase ph[2];       // the current and the next phase record (copied ahead with cp.async)
  uint64_t bars[3];  // weights, X, MMA done
  uint32_t tslot;
  int abort;
  float rms[kFMaxN];
  int meta[2 * kFMaxN];
  float red[33];
  float rv[32];
  int ri[32];
  AttnSmem attn;
};

constexpr size_t kFSmem = (size_t)kFW + kFOverlay + sizeof(FMisc) + 1024;

struct FSmem {
  unsigned char *w, *x;
  float *tile;
  FMisc *m;
};

// Named barrier of warps 0..3 (the attention work group).
struct AttnGroupSync {
  __device__ void operator()() const { asm volatile("bar.sync 1, 128;" ::: "memory"); }
};

Q3T_DEV uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

Q3T_DEV unsigned ld_acquire(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Grid barrier number `i` of the launch: the counter (zeroed before the
// launch) reaches (i + 1) x grid once every CTA has arrived.
Q3T_DEV void grid_barrier(unsigned *cnt, unsigned target, FMisc &M, uint32_t &err) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(cnt, 1u);
    if (!M.abort) {
      int k = 0;
      while (ld_acquire(cnt) < target) {
        if (++k >= kGridPolls) {
          err |= 1u << 4;
          M.abort = 1;
          break;
        }
        __nanosleep(64);
      }
    }
  }
  __syncthreads();
}

// An mbarrier wait that is skipped once the CTA has given up.
Q3T_DEV bool fwait(uint64_t *bar, uint32_t parity, FMisc &M) {
  if (M.abort) return false;
  if (mbar_wait(bar, parity)) return true;
  M.abort = 1;
  return false;
}

Q3T_DEV void store_bf16x4f(uint16_t *dst, float a, float b, float c, float d) {
  uint2 p;
  p.x = pack_bf16x2(a, b);
  p.y = pack_bf16x2(c, d);
  *reinterpret_cast<uint2 *>(dst) = p;
}

// The epilogue of k_gemm (lm_kernels.cu gemm_epilogue): rows rg*128 + 4*lane
// .. +3 of token t.
Q3T_DEV void f_epilogue(const GemmArgs &a, int t, int rg, int lane, float4 v, const int *tm, float4 xpre,
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
    const float ss = warp_sum(x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w);
    if (lane == 0) a.ss_out[(size_t)rg * a.ss_ld + t] = ss;
  } else if (a.epi == GE_BIAS_SILU || a.epi == GE_BIAS_BF16) {
    const float4 b = *reinterpret_cast<const float4 *>(a.bias + n);
    const float y0 = v.x + b.x, y1 = v.y + b.y, y2 = v.z + b.z, y3 = v.w + b.w;
    if (a.epi == GE_BIAS_SILU)
      store_bf16x4f(a.h + (size_t)t * a.ldh + n, silu(y0), silu(y1), silu(y2), silu(y3));
    else
      *reinterpret_cast<float4 *>(a.y + (size_t)t * a.ldy + n) =
          make_float4(bf16_round(y0), bf16_round(y1), bf16_round(y2), bf16_round(y3));
  } else if (a.epi == GE_SILU) {
    const float ux = __shfl_xor_sync(0xffffffffu, v.x, 16), uy = __shfl_xor_sync(0xffffffffu, v.y, 16);
    const float uz = __shfl_xor_sync(0xffffffffu, v.z, 16), uw = __shfl_xor_sync(0xffffffffu, v.w, 16);
    if (lane < 16)
      store_bf16x4f(a.h + (size_t)t * a.ldh + rg * 64 + lane * 4, silu(v.x) * ux, silu(v.y) * uy, silu(v.z) * uz,
                    silu(v.w) * uw);
  } else {  // GE_QKV
    const int pos = tm[0];
    float o[4];
    if (rg < a.nh) {
      norm_rope_reg(v, gqk, fr, a.eps, lane, pos, o);
      store_bf16x4f(a.q + (size_t)t * a.nh * 128 + rg * 128 + lane * 4, o[0], o[1], o[2], o[3]);
      return;
    }
    const int h = rg < a.nh + a.nkv ? rg - a.nh : rg - a.nh - a.nkv;
    const size_t e = a.layer * a.kv.layer_stride + (((size_t)tm[1] * a.kv.n_kv + h) * 16 + (pos & 15)) * 128 + lane * 4;
    if (rg < a.nh + a.nkv) {
      norm_rope_reg(v, gqk, fr, a.eps, lane, pos, o);
      store_bf16x4f(a.kv.k + e, o[0], o[1], o[2], o[3]);
    } else {
      store_bf16x4f(a.kv.v + e, v.x, v.y, v.z, v.w);
    }
  }
}

// This CTA's part of round r of a GEMM phase: K split rank ks of virtual
// cluster (rg, tok0), whose rank 0 is hardware cluster rank base.
struct FTile {
  bool valid;
  int ks, rg, tok0;
  uint32_t base;
};

Q3T_DEV int f_rounds(const GemmArgs &a, int max_tok, int HC) {
  const int per_round = (int)(gridDim.x / HC) * (HC / a.cs);
  const int vcs = (a.N / 128) * ((max_tok + a.nt * 8 - 1) / (a.nt * 8));
  return (vcs + per_round - 1) / per_round;
}

Q3T_DEV FTile f_tile(const GemmArgs &a, int max_tok, int HC, int r) {
  const int cs = a.cs, per = HC / cs;
  const int groups = a.N / 128, vcs = groups * ((max_tok + a.nt * 8 - 1) / (a.nt * 8));
  const int nhc = gridDim.x / HC, hc = blockIdx.x / HC;
  const uint32_t hr = cluster_rank();
  const int sub = (int)hr / cs;
  const int vc = (r * nhc + hc) * per + sub;
  FTile t;
  t.valid = vc < vcs && sub < per;
  t.ks = (int)hr % cs;
  t.rg = t.valid ? vc % groups : 0;
  t.tok0 = t.valid ? (vc / groups) * a.nt * 8 : 0;
  t.base = (uint32_t)(sub * cs);
  return t;
}

// Weight-tile prefetch (thread 0): once a tile's MMAs have completed, the
// weight buffer is free and the CTA's next tile (the next round of this
// phase, or round 0 of the next GEMM phase, Phase::pad) starts loading, so
// its stream overlaps the epilogue, the grid barrier and any attention /
// norm / sampler phases in between.
struct FPrefetch {
  int phase = -1, round = -1;  // the tile whose weights are loading or loaded
  bool outstanding = false;     // issued and not yet waited for
};

// TMA tensor maps must be read from global (or parameter) memory: `ag` is
// the phase record in global memory, the scalars come from its shared copy.
Q3T_DEV void f_issue_weights(const GemmArgs &ag, const FTile &t, FMisc &M, unsigned char *w) {
  const int ka = (ag.K / 64) / ag.cs, k0 = t.ks * ka * 64;
  mbar_expect_tx(&M.bars[0], (uint32_t)ka * 16384u);
  for (int i = 0; i < ka; i++) tma_load_2d(w + i * 16384, &ag.tw, k0 + 64 * i, t.rg * 128, &M.bars[0]);
}

Q3T_DEV void stamp_f(const FrameArgs &fa, int pi, int k) {
  if (fa.trace) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    fa.trace[((size_t)blockIdx.x * fa.n + pi) * 8 + k] = t;
  }
}

// One virtual CTA of a k_gemm phase (the per-phase kernel's body, see
// lm_kernels.cu k_gemm): K split rank ks of virtual cluster (rg, tok0), whose
// rank 0 is hardware cluster rank `base`.  valid = false: this CTA hosts no
// virtual cluster in this round and only joins the cluster barriers.
// par: parity of the three mbarriers (bit b = the next phase of bars[b]).
template <int NT, int KA>
__device__ __noinline__ void f_gemm(const GemmArgs &a, const GemmArgs &ag, const FTile &tl, int pi, int r,
                                    const FrameArgs &fa, FPrefetch &pf, FSmem &S, uint32_t tmem, uint32_t &par,
                                    uint32_t &err) {
  constexpr int N = NT * 8, KC = KA * 64;
  constexpr int kXAtom = N * 128;
  FMisc &M = *S.m;
  const bool valid = tl.valid && !*(volatile int *)&M.abort;
  const int cs = a.cs, ks = tl.ks, rg = tl.rg, tok0 = tl.tok0;
  const uint32_t base = tl.base;
  const int k0 = ks * KC;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float *rms = M.rms;
  int *meta = M.meta;
  if (valid && threadIdx.x == 0 && !(pf.phase == pi && pf.round == r)) {
    f_issue_weights(ag, tl, M, S.w);
    pf.outstanding = true;
  }
  constexpr int c8n = KC / 8, rstep = 256 / c8n, NR = (N + rstep - 1) / rstep;
  const int c8 = threadIdx.x % c8n, r0 = threadIdx.x / c8n;
  float4 g0 = make_float4(0.f, 0.f, 0.f, 0.f), g1 = g0, gqk = g0, fr = g0;
  const int ts = (N + cs - 1) / cs, t_lo = ks * ts;
  float4 xres[2] = {g0, g0};
  float4 xv[KA <= 4 ? NR : 1][2];
  float ssp[16];
  int ntok = 0;
  if (valid) {
    if (a.epi == GE_QKV && rg < a.nh + a.nkv) {
      gqk = *reinterpret_cast<const float4 *>((rg < a.nh ? a.q_norm : a.k_norm) + lane * 4);
      fr = *reinterpret_cast<const float4 *>(a.inv_freq + ((lane * 4) & 63));
    }
    if constexpr (KA <= 4) {
      if (a.xmode == GX_NORM && r0 < rstep) {
        g0 = *reinterpret_cast<const float4 *>(a.gamma + k0 + c8 * 8);
        g1 = *reinterpret_cast<const float4 *>(a.gamma + k0 + c8 * 8 + 4);
      }
    }
    if (a.epi == GE_RESID) {
#pragma unroll
      for (int i = 0; i < 2; i++) {
        const int tt = t_lo + warp + 8 * i;
        if (tt < t_lo + ts && tt < N)
          xres[i] = *reinterpret_cast<const float4 *>(a.y + (size_t)(tok0 + tt) * a.ldy + rg * 128 + lane * 4);
      }
    }
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
          for (int i = 0; i < 16; i++) ssp[i] = i < a.nss ? sp[(size_t)i * a.ss_ld] : 0.f;
        }
      }
    }
    ntok = *a.ntok - tok0;
    ntok = ntok < 0 ? 0 : (ntok > N ? N : ntok);
  }
  const int t_hi = min(t_lo + ts, ntok);
  if (valid && a.epi == GE_QKV && (int)threadIdx.x < t_hi - t_lo) {
    const int t = tok0 + t_lo + threadIdx.x;
    const int pos = a.tv.pos[t] + a.tv.pos_add;
    meta[2 * threadIdx.x] = pos;
    meta[2 * threadIdx.x + 1] = a.kv.page_table[(size_t)a.tv.seq[t] * a.kv.pt_stride + (pos >> 4)];
  }
  if (valid) {
    if (a.xmode == GX_BF16) {
      if (threadIdx.x == 0) {
        mbar_expect_tx(&M.bars[1], KA * kXAtom);
#pragma unroll
        for (int i = 0; i < KA; i++) tma_load_2d(S.x + i * kXAtom, &ag.tx, k0 + 64 * i, tok0, &M.bars[1]);
      }
    } else if constexpr (KA <= 4) {
      if ((int)threadIdx.x < ntok) {
        float sum = ssp[0];
#pragma unroll
        for (int i = 1; i < 16; i++) sum += ssp[i];
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
          *reinterpret_cast<uint4 *>(S.x + (c8 >> 3) * kXAtom + r * 128 + (((c8 & 7) ^ (r & 7)) << 4)) = v;
        }
      }
      fence_proxy_async();
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) stamp_f(fa, pi, 1);
  if (valid && threadIdx.x == 0) {
    if (!fwait(&M.bars[0], par & 1u, M)) err |= 1u;
    par ^= 1u;
    pf.outstanding = false;
    stamp_f(fa, pi, 2);
    if (a.xmode == GX_BF16) {
      if (!fwait(&M.bars[1], (par >> 1) & 1u, M)) err |= 2u;
      par ^= 2u;
    }
    tc_fence_after();
    constexpr uint32_t idesc = umma_idesc_bf16(128, N);
#pragma unroll
    for (int s = 0; s < KA * 4; s++) {
      const int at = s >> 2, off = (s & 3) * 32;
      umma_kf16(tmem, sw128_desc(S.w + at * 16384 + off), sw128_desc(S.x + at * kXAtom + off), idesc,
                s > 0 ? 1u : 0u);
    }
    umma_commit(&M.bars[2]);
    // the next tile of this CTA, looked up while the MMAs run
    int npi = -1, nr = 0;
    if (r + 1 < f_rounds(a, fa.ph[pi].max_tok, fa.hc)) {
      npi = pi;
      nr = r + 1;
    } else {
      npi = fa.ph[pi].pad;
    }
    FTile nt{};
    if (npi >= 0) nt = f_tile(fa.ph[npi].gemm, fa.ph[npi].max_tok, fa.hc, nr);
    const bool mma_ok = fwait(&M.bars[2], (par >> 2) & 1u, M);
    if (!mma_ok) err |= 4u;
    par ^= 4u;
    stamp_f(fa, pi, 3);
    if (mma_ok && npi >= 0 && nt.valid) {  // the weight buffer is free once the MMAs completed
      f_issue_weights(fa.ph[npi].gemm, nt, M, S.w);
      pf.phase = npi;
      pf.round = nr;
      pf.outstanding = true;
    } else {
      pf.phase = -1;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (valid && warp < 4) {
    const uint32_t tq = tmem + ((uint32_t)(32 * warp) << 16);
    const int row = 32 * warp + lane;
#pragma unroll
    for (int c0 = 0; c0 < N; c0 += 8) {
      float v[8];
      tmem_ld8(tq + c0, v);
#pragma unroll
      for (int j = 0; j < 8; j++) S.tile[(c0 + j) * kFTileLd + row] = v[j];
    }
  }
  tc_fence_before();
  cluster_sync();
  if (threadIdx.x == 0) stamp_f(fa, pi, 4);
  if (valid) {
    for (int tt = t_lo + warp; tt < t_hi; tt += 8) {
      const float *src = S.tile + tt * kFTileLd + 4 * lane;
      float4 v;
      if (cs == 1) {
        v = *reinterpret_cast<const float4 *>(src);
      } else {
        float4 p[8];
#pragma unroll
        for (int c = 0; c < 8; c++)
          if (c < cs) p[c] = ld_cluster_f4(src, base + (uint32_t)c);
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
      const int i = (tt - t_lo - warp) >> 3;
      f_epilogue(a, tok0 + tt, rg, lane, v, meta + 2 * (tt - t_lo), i == 0 ? xres[0] : xres[1], i < 2, gqk, fr);
    }
  }
  if (threadIdx.x == 0) stamp_f(fa, pi, 5);
  cluster_sync();  // no CTA reuses its tile while another still reads it
  if (threadIdx.x == 0) stamp_f(fa, pi, 6);
}

template <int NT>
Q3T_DEV void f_gemm_ka(const GemmArgs &a, const GemmArgs &ag, const FTile &tl, int pi, int r, const FrameArgs &fa,
                       FPrefetch &pf, FSmem &S, uint32_t tmem, uint32_t &par, uint32_t &err) {
  switch ((a.K / 64) / a.cs) {
    case 2: f_gemm<NT, 2>(a, ag, tl, pi, r, fa, pf, S, tmem, par, err); break;
    case 4: f_gemm<NT, 4>(a, ag, tl, pi, r, fa, pf, S, tmem, par, err); break;
    default: f_gemm<NT, 6>(a, ag, tl, pi, r, fa, pf, S, tmem, par, err); break;
  }
}

// All rounds of a GEMM phase on this CTA.  After a give-up nothing more is
// issued (no copy or MMA can be left in flight); the CTA still joins every
// cluster and grid barrier.
Q3T_DEV void f_gemm_phase(const GemmArgs &a, const GemmArgs &ag, int max_tok, int pi, const FrameArgs &fa,
                          FPrefetch &pf, FSmem &S, uint32_t tmem, uint32_t &par, uint32_t &err) {
  const int rounds = f_rounds(a, max_tok, fa.hc);
  for (int r = 0; r < rounds; r++) {
    const FTile tl = f_tile(a, max_tok, fa.hc, r);
    switch (a.nt) {
      case 1: f_gemm_ka<1>(a, ag, tl, pi, r, fa, pf, S, tmem, par, err); break;
      case 2: f_gemm_ka<2>(a, ag, tl, pi, r, fa, pf, S, tmem, par, err); break;
      case 4: f_gemm_ka<4>(a, ag, tl, pi, r, fa, pf, S, tmem, par, err); break;
      default: f_gemm_ka<8>(a, ag, tl, pi, r, fa, pf, S, tmem, par, err); break;
    }
  }
}

// The other phase kinds, each its own function so that its register
// allocation does not add to the GEMM's.
__device__ __noinline__ void f_attn(const AttnArgs &a, FSmem &S) {
  d_attn(a, threadIdx.x, blockIdx.x * kAttnWarps, gridDim.x * kAttnWarps, S.m->attn, reinterpret_cast<uint16_t *>(S.x),
         AttnGroupSync{});
}
__device__ __noinline__ void f_norm(const RmsArgs &a, int t, FSmem &S) { d_rmsnorm(a, t, S.m->red); }
__device__ __noinline__ void f_sample(const SampleArgs &a, int t, FSmem &S) {
  float *lg = reinterpret_cast<float *>(S.x);
  d_sample(a, t, lg, lg + kSampleMaxV, reinterpret_cast<int *>(lg + 2 * kSampleMaxV), S.m->rv, S.m->ri);
}

__global__ void __launch_bounds__(kFThreads, 1) k_frame(const __grid_constant__ FrameArgs fa) {
  extern __shared__ unsigned char f_raw[];
  unsigned char *sm = f_raw + ((1024 - (smem_addr(f_raw) & 1023)) & 1023);
  FSmem S;
  S.w = sm;
  S.x = sm + kFW;
  S.tile = reinterpret_cast<float *>(sm + kFW + kFX);
  S.m = reinterpret_cast<FMisc *>(sm + kFW + kFOverlay);
  FMisc &M = *S.m;
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    mbar_init(&M.bars[0], 1);
    mbar_init(&M.bars[1], 1);
    mbar_init(&M.bars[2], 1);
    M.abort = 0;
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(&M.tslot, kFMaxN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = M.tslot;
  uint32_t par = 0, err = 0;
  FPrefetch pf;
  // phase records: phase 0 now, then each next one copied (cp.async) while the
  // current phase runs; the copy has landed before the grid barrier
  constexpr int kPhChunks = (int)(sizeof(Phase) / 16);
  auto copy_phase = [&](int i) {
    if (i < fa.n && (int)threadIdx.x < kPhChunks)
      cp_async16(reinterpret_cast<unsigned char *>(&M.ph[i & 1]) + 16 * threadIdx.x,
                 reinterpret_cast<const unsigned char *>(fa.ph + i) + 16 * threadIdx.x, 16);
    cp_async_commit();
  };
  copy_phase(0);
  cp_async_wait<0>();
  __syncthreads();
  for (int pi = 0; pi < fa.n; pi++) {
    const Phase &p = M.ph[pi & 1];
    const int type = p.type;
    if (threadIdx.x == 0) stamp_f(fa, pi, 0);
    copy_phase(pi + 1);
    if (type == PH_GEMM) {
      f_gemm_phase(p.gemm, fa.ph[pi].gemm, p.max_tok, pi, fa, pf, S, tmem, par, err);
    } else if (type == PH_ATTN) {
      if (threadIdx.x < 128) f_attn(p.attn, S);
    } else if (type == PH_NORM) {
      for (int t = blockIdx.x; t < p.max_tok; t += gridDim.x) f_norm(p.norm, t, S);
    } else if (type == PH_SAMPLE) {
      for (int t = blockIdx.x; t < p.max_tok; t += gridDim.x) {
        f_sample(p.smp, t, S);
        if (p.has_tail) f_norm(p.tail, t, S);
      }
    }
    if (threadIdx.x == 0) stamp_f(fa, pi, 7);
    cp_async_wait<0>();  // the next phase record (grid_barrier's block barrier makes it visible)
    if (pi + 1 < fa.n) grid_barrier(fa.bar, (unsigned)(pi + 1) * gridDim.x, M, err);
  }
  if (threadIdx.x == 0 && pf.outstanding) {  // a prefetch issued before a give-up lands before the CTA leaves
    if (!mbar_wait(&M.bars[0], par & 1u)) err |= 1u;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kFMaxN);
  if (err && fa.err) atomicOr(fa.err, (int)(err | (1u << 12)));
}

int g_frame_grid[64] = {0};
int g_frame_hc[64] = {0};

}  // namespace

bool frame_phase_ok(const Phase &p, int hc) {
  if (p.type == PH_GEMM) {
    const GemmArgs &a = p.gemm;
    const int atoms = a.K / 64;
    if (a.cs < 1 || hc % a.cs || atoms % a.cs) return false;
    const int ka = atoms / a.cs;
    if (ka != 2 && ka != 4 && ka != 6) return false;
    if (a.xmode == GX_NORM && ka > 4) return false;
    if (a.nt * 8 > kFMaxN) return false;
    return true;
  }
  if (p.type == PH_ATTN) return p.max_tok <= kAttnMaxTok;
  if (p.type == PH_SAMPLE) return p.smp.V <= kSampleMaxV;
  return p.type == PH_NORM;
}

bool frame_init(int device, int *grid, int *hc) {
  if (device < 0 || device >= 64) return false;
  if (g_frame_grid[device] == 0) {
    g_frame_grid[device] = -1;
    if (cudaFuncSetAttribute(k_frame, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kFSmem) != cudaSuccess) {
      cudaGetLastError();
      return false;
    }
    for (int c : {8, 4}) {  // the widest cluster that keeps most SMs busy
      cudaLaunchConfig_t cfg = {};
      cfg.blockDim = dim3(kFThreads);
      cfg.dynamicSmemBytes = kFSmem;
      cfg.gridDim = dim3(c * 16);
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = c;
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = 1;
      cfg.attrs = at;
      cfg.numAttrs = 1;
      int ncl = 0;
      if (cudaOccupancyMaxActiveClusters(&ncl, k_frame, &cfg) != cudaSuccess) {
        cudaGetLastError();
        continue;
      }
      int sms = 0;
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
      if (ncl * c >= (sms * 3) / 4) {
        g_frame_grid[device] = ncl * c;
        g_frame_hc[device] = c;
        break;
      }
    }
  }
  if (g_frame_grid[device] <= 0) return false;
  *grid = g_frame_grid[device];
  *hc = g_frame_hc[device];
  return true;
}

void frame_launch(const FrameArgs &a, int grid, cudaStream_t st) {
  if (grid <= 0 || a.hc <= 0 || grid % a.hc || a.n <= 0) {
    note_launch(cudaErrorInvalidValue, "k_frame (grid / cluster / program)");
    return;
  }
  note_launch(cudaMemsetAsync(a.bar, 0, sizeof(unsigned), st), "k_frame barrier reset");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kFThreads);
  cfg.dynamicSmemBytes = kFSmem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = a.hc;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeCooperative;
  at[1].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 2;
  note_launch(cudaLaunchKernelEx(&cfg, k_frame, a), "k_frame");
  g_launches++;
}

}  // namespace q3t

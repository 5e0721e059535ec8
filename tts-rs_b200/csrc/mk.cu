// Streamed small-batch decoder kernel (see mk.cuh for the design).
//
// The math follows the same reference code as the multi-kernel path:
// decoder layer tts_qwen3_tts/src/model/talker/network/layer.rs:23-44
// (pre-norm residual blocks), RMSNorm (burn::nn::RmsNorm, eps from the
// config), attention.rs:31-85 (q/k RMSNorm per head, rotate-half RoPE,
// :126-134), GQA attention with an f32 softmax (attention.rs:88-123,
// model/nn/attention.rs:5-27) and the SwiGLU MLP (mlp.rs:18-23).  Rounding
// points match the multi-kernel path: the GEMV inputs are bf16
// (RMSNorm(x) * gamma rounded once), q / k / v are rounded to bf16 after the
// norm and RoPE, the attention output is rounded to bf16 before o_proj, the
// residual stream stays f32.
#include <cfloat>
#include <cstdio>

#include "lm_device.cuh"
#include "mk.cuh"
#include "umma.cuh"

namespace q3t {

namespace {

// Polls of tagged data before a wait gives up (each poll is an L2 round trip
// plus a short sleep, so a wait ends after roughly a quarter of a second).
constexpr int kMkPolls = 1 << 18;

constexpr size_t kRingBytes = (size_t)kMkSlots * kMkSlot;
// float4 pieces per thread of one normalised input row of up to kMkMaxK values
constexpr int kNormPieces = (kMkMaxK + 4 * kMkWarps * 32 - 1) / (4 * kMkWarps * 32);
constexpr size_t kXsBytes = (size_t)kMkMaxTok * kMkMaxK * 2;

struct alignas(16) MkMisc {
  float red[kMkWarps][kMkMaxTok];
  float xres[kMkMaxTok][kMkMaxRes];
  float qs[2][128];
  float sc[2][kMkChunkPages * 16];  // scores, then p = exp(s - m)
  float ml[2][2];                    // running (m, l) of the unit's two query heads
  float corr[2];
  unsigned epoch;
  int abort;  // set once any wait of this CTA gave up: later waits are skipped so the launch ends quickly
  int polls;  // poll limit of the tagged-data waits
  int pad;
  uint64_t full[kMkSlots], empty[kMkSlots];
};

constexpr size_t kMkSmemBytes = kRingBytes + kXsBytes + sizeof(MkMisc) + 2 * sizeof(MkStage) + 128;

// Named barrier of the compute warps (the producer warp never joins it); the
// warp reconverges first, as the aligned barrier requires.
Q3T_DEV void bar_compute() {
  __syncwarp();
  asm volatile("bar.sync 1, %0;" ::"n"(kMkWarps * 32) : "memory");
}

// Bounded mbarrier wait that suspends the thread (up to 1 ms per poll, woken
// when the phase completes) instead of re-polling: a waiting producer or
// consumer then takes no issue slots from the compute warps.  Gives up after
// about a quarter of a second.
Q3T_DEV bool mbar_sleep_wait(uint64_t *bar, uint32_t parity) {
  const uint32_t addr = smem_addr(bar);
  for (int i = 0; i < 256; i++) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(addr), "r"(parity), "r"(1000000u)
        : "memory");
    if (ok) return true;
  }
  return false;
}

Q3T_DEV void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// 1-D bulk async copy global -> shared (16-byte aligned, bytes % 16 == 0),
// completion counted in bytes on `bar`.
Q3T_DEV void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_addr(dst)),
               "l"(src), "r"(bytes), "r"(smem_addr(bar))
               : "memory");
}

// ---- tagged words ----
Q3T_DEV unsigned tag_of(unsigned epoch, int stage) { return (epoch << 10) | (unsigned)stage; }
Q3T_DEV uint4 ld_tag4(const uint2 *p) {  // two consecutive tagged words
  uint4 v;
  asm volatile("ld.relaxed.gpu.global.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
Q3T_DEV uint2 ld_tag2(const uint2 *p) {
  uint2 v;
  asm volatile("ld.relaxed.gpu.global.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p) : "memory");
  return v;
}
Q3T_DEV void st_tag(uint2 *p, float v, unsigned tag) {
  asm volatile("st.relaxed.gpu.global.v2.u32 [%0], {%1,%2};" ::"l"(p), "r"(__float_as_uint(v)), "r"(tag) : "memory");
}
// One more poll of a tagged wait?  false once the CTA gave up (or now gives up).
Q3T_DEV bool poll_again(MkMisc &M, int &k, uint32_t &err) {
  if (*(volatile int *)&M.abort) return false;
  if (++k >= M.polls) {
    err |= 1u << 8;
    *(volatile int *)&M.abort = 1;
    return false;
  }
  __nanosleep(20);
  return true;
}

// 4 consecutive values t, k..k+3 of an input (plain or tagged); ok &= tags match
Q3T_DEV float4 in_load4(const MkIn &in, int t, int k, unsigned tag, bool &ok) {
  if (in.stage < 0) return *reinterpret_cast<const float4 *>(in.f + (size_t)t * in.ld + k);
  const uint2 *p = in.w + (size_t)t * in.ld + k;
  const uint4 a = ld_tag4(p), b = ld_tag4(p + 2);
  ok = ok && a.y == tag && a.w == tag && b.y == tag && b.w == tag;
  return make_float4(__uint_as_float(a.x), __uint_as_float(a.z), __uint_as_float(b.x), __uint_as_float(b.z));
}
Q3T_DEV float in_load1(const MkIn &in, int t, int k, unsigned tag, bool &ok) {
  if (in.stage < 0) return in.f[(size_t)t * in.ld + k];
  const uint2 v = ld_tag2(in.w + (size_t)t * in.ld + k);
  ok = ok && v.y == tag;
  return __uint_as_float(v.x);
}

Q3T_DEV void unpack8(const uint4 &u, float *f) {
  f[0] = __uint_as_float(u.x << 16);
  f[1] = __uint_as_float(u.x & 0xffff0000u);
  f[2] = __uint_as_float(u.y << 16);
  f[3] = __uint_as_float(u.y & 0xffff0000u);
  f[4] = __uint_as_float(u.z << 16);
  f[5] = __uint_as_float(u.z & 0xffff0000u);
  f[6] = __uint_as_float(u.w << 16);
  f[7] = __uint_as_float(u.w & 0xffff0000u);
}

Q3T_DEV unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
Q3T_DEV void stamp(const MkArgs &a, int si, int k) {
  if (a.trace) a.trace[((size_t)blockIdx.x * a.n + si) * 8 + k] = globaltimer();
}

Q3T_DEV int ntok_of(const MkArgs &a) {
  const int n = *a.tv.ntok;
  return n < 0 ? 0 : (n > kMkMaxTok ? kMkMaxTok : n);
}

// ---- work partition (producer and consumers derive the same lists) --------

// rows [r0, r1) (or pairs, for gate/up) of CTA c out of G
Q3T_DEV void gemv_slice(const MkGemv &g, int c, int G, int &r0, int &r1) {
  const long long n = g.pairs ? g.N / 2 : g.N;
  r0 = (int)(n * c / G);
  r1 = (int)(n * (c + 1) / G);
}
// rows (pairs) per ring slot
Q3T_DEV int gemv_chunk(const MkGemv &g) {
  const int rows = kMkSlot / (2 * g.K);
  return g.pairs ? rows / 2 : rows;
}
// end of the chunk starting at `a` (pairs never cross a 64-pair block)
Q3T_DEV int gemv_chunk_end(const MkGemv &g, int a, int r1) {
  int b = a + gemv_chunk(g);
  if (b > r1) b = r1;
  if (g.pairs) {
    const int blk = (a / 64 + 1) * 64;
    if (b > blk) b = blk;
  }
  return b;
}

// Attention units: (token t, kv head h, pages [pb, pe)) numbered token-major,
// heads, then page runs; CTA c takes units c, c + G, ...
struct MkPlan {
  int T, ppu, total;
  int pos[kMkMaxTok], pages[kMkMaxTok], nu[kMkMaxTok], base[kMkMaxTok + 1];
};

Q3T_DEV void attn_plan(const MkArgs &a, int T, int nkv, int G, MkPlan &P) {
  P.T = T;
  int tot = 0;
  for (int t = 0; t < T; t++) {
    P.pos[t] = a.tv.pos[t] + a.tv.pos_add;
    P.pages[t] = (P.pos[t] + 16) >> 4;
    tot += P.pages[t];
  }
  int ppu = (tot * nkv + G - 1) / G;
  if (ppu < 1) ppu = 1;
  for (int t = 0; t < T; t++) {
    const int need = (P.pages[t] + kAttnMaxUnits - 1) / kAttnMaxUnits;
    if (ppu < need) ppu = need;
  }
  P.ppu = ppu;
  P.base[0] = 0;
  for (int t = 0; t < T; t++) {
    P.nu[t] = (P.pages[t] + ppu - 1) / ppu;
    P.base[t + 1] = P.base[t] + P.nu[t] * nkv;
  }
  P.total = P.base[T];
}

Q3T_DEV void attn_unit_of(const MkPlan &P, int u, int &t, int &h, int &j, int &pb, int &pe) {
  t = 0;
  while (t + 1 < P.T && P.base[t + 1] <= u) t++;
  const int r = u - P.base[t];
  h = r / P.nu[t];
  j = r - h * P.nu[t];
  pb = j * P.ppu;
  pe = min(pb + P.ppu, P.pages[t]);
}

// ---- producer: one thread streams every stage's bytes into the ring -------

// Once the CTA has given up (M.abort) the producer issues nothing more: the
// consumers then skip their waits and may release a slot whose copy has not
// landed, so a later copy into that slot could overlap it.  The abort check
// after the slot wait sees every abort made before the consumers released the
// slot (their arrive is a release, the wait an acquire), so at most one copy
// per slot is ever in flight and the kernel's final wait on each slot's last
// chunk covers every copy issued.
Q3T_DEV void produce(const MkArgs &a, unsigned char *ring, MkMisc &M, int T, uint32_t *last_chunk) {
  const int c = blockIdx.x, G = gridDim.x;
  uint32_t i = 0;
  uint32_t err = 0;
  auto acquire_slot = [&](uint32_t bytes) -> unsigned char * {
    const int s = (int)(i % kMkSlots);
    if (*(volatile int *)&M.abort) return nullptr;
    if (!mbar_sleep_wait(&M.empty[s], ((i / kMkSlots) & 1u) ^ 1u)) {
      err |= 1u << 9;
      *(volatile int *)&M.abort = 1;
    }
    if (*(volatile int *)&M.abort) return nullptr;
    mbar_expect_tx(&M.full[s], bytes);
    last_chunk[s] = i;
    i++;
    return ring + (size_t)s * kMkSlot;
  };
  for (int si = 0; si < a.n; si++) {
    const MkStage &S = a.st[si];
    stamp(a, si, 5);
    if (S.op == MK_GEMV) {
      const MkGemv &g = S.g;
      int r0, r1;
      gemv_slice(g, c, G, r0, r1);
      const size_t rb = (size_t)g.K * 2;
      for (int p = r0; p < r1;) {
        const int q = gemv_chunk_end(g, p, r1), np = q - p;
        const int s = (int)(i % kMkSlots);
        unsigned char *dst = acquire_slot((uint32_t)(np * rb * (g.pairs ? 2 : 1)));
        if (!dst) goto done;
        if (p == r0) stamp(a, si, 6);
        if (g.pairs) {
          const size_t rg = (size_t)128 * (p / 64) + (p % 64);
          bulk_g2s(dst, g.w + rg * g.K, (uint32_t)(np * rb), &M.full[s]);
          bulk_g2s(dst + np * rb, g.w + (rg + 64) * g.K, (uint32_t)(np * rb), &M.full[s]);
        } else {
          bulk_g2s(dst, g.w + (size_t)p * g.K, (uint32_t)(np * rb), &M.full[s]);
        }
        p = q;
      }
    } else if (S.op == MK_ATTN) {
      const MkAttn &at = S.a;
      MkPlan P;
      attn_plan(a, T, at.kv.n_kv, G, P);
      const uint16_t *kb = at.kv.k + (size_t)at.layer * at.kv.layer_stride;
      const uint16_t *vb = at.kv.v + (size_t)at.layer * at.kv.layer_stride;
      for (int u = c; u < P.total; u += G) {
        int t, h, j, pb, pe;
        attn_unit_of(P, u, t, h, j, pb, pe);
        const int *pt = at.kv.page_table + (size_t)a.tv.seq[t] * at.kv.pt_stride;
        int pages[kMkChunkPages];
        for (int p = pb; p < pe; p += kMkChunkPages) {
          const int np = min(kMkChunkPages, pe - p);
#pragma unroll
          for (int e = 0; e < kMkChunkPages; e++) pages[e] = e < np ? pt[p + e] : 0;
          const int s = (int)(i % kMkSlots);
          unsigned char *dst = acquire_slot((uint32_t)np * 8192u);
          if (!dst) goto done;
          if (p == pb && u == c) stamp(a, si, 6);
          for (int e = 0; e < np; e++) {
            const size_t off = ((size_t)pages[e] * at.kv.n_kv + h) * (16 * 128);
            bulk_g2s(dst + e * 4096, kb + off, 4096u, &M.full[s]);
            bulk_g2s(dst + 16384 + e * 4096, vb + off, 4096u, &M.full[s]);
          }
        }
      }
    }
  }
done:
  if (err && a.err) atomicOr(a.err, (int)err);
}

// ---- consumers: eight warps -----------------------------------------------

// Waits for ring chunk ci to land (skipped once the CTA has given up).
Q3T_DEV void wait_full(MkMisc &M, uint32_t ci, uint32_t &err) {
  const int s = (int)(ci % kMkSlots);
  if (!*(volatile int *)&M.abort && !mbar_sleep_wait(&M.full[s], (ci / kMkSlots) & 1u)) {
    err |= 1u << 9;
    *(volatile int *)&M.abort = 1;
  }
}

// Rows [p, q) of a ring chunk that belong to this warp ((r - r0) % 8 == warp):
// KI 16-byte pieces per lane per row, T tokens, gate/up pairs when PAIRS.
template <int KI, int T, bool PAIRS>
Q3T_DEV void gemv_rows(const MkGemv &g, const unsigned char *slot, int p, int q, int r0, const uint16_t *xs,
                       const MkMisc &M, unsigned tag, int warp, int lane) {
  constexpr int K8 = KI * 32;
  const int np = q - p;
  const uint4 *xs4 = reinterpret_cast<const uint4 *>(xs);
  for (int r = p + ((warp - (p - r0)) % kMkWarps + kMkWarps) % kMkWarps; r < q; r += kMkWarps) {
    const uint4 *w0 = reinterpret_cast<const uint4 *>(slot + (size_t)(r - p) * K8 * 16);
    const uint4 *w1 = reinterpret_cast<const uint4 *>(slot + (size_t)(np + r - p) * K8 * 16);
    uint4 wv[KI], uv[PAIRS ? KI : 1];
#pragma unroll
    for (int i = 0; i < KI; i++) {
      wv[i] = w0[lane + 32 * i];
      if (PAIRS) uv[i] = w1[lane + 32 * i];
    }
    float acc[T][2], accu[T][2];
#pragma unroll
    for (int t = 0; t < T; t++) acc[t][0] = acc[t][1] = accu[t][0] = accu[t][1] = 0.f;
#pragma unroll
    for (int i = 0; i < KI; i++) {
      float wf[8], uf[8];
      unpack8(wv[i], wf);
      if (PAIRS) unpack8(uv[PAIRS ? i : 0], uf);
#pragma unroll
      for (int t = 0; t < T; t++) {
        float xf[8];
        unpack8(xs4[t * K8 + lane + 32 * i], xf);
#pragma unroll
        for (int e = 0; e < 8; e++) {
          acc[t][e & 1] = fmaf(wf[e], xf[e], acc[t][e & 1]);
          if (PAIRS) accu[t][e & 1] = fmaf(uf[e], xf[e], accu[t][e & 1]);
        }
      }
    }
    float v0 = 0.f, v1 = 0.f;
#pragma unroll
    for (int t = 0; t < T; t++) {
      const float s0 = warp_sum(acc[t][0] + acc[t][1]);
      const float s1 = PAIRS ? warp_sum(accu[t][0] + accu[t][1]) : 0.f;
      if (lane == t) v0 = s0, v1 = s1;
    }
    if (lane < T) {
      const int t = lane;
      if (PAIRS) {
        st_tag(g.yt + (size_t)t * g.ldy + r, bf16_round(silu(v0) * v1), tag);
      } else if (g.epi == MKE_F32) {
        g.y[(size_t)t * g.ldy + r] = v0;
      } else if (g.epi == MKE_TAG) {
        st_tag(g.yt + (size_t)t * g.ldy + r, v0, tag);
      } else {
        st_tag(g.yt + (size_t)t * g.ldy + r, M.xres[t][r - r0] + v0, tag);
      }
    }
  }
}

template <int KI, int T>
Q3T_DEV void gemv_rows_p(const MkGemv &g, const unsigned char *slot, int p, int q, int r0, const uint16_t *xs,
                         const MkMisc &M, unsigned tag, int warp, int lane) {
  if (g.pairs)
    gemv_rows<KI, T, true>(g, slot, p, q, r0, xs, M, tag, warp, lane);
  else
    gemv_rows<KI, T, false>(g, slot, p, q, r0, xs, M, tag, warp, lane);
}
template <int KI>
Q3T_DEV void gemv_rows_t(int T, const MkGemv &g, const unsigned char *slot, int p, int q, int r0,
                         const uint16_t *xs, const MkMisc &M, unsigned tag, int warp, int lane) {
  switch (T) {
    case 1: gemv_rows_p<KI, 1>(g, slot, p, q, r0, xs, M, tag, warp, lane); break;
    case 2: gemv_rows_p<KI, 2>(g, slot, p, q, r0, xs, M, tag, warp, lane); break;
    default: break;
  }
}

Q3T_DEV void gemv_stage(const MkArgs &a, int si, const MkGemv &g, int T, unsigned char *ring, unsigned char *xsb,
                        MkMisc &M, uint32_t &ci, uint32_t &err) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x, G = gridDim.x, K = g.K, K8 = K / 8;
  uint16_t *xs = reinterpret_cast<uint16_t *>(xsb);
  int r0, r1;
  gemv_slice(g, c, G, r0, r1);
  if (r0 >= r1 && !(g.hid_out && c == 0)) return;  // no rows here: nothing to read or write
  const bool res = g.epi == MKE_RESID;
  const unsigned otag = tag_of(M.epoch, si);
  // ---- residual rows of this slice (RESID; at most kMkMaxRes per token) ----
  float rv[2] = {0.f, 0.f};
  if (res) {
    const unsigned rtag = tag_of(M.epoch, g.res.stage);
#pragma unroll
    for (int i = 0; i < 2; i++) {
      const int e = tid + i * kMkWarps * 32;
      if (e < T * (r1 - r0)) {
        const int t = e / (r1 - r0), r = e - t * (r1 - r0);
        int k = 0;
        bool ok;
        do {
          ok = true;
          rv[i] = in_load1(g.res, t, r0 + r, rtag, ok);
        } while (!ok && poll_again(M, k, err));
      }
    }
  }
  // ---- X rows into shared memory (bf16 [T][K]) ----
  if (g.xsrc == MKX_NORM) {
    float4 gm[kNormPieces];
#pragma unroll
    for (int e = 0; e < kNormPieces; e++) {
      const int k = (tid + e * kMkWarps * 32) * 4;
      gm[e] = k < K ? *reinterpret_cast<const float4 *>(g.gamma + k) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const unsigned xtag = tag_of(M.epoch, g.x.stage);
    float4 v[kMkMaxTok][kNormPieces];
    float ss[kMkMaxTok];
#pragma unroll
    for (int t = 0; t < kMkMaxTok; t++) {
      ss[t] = 0.f;
#pragma unroll
      for (int e = 0; e < kNormPieces; e++) {
        const int k = (tid + e * kMkWarps * 32) * 4;
        v[t][e] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (t < T && k < K) {
          int kk = 0;
          bool ok;
          do {
            ok = true;
            v[t][e] = in_load4(g.x, t, k, xtag, ok);
          } while (!ok && poll_again(M, kk, err));
          ss[t] += v[t][e].x * v[t][e].x + v[t][e].y * v[t][e].y + v[t][e].z * v[t][e].z + v[t][e].w * v[t][e].w;
        }
      }
    }
    if (tid == 0) stamp(a, si, 0);
#pragma unroll
    for (int t = 0; t < kMkMaxTok; t++) {
      const float s = warp_sum(ss[t]);
      if (lane == 0) M.red[warp][t] = s;
    }
    bar_compute();  // also: the previous stage's rows are done with xs
    float d[kMkMaxTok];
#pragma unroll
    for (int t = 0; t < kMkMaxTok; t++) {
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < kMkWarps; w++) s += M.red[w][t];
      d[t] = 1.f / sqrtf(s / (float)K + g.eps);
    }
#pragma unroll
    for (int e = 0; e < kNormPieces; e++) {
      const int k = (tid + e * kMkWarps * 32) * 4;
      if (k < K) {
#pragma unroll
        for (int t = 0; t < kMkMaxTok; t++) {
          if (t < T) {
            const float4 y = make_float4(v[t][e].x * d[t] * gm[e].x, v[t][e].y * d[t] * gm[e].y,
                                         v[t][e].z * d[t] * gm[e].z, v[t][e].w * d[t] * gm[e].w);
            uint2 p;
            p.x = pack_bf16x2(y.x, y.y);
            p.y = pack_bf16x2(y.z, y.w);
            *reinterpret_cast<uint2 *>(xs + (size_t)t * K + k) = p;
            if (g.hid_out && c == 0) *reinterpret_cast<float4 *>(g.hid_out + (size_t)g.hid_slot[t] * K + k) = y;
          }
        }
      }
    }
  } else {  // MKX_TAGGED
    const unsigned xtag = tag_of(M.epoch, g.x.stage);
    constexpr int kMaxPk = kMkMaxTok * kMkMaxK / 8 / (kMkWarps * 32);  // 16-byte pieces per thread
    uint4 pk[kMaxPk];
#pragma unroll
    for (int i = 0; i < kMaxPk; i++) {
      const int e = tid + i * kMkWarps * 32;
      pk[i] = make_uint4(0u, 0u, 0u, 0u);
      if (e < T * K8) {
        const int t = e / K8, q = e - t * K8;
        int kk = 0;
        bool ok;
        float4 lo, hi;
        do {
          ok = true;
          lo = in_load4(g.x, t, q * 8, xtag, ok);
          hi = in_load4(g.x, t, q * 8 + 4, xtag, ok);
        } while (!ok && poll_again(M, kk, err));
        pk[i] = make_uint4(pack_bf16x2(lo.x, lo.y), pack_bf16x2(lo.z, lo.w), pack_bf16x2(hi.x, hi.y),
                           pack_bf16x2(hi.z, hi.w));
      }
    }
    if (tid == 0) stamp(a, si, 0);
    bar_compute();  // the previous stage's rows are done with xs
#pragma unroll
    for (int i = 0; i < kMaxPk; i++) {
      const int e = tid + i * kMkWarps * 32;
      if (e < T * K8) reinterpret_cast<uint4 *>(xs)[e] = pk[i];
    }
  }
  if (res)
#pragma unroll
    for (int i = 0; i < 2; i++) {
      const int e = tid + i * kMkWarps * 32;
      if (e < T * (r1 - r0)) M.xres[e / (r1 - r0)][e % (r1 - r0)] = rv[i];
    }
  bar_compute();
  if (tid == 0) stamp(a, si, 1);
  // ---- chunks of rows from the ring ----
  for (int p = r0; p < r1;) {
    const int q = gemv_chunk_end(g, p, r1);
    const int s = (int)(ci % kMkSlots);
    wait_full(M, ci, err);
    if (p == r0 && tid == 0) stamp(a, si, 2);
    const unsigned char *slot = ring + (size_t)s * kMkSlot;
    switch (K) {
      case 1024: gemv_rows_t<4>(T, g, slot, p, q, r0, xs, M, otag, warp, lane); break;
      case 2048: gemv_rows_t<8>(T, g, slot, p, q, r0, xs, M, otag, warp, lane); break;
      case 3072: gemv_rows_t<12>(T, g, slot, p, q, r0, xs, M, otag, warp, lane); break;
      default: break;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&M.empty[s]);
    if (tid == 0) stamp(a, si, p == r0 ? 4 : 7);
    ci++;
    p = q;
  }
}

Q3T_DEV void attn_stage(const MkArgs &a, int si, const MkAttn &at, int T, unsigned char *ring, MkMisc &M,
                        uint32_t &ci, uint32_t &err) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x, G = gridDim.x;
  const int nkv = at.kv.n_kv, nh = at.nh;
  const unsigned itag = tag_of(M.epoch, at.qkv_stage), otag = tag_of(M.epoch, si);
  MkPlan P;
  attn_plan(a, T, nkv, G, P);
  const int hh = tid >> 7, d = tid & 127;  // p.v thread: head 2h + hh, dim d
  const MkIn qin{nullptr, at.qkv, 0, at.ldq};
  // constants of the stage, loaded before any wait
  const float4 gq = *reinterpret_cast<const float4 *>(at.q_norm + 4 * lane);
  const float4 gk = *reinterpret_cast<const float4 *>(at.k_norm + 4 * lane);
  const float4 fr = *reinterpret_cast<const float4 *>(at.inv_freq + ((4 * lane) & 63));
  bool first = true;
  for (int u = c; u < P.total; u += G) {
    int t, h, j, pb, pe;
    attn_unit_of(P, u, t, h, j, pb, pe);
    const int pos = P.pos[t], L = pos + 1;
    const int seq = a.tv.seq[t];
    // new keys of this launch visible to token t: its own position and those
    // of the tokens right before it in the same sequence (a prompt pair)
    int nd = 1;
    while (nd <= t && a.tv.seq[t - nd] == seq && P.pos[t - nd] == pos - nd) nd++;
    // raw rows: q of heads 2h, 2h + 1 (warps 0, 1); the new keys' k / v
    // (warps 2dd, 2dd + 1 for key pos - dd) if they fall in this unit
    const int kp = pos - (warp >> 1);
    const bool has_new = warp < 2 * nd && kp >= pb * 16 && kp < pe * 16;
    float4 qv = make_float4(0.f, 0.f, 0.f, 0.f), raw = make_float4(0.f, 0.f, 0.f, 0.f);
    if (warp < 2 || has_new) {
      int k = 0;
      bool ok;
      do {
        ok = true;
        if (warp < 2) qv = in_load4(qin, t, (2 * h + warp) * 128 + 4 * lane, itag, ok);
        if (has_new)
          raw = in_load4(qin, t - (warp >> 1), ((warp & 1 ? nh + nkv : nh) + h) * 128 + 4 * lane, itag, ok);
      } while (!__all_sync(0xffffffffu, ok) && poll_again(M, k, err));
    }
    if (first && tid == 0) stamp(a, si, 0);
    first = false;
    if (warp < 2) {
      float o4[4];
      norm_rope_reg(qv, gq, fr, at.eps, lane, pos, o4);
#pragma unroll
      for (int e = 0; e < 4; e++) M.qs[warp][4 * lane + e] = bf16_round(o4[e]);
      if (lane == 0) {
        M.ml[warp][0] = -FLT_MAX;
        M.ml[warp][1] = 0.f;
      }
    }
    bar_compute();
    float q0[4], q1[4];
#pragma unroll
    for (int e = 0; e < 4; e++) {
      q0[e] = M.qs[0][4 * lane + e];
      q1[e] = M.qs[1][4 * lane + e];
    }
    float o = 0.f;
    for (int p = pb; p < pe; p += kMkChunkPages) {
      const int np = min(kMkChunkPages, pe - p);
      const int s = (int)(ci % kMkSlots);
      wait_full(M, ci, err);
      unsigned char *ks = ring + (size_t)s * kMkSlot, *vs = ks + 16384;
      const int k0 = p * 16, nk = min(np * 16, L - k0);
      // keys written by this launch: normed, roped and rounded from the raw
      // rows; the owning token's unit appends them to the cache
      if (has_new && kp >= k0 && kp < k0 + nk) {
        const int row = kp - k0;
        uint16_t *srow = reinterpret_cast<uint16_t *>((warp & 1 ? vs : ks) + (row >> 4) * 4096 + (row & 15) * 256);
        float o4[4] = {raw.x, raw.y, raw.z, raw.w};
        if (!(warp & 1)) norm_rope_reg(raw, gk, fr, at.eps, lane, kp, o4);
        uint2 pk;
        pk.x = pack_bf16x2(o4[0], o4[1]);
        pk.y = pack_bf16x2(o4[2], o4[3]);
        *reinterpret_cast<uint2 *>(srow + 4 * lane) = pk;
        if (warp < 2) {  // token t's own key
          const int page = at.kv.page_table[(size_t)seq * at.kv.pt_stride + (kp >> 4)];
          uint16_t *base = (warp & 1 ? at.kv.v : at.kv.k) + (size_t)at.layer * at.kv.layer_stride;
          *reinterpret_cast<uint2 *>(base + (((size_t)page * nkv + h) * 16 + (kp & 15)) * 128 + 4 * lane) = pk;
        }
      }
      bar_compute();
      // scores: warp w takes keys w, w + 8, ... (all loads first, then the
      // 16 reductions interleaved)
      {
        constexpr int kPer = (kMkChunkPages * 16 + kMkWarps - 1) / kMkWarps;  // keys per warp
        float s0[kPer], s1[kPer];
#pragma unroll
        for (int i = 0; i < kPer; i++) {
          const int kk = warp + kMkWarps * i;
          s0[i] = s1[i] = 0.f;
          if (kk < nk) {
            const uint2 kr = *reinterpret_cast<const uint2 *>(ks + (kk >> 4) * 4096 + (kk & 15) * 256 + lane * 8);
            const float k4[4] = {__uint_as_float(kr.x << 16), __uint_as_float(kr.x & 0xffff0000u),
                                 __uint_as_float(kr.y << 16), __uint_as_float(kr.y & 0xffff0000u)};
#pragma unroll
            for (int e = 0; e < 4; e++) {
              s0[i] = fmaf(q0[e], k4[e], s0[i]);
              s1[i] = fmaf(q1[e], k4[e], s1[i]);
            }
          }
        }
#pragma unroll
        for (int o2 = 16; o2 > 0; o2 >>= 1)
#pragma unroll
          for (int i = 0; i < kPer; i++) {
            s0[i] += __shfl_xor_sync(0xffffffffu, s0[i], o2);
            s1[i] += __shfl_xor_sync(0xffffffffu, s1[i], o2);
          }
        if (lane == 0)
#pragma unroll
          for (int i = 0; i < kPer; i++) {
            const int kk = warp + kMkWarps * i;
            if (kk < nk) {
              M.sc[0][kk] = s0[i] * at.scale;
              M.sc[1][kk] = s1[i] * at.scale;
            }
          }
      }
      bar_compute();
      // online softmax per head (warps 0, 1): p = exp(s - m_new) once per key
      if (warp < 2) {
        const float a0 = lane < nk ? M.sc[warp][lane] : -FLT_MAX;
        const float a1 = lane + 32 < nk ? M.sc[warp][lane + 32] : -FLT_MAX;
        const float mold = M.ml[warp][0];
        const float mn = fmaxf(mold, warp_max(fmaxf(a0, a1)));
        const float p0 = lane < nk ? expf(a0 - mn) : 0.f, p1 = lane + 32 < nk ? expf(a1 - mn) : 0.f;
        M.sc[warp][lane] = p0;
        M.sc[warp][lane + 32] = p1;
        const float ps = warp_sum(p0 + p1);
        if (lane == 0) {
          const float cr = expf(mold - mn);
          M.ml[warp][0] = mn;
          M.ml[warp][1] = M.ml[warp][1] * cr + ps;
          M.corr[warp] = cr;
        }
      }
      bar_compute();
      // o = o * corr + p . V (thread (hh, d), the first 256 threads)
      if (tid < 256) {
        const uint16_t *vcol = reinterpret_cast<const uint16_t *>(vs) + d;
        const float *pr = M.sc[hh];
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        int kk = 0;
        for (; kk + 4 <= nk; kk += 4) {
#pragma unroll
          for (int e = 0; e < 4; e++)
            acc[e] = fmaf(pr[kk + e], bf2f(vcol[((kk + e) >> 4) * 2048 + ((kk + e) & 15) * 128]), acc[e]);
        }
        for (; kk < nk; kk++) acc[0] = fmaf(pr[kk], bf2f(vcol[(kk >> 4) * 2048 + (kk & 15) * 128]), acc[0]);
        o = o * M.corr[hh] + ((acc[0] + acc[1]) + (acc[2] + acc[3]));
      }
      bar_compute();  // the slot and sc are free again
      if (lane == 0) mbar_arrive(&M.empty[s]);
      ci++;
    }
    if (tid >= 256) {
    } else if (P.nu[t] == 1) {  // the whole key range: the output itself
      st_tag(at.out + (size_t)t * at.ldo + (2 * h + hh) * 128 + d, bf16_round(o / M.ml[hh][1]), otag);
    } else {  // an (o, m, l) partial, merged below by unit 0 of (t, h)
      uint2 *Pj = at.part + ((((size_t)t * nkv + h) * kAttnMaxUnits + j) * 2 + hh) * kMkPartLd;
      st_tag(Pj + d, o, otag);
      if (d == 0) {
        st_tag(Pj + 128, M.ml[hh][0], otag);
        st_tag(Pj + 129, M.ml[hh][1], otag);
      }
    }
    bar_compute();  // qs / ml are rewritten by the next unit
  }
  // Merges, after all of this CTA's units (a merge waits on other CTAs'
  // units; none of those waits on this CTA): unit 0 of (t, h) combines the
  // partials of units 0..nu-1 in unit order (the multi-kernel path's order
  // and math) and writes query heads 2h, 2h + 1 rounded to bf16.
  for (int u = c; u < P.total; u += G) {
    int t, h, j, pb, pe;
    attn_unit_of(P, u, t, h, j, pb, pe);
    const int nu = P.nu[t];
    if (j != 0 || nu == 1 || tid >= 256) continue;
    const uint2 *P0 = at.part + (((size_t)t * nkv + h) * kAttnMaxUnits * 2 + hh) * kMkPartLd;
    float Mx = -FLT_MAX, Ls = 0.f, acc = 0.f;
    for (int r0 = 0; r0 < nu; r0 += 8) {
      float om[8], mm[8], ll[8];
      int k = 0;
      bool ok;
      do {
        ok = true;
#pragma unroll
        for (int i = 0; i < 8; i++) {
          om[i] = mm[i] = ll[i] = 0.f;
          if (r0 + i < nu) {
            const uint2 *Pr = P0 + (size_t)(r0 + i) * 2 * kMkPartLd;
            const uint2 ov = ld_tag2(Pr + d), m2 = ld_tag2(Pr + 128), l2 = ld_tag2(Pr + 129);
            ok = ok && ov.y == otag && m2.y == otag && l2.y == otag;
            om[i] = __uint_as_float(ov.x);
            mm[i] = __uint_as_float(m2.x);
            ll[i] = __uint_as_float(l2.x);
          }
        }
      } while (!ok && poll_again(M, k, err));
#pragma unroll
      for (int i = 0; i < 8; i++) {
        if (r0 + i < nu) {
          const float Mn = fmaxf(Mx, mm[i]), fa = expf(Mx - Mn), fb = expf(mm[i] - Mn);
          Ls = Ls * fa + ll[i] * fb;
          acc = acc * fa + om[i] * fb;
          Mx = Mn;
        }
      }
    }
    st_tag(at.out + (size_t)t * at.ldo + (2 * h + hh) * 128 + d, bf16_round(acc / Ls), otag);
  }
}

__global__ void __launch_bounds__(kMkThreads, 1) k_mk(const __grid_constant__ MkArgs a) {
  extern __shared__ unsigned char mk_raw[];
  unsigned char *sm = mk_raw + ((128 - (smem_addr(mk_raw) & 127)) & 127);
  unsigned char *ring = sm, *xsb = sm + kRingBytes;
  MkMisc &M = *reinterpret_cast<MkMisc *>(xsb + kXsBytes);
  MkStage *St = reinterpret_cast<MkStage *>(xsb + kXsBytes + sizeof(MkMisc));  // [2], by stage parity
  const int warp = threadIdx.x >> 5;
  __shared__ uint32_t last_chunk[kMkSlots];
  if (threadIdx.x == 0) {
    for (int s = 0; s < kMkSlots; s++) {
      mbar_init(&M.full[s], 1);
      mbar_init(&M.empty[s], kMkWarps);
      last_chunk[s] = 0xffffffffu;
    }
    M.abort = 0;
    M.polls = a.polls > 0 ? a.polls : kMkPolls;
    M.epoch = a.ctr[0];
    fence_mbar_init();
  }
  __syncthreads();
  const int T = ntok_of(a);
  uint32_t err = 0;
  if (warp == kMkWarps) {
    if ((threadIdx.x & 31) == 0) produce(a, ring, M, T, last_chunk);
    __syncwarp();
  } else {
    uint32_t ci = 0;
    if (a.stall && threadIdx.x == 0) {  // a plain global-memory wait for a word nothing sets
      int k = 0;
      while (*(volatile const int *)a.stall != 1 && poll_again(M, k, err)) {
      }
    }
    constexpr int n16 = sizeof(MkStage) / 16;
    static_assert(sizeof(MkStage) % 16 == 0, "MkStage is copied in 16-byte pieces");
    for (int si = 0; si < a.n; si++) {
      // the descriptor (independent of other CTAs) into the buffer of this
      // parity: every warp left stage si - 2 before it passed stage si - 1's
      // staging barrier
      MkStage &S = St[si & 1];
      if ((int)threadIdx.x < n16)
        reinterpret_cast<uint4 *>(&S)[threadIdx.x] = reinterpret_cast<const uint4 *>(a.st + si)[threadIdx.x];
      bar_compute();
      if (S.op == MK_GEMV)
        gemv_stage(a, si, S.g, T, ring, xsb, M, ci, err);
      else
        attn_stage(a, si, S.a, T, ring, M, ci, err);
      if (threadIdx.x == 0) stamp(a, si, 3);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // every issued copy has landed before the CTA leaves (already true unless a wait gave up)
    for (int s = 0; s < kMkSlots; s++)
      if (last_chunk[s] != 0xffffffffu && !mbar_sleep_wait(&M.full[s], (last_chunk[s] / kMkSlots) & 1u)) err |= 1u << 9;
    __threadfence();
    const unsigned done = atomicAdd(a.ctr + 1, 1u);
    if (done == gridDim.x - 1) {  // the last CTA starts the next epoch (0 mod 2^22 is skipped: fresh buffers hold tag 0)
      unsigned e = a.ctr[0] + 1u;
      if ((e & 0x3fffffu) == 0u) e++;
      a.ctr[0] = e;
      a.ctr[1] = 0u;
      __threadfence();
    }
  }
  if (err && a.err) atomicOr(a.err, (int)err);
}

}  // namespace

size_t mk_smem_bytes() { return kMkSmemBytes; }

bool mk_init_attributes() {
  return cudaFuncSetAttribute(k_mk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMkSmemBytes) == cudaSuccess;
}

int mk_grid(int device) {
  static int cached[64] = {0};
  if (device < 0 || device >= 64) return 0;
  if (cached[device]) return cached[device];
  int sms = 0, occ = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k_mk, kMkThreads, kMkSmemBytes) != cudaSuccess) return 0;
  cached[device] = sms * (occ > 1 ? 1 : occ);
  return cached[device];
}

void mk_launch(const MkArgs &a, int grid, cudaStream_t st) {
  if (grid <= 0 || a.n <= 0 || a.n > kMkMaxStages) {
    note_launch(cudaErrorInvalidValue, "k_mk (grid / program size)");
    return;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kMkThreads);
  cfg.dynamicSmemBytes = kMkSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  note_launch(cudaLaunchKernelEx(&cfg, k_mk, a), "k_mk");
  g_launches++;
}

}  // namespace q3t

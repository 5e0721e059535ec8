// Device-side implementations of the talker / code-predictor ops.  Each op
// is a __device__ function over explicit work-item indices, so the same code
// runs in a standalone kernel (prefill, sessions) and inside the persistent
// frame kernel (one launch per decode frame).
#pragma once
#include <cfloat>

#include "common.cuh"
#include "lm_kernels.cuh"

namespace q3t {

// ---------------------------------------------------------------------------
// shared helpers
// ---------------------------------------------------------------------------
// Sum of the split partials at (t, n..n+3), in split order.  The loads of a
// batch of 8 splits are issued before any add, so a fold costs one memory
// latency per 8 splits rather than one per split.
Q3T_DEV float4 part4(const Part &P, int t, int n) {
  const float *p = P.p + (size_t)t * P.ld + n;
  float4 a = *reinterpret_cast<const float4 *>(p);
  for (int s = 1; s < P.splits; s += 8) {
    float4 b[8];
#pragma unroll
    for (int i = 0; i < 8; i++)
      b[i] = s + i < P.splits ? *reinterpret_cast<const float4 *>(p + (s + i) * P.stride)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int i = 0; i < 8; i++) {
      a.x += b[i].x;
      a.y += b[i].y;
      a.z += b[i].z;
      a.w += b[i].w;
    }
  }
  return a;
}

Q3T_DEV size_t page_elem(const KVView &kv, int seq, int pos, int h) {
  const int page = kv.page_table[(size_t)seq * kv.pt_stride + (pos >> 4)];
  return (((size_t)page * kv.n_kv + h) * 16 + (pos & 15)) * 128;
}

// q_norm / k_norm + rotate-half RoPE (attention.rs:49-69, 126-134): one warp
// per head, lane l holds dims [4l, 4l+4); the partner of dim d is d +- 64,
// i.e. lane l ^ 16.  gm / fr: this lane's gamma and inverse frequencies.
Q3T_DEV void norm_rope_reg(float4 v, float4 gm, float4 fr, float eps, int lane, int pos, float out[4]) {
  const float ss = warp_sum(v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w);
  const float rms = sqrtf(ss / 128.f + eps);
  const float e[4] = {v.x / rms * gm.x, v.y / rms * gm.y, v.z / rms * gm.z, v.w / rms * gm.w};
  const float f[4] = {fr.x, fr.y, fr.z, fr.w};
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const float p = __shfl_xor_sync(0xffffffffu, e[i], 16);
    const int d = lane * 4 + i;
    float s, c;
    sincosf((float)pos * f[i], &s, &c);
    out[i] = d < 64 ? e[i] * c - p * s : e[i] * c + p * s;
  }
}
// The same with gamma and the inverse frequencies read here: lane l uses
// gm[4l .. 4l + 3] and inv_freq[(4l .. 4l + 3) mod 64].
Q3T_DEV void norm_rope_lane(float4 v, const float *__restrict__ gm, float eps, int lane, int pos,
                            const float *__restrict__ inv_freq, float out[4]) {
  norm_rope_reg(v, *reinterpret_cast<const float4 *>(gm + lane * 4),
                *reinterpret_cast<const float4 *>(inv_freq + ((lane * 4) & 63)), eps, lane, pos, out);
}

// ---------------------------------------------------------------------------
// RMSNorm of residual row r = t*row_mul + row_add, optionally first building
// the row from embeddings (the decode-step inputs of infer/mod.rs):
//   src 1: rows 2b / 2b+1 = hidden[slot[b]] / emb0[codes[slot[b]][0]]
//          (code-predictor prefill, infer/mod.rs:475-485)
//   src 2: row t = emb[codes[slot[t]][col]]            (:507-511)
//   src 3: row t = sum_g emb_g[codes[slot[t]][g]] + extra[t] (:343-383),
//          recording the frame's codes into hist
// and folding pending split-K partials into the row.  Block-wide; any
// blockDim that divides H / 4.
// ---------------------------------------------------------------------------
Q3T_DEV void d_rmsnorm(const RmsArgs &a, int t, float *red) {
  if (t >= *a.ntok) return;
  const int r = a.row_idx ? a.row_idx[t] : t * a.row_mul + a.row_add;
  float *xr = a.x + (size_t)r * a.ldx;
  const int H = a.H;
  const EmbedArgs &e = a.emb;
  if (e.src != 0) {
    int s = 0;
    const uint16_t *row0 = nullptr;
    const float *frow = nullptr;
    const int64_t *c = nullptr;
    if (e.src == 1) {
      s = e.slot[t >> 1];
      if (t & 1)
        row0 = e.emb0 + (size_t)e.codes[(size_t)s * e.G] * H;
      else
        frow = e.hidden + (size_t)s * H;
    } else if (e.src == 2) {
      s = e.slot[t];
      row0 = e.emb + (size_t)e.codes[(size_t)s * e.G + e.col] * H;
    } else {
      s = e.slot[t];
      c = e.codes + (size_t)s * e.G;
      row0 = e.emb0 + (size_t)c[0] * H;
      frow = e.extra ? e.extra[t] : nullptr;
    }
    for (int i = threadIdx.x * 4; i < H; i += blockDim.x * 4) {
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (row0) {
        const uint2 u = *reinterpret_cast<const uint2 *>(row0 + i);
        v = make_float4(bf2f(u.x & 0xffffu), bf2f(u.x >> 16), bf2f(u.y & 0xffffu), bf2f(u.y >> 16));
      }
      if (e.src == 3) {
        for (int q = 1; q < e.G; q++) {
          const uint2 u = *reinterpret_cast<const uint2 *>(e.embs[q - 1] + (size_t)c[q] * H + i);
          v.x += bf2f(u.x & 0xffffu);
          v.y += bf2f(u.x >> 16);
          v.z += bf2f(u.y & 0xffffu);
          v.w += bf2f(u.y >> 16);
        }
      }
      if (frow) {
        const float4 f = *reinterpret_cast<const float4 *>(frow + i);
        if (e.src == 1) {
          v = f;
        } else {
          v.x += f.x;
          v.y += f.y;
          v.z += f.z;
          v.w += f.w;
        }
      }
      *reinterpret_cast<float4 *>(xr + i) = v;
    }
    if (e.src == 3 && e.hist && (int)threadIdx.x < e.G)
      e.hist[((size_t)s * e.hist_frames + e.frame[t]) * e.G + threadIdx.x] = c[threadIdx.x];
    __syncthreads();
  }
  float ss = 0.f;
  for (int i = threadIdx.x * 4; i < H; i += blockDim.x * 4) {
    float4 v = *reinterpret_cast<const float4 *>(xr + i);
    if (a.add.splits > 0) {
      const float4 p = part4(a.add, r, i);
      v.x += p.x;
      v.y += p.y;
      v.z += p.z;
      v.w += p.w;
      *reinterpret_cast<float4 *>(xr + i) = v;
    }
    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  ss = block_sum(ss, red);
  const float rms = sqrtf(ss / (float)H + a.eps);
  for (int i = threadIdx.x * 4; i < H; i += blockDim.x * 4) {
    const float4 v = *reinterpret_cast<const float4 *>(xr + i);
    const float4 gm = *reinterpret_cast<const float4 *>(a.gamma + i);
    const float4 y = make_float4(v.x / rms * gm.x, v.y / rms * gm.y, v.z / rms * gm.z, v.w / rms * gm.w);
    uint2 p;
    p.x = pack_bf16x2(y.x, y.y);
    p.y = pack_bf16x2(y.z, y.w);
    *reinterpret_cast<uint2 *>(a.out + (size_t)t * a.ldo + i) = p;
    if (a.out_f32) *reinterpret_cast<float4 *>(a.out_f32 + (size_t)a.slot[t] * H + i) = y;
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------
// Split-K flash-decoding GQA attention (attention.rs:88-123 with the f32
// softmax of nn/attention.rs:13-26) over the paged cache, as independent
// warp work units.  A unit is (token t, kv head g, a run of up to pw pages of
// t's keys [0, pos]); both query heads 2g, 2g+1 share every K/V page read.
// Units are numbered token-major (all heads and page runs of token 0, then
// token 1, ...) and handed to warps round-robin, so a launch is a few
// balanced waves whatever the mix of sequence lengths.  A token whose keys
// fit one unit writes its output directly; otherwise each unit writes an
// (o, m, l) partial and the last unit of (t, g) to finish merges them in unit
// order and resets the counter.  q (normed, rotated, bf16) and the token's
// own K/V come from the QKV projection's epilogue.
//
// Per 16-key page, q.k runs on the tensor cores as S^T = K * Q^T
// (m16n8k16: A = 16 keys x 16 dims, B = 16 dims x 8 columns of which
// columns 0/1 are the two heads).  The dims of each k-step are permuted so
// that every lane's A and B fragments are one 16-byte load: lane (g, t)
// holds dims [8(t + 4kp), +8) of keys g and g + 8 for kp < 4, which feed
// k-steps 2kp (dims +0..3) and 2kp+1 (dims +4..7); q uses the same map, so
// the dot products are unchanged.  Softmax and p.v stay in f32 on the CUDA
// cores (p is not rounded).
// ---------------------------------------------------------------------------
constexpr int kPart = 132;
constexpr int kAttnWarps = 4;

struct AttnSmem {
  float ps[kAttnWarps][2][16];
  float ob[kAttnWarps][2][128];
  int pre[kAttnMaxTok + 1];  // first unit of each token
};

// Per-warp ring of kAttnStages pages in shared memory, filled with cp.async.
// K and V rows are stored with their 16-byte chunks XOR-swizzled by
// (row & 7), so the K fragment loads (8 rows x 4 chunks) and the V ldmatrix
// loads (8 rows of one chunk) hit distinct banks.  Rows at or beyond the
// valid key count are zero-filled (the pool may hold stale or uninitialised
// values there).
constexpr int kAttnStages = 2;
constexpr int kPageElems = 16 * 128;
constexpr size_t kAttnDynSmem = (size_t)kAttnWarps * kAttnStages * 2 * kPageElems * 2;  // 64 KB

Q3T_DEV void issue_page(uint16_t *ks, uint16_t *vs, const uint16_t *kp, const uint16_t *vp, int nv, int lane) {
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const int idx = lane + 32 * j, row = idx >> 4, c = idx & 15, sw = ((c ^ (row & 7)) << 3);
    const int n = row < nv ? 16 : 0;
    cp_async16(ks + row * 128 + sw, kp + row * 128 + c * 8, n);
    cp_async16(vs + row * 128 + sw, vp + row * 128 + c * 8, n);
  }
}

// Running softmax state of one warp: m / l per head (l = this lane's share);
// c[dt] = the m16n8k16 accumulator of O^T dims [16dt, 16dt + 16) x columns
// (heads) 0..7: on lanes with (lane & 3) == 0, c0/c1 = dim 16dt + lane/4 of
// heads 0/1 and c2/c3 = dim 16dt + 8 + lane/4.
struct AttnAcc {
  float m[2], l[2], c[8][4];
};

// One staged page: ks / vs = the page's K / V in the warp's ring; nv valid keys.
Q3T_DEV void attn_page(AttnAcc &A, const uint16_t *ks, const uint16_t *vs, const uint4 *qf, int nv, float scale,
                       float (*ps)[16], int lane) {
  const int g = lane >> 2, t = lane & 3;
  // S^T = K Q^T on the tensor cores (two accumulators halve the dependent chain)
  float c[4] = {0.f, 0.f, 0.f, 0.f}, c2[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int q = 0; q < 4; q++) {
    const int ch = ((t + 4 * q) ^ g) << 3;  // rows g and g + 8 share the swizzle
    const uint4 k0 = *reinterpret_cast<const uint4 *>(ks + g * 128 + ch);
    const uint4 k1 = *reinterpret_cast<const uint4 *>(ks + (g + 8) * 128 + ch);
    mma_16816(c, k0.x, k1.x, k0.y, k1.y, qf[q].x, qf[q].y);
    mma_16816(c2, k0.z, k1.z, k0.w, k1.w, qf[q].z, qf[q].w);
  }
#pragma unroll
  for (int i = 0; i < 4; i++) c[i] += c2[i];
  // c0/c1 = key g, heads 0/1; c2/c3 = key g + 8 (valid on lanes t == 0)
  const bool ok0 = t == 0 && g < nv, ok1 = t == 0 && g + 8 < nv;
  const float s00 = ok0 ? c[0] * scale : -FLT_MAX, s01 = ok0 ? c[1] * scale : -FLT_MAX;
  const float s10 = ok1 ? c[2] * scale : -FLT_MAX, s11 = ok1 ? c[3] * scale : -FLT_MAX;
  float mx0 = fmaxf(s00, s10), mx1 = fmaxf(s01, s11);
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
  }
  mx0 = __shfl_sync(0xffffffffu, mx0, 0);
  mx1 = __shfl_sync(0xffffffffu, mx1, 0);
  const float mn0 = fmaxf(A.m[0], mx0), mn1 = fmaxf(A.m[1], mx1);
  const float cr0 = expf(A.m[0] - mn0), cr1 = expf(A.m[1] - mn1);
  A.m[0] = mn0;
  A.m[1] = mn1;
  const float p00 = ok0 ? expf(s00 - mn0) : 0.f, p01 = ok0 ? expf(s01 - mn1) : 0.f;
  const float p10 = ok1 ? expf(s10 - mn0) : 0.f, p11 = ok1 ? expf(s11 - mn1) : 0.f;
  A.l[0] = A.l[0] * cr0 + p00 + p10;
  A.l[1] = A.l[1] * cr1 + p01 + p11;
  if (t == 0) {
    ps[0][g] = p00;
    ps[0][g + 8] = p10;
    ps[1][g] = p01;
    ps[1][g + 8] = p11;
  }
#pragma unroll
  for (int dt = 0; dt < 8; dt++) {
    A.c[dt][0] *= cr0;
    A.c[dt][1] *= cr1;
    A.c[dt][2] *= cr0;
    A.c[dt][3] *= cr1;
  }
  __syncwarp();
  // O^T += V^T P^T: B = P^T (16 keys x heads), split p = hi + lo in bf16 so
  // the products keep ~16 mantissa bits of p
  uint32_t bh0 = 0u, bh1 = 0u, bl0 = 0u, bl1 = 0u;
  if (g < 2) {
    const float pv[4] = {ps[g][2 * t], ps[g][2 * t + 1], ps[g][2 * t + 8], ps[g][2 * t + 9]};
    float hi[4], lo[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
      hi[i] = bf16_round(pv[i]);
      lo[i] = pv[i] - hi[i];
    }
    bh0 = pack_bf16x2(hi[0], hi[1]);
    bh1 = pack_bf16x2(hi[2], hi[3]);
    bl0 = pack_bf16x2(lo[0], lo[1]);
    bl1 = pack_bf16x2(lo[2], lo[3]);
  }
  const int mi = lane >> 3, vr = (lane & 7) + ((mi >> 1) << 3);  // ldmatrix: matrix mi, key row vr
#pragma unroll
  for (int dt = 0; dt < 8; dt++) {
    const int ch = ((2 * dt + (mi & 1)) ^ (vr & 7)) << 3;
    uint32_t a0, a1, a2, a3;
    ldmatrix_x4_trans(a0, a1, a2, a3, vs + vr * 128 + ch);
    mma_16816(A.c[dt], a0, a1, a2, a3, bh0, bh1);
    mma_16816(A.c[dt], a0, a1, a2, a3, bl0, bl1);
  }
  __syncwarp();
}

// pages per unit for a sequence of `pages` pages (at most kAttnMaxUnits units)
Q3T_DEV int attn_unit_pages(int pages, int pw) {
  const int m = (pages + kAttnMaxUnits - 1) / kAttnMaxUnits;
  return pw > m ? pw : m;
}

Q3T_DEV void store_bf16x8(uint16_t *dst, const float *v, float inv) {
  uint4 u;
  u.x = pack_bf16x2(v[0] * inv, v[1] * inv);
  u.y = pack_bf16x2(v[2] * inv, v[3] * inv);
  u.z = pack_bf16x2(v[4] * inv, v[5] * inv);
  u.w = pack_bf16x2(v[6] * inv, v[7] * inv);
  *reinterpret_cast<uint4 *>(dst) = u;
}

// Unit r of token t, run by one warp (ps, ob, ring: the warp's shared buffers).
Q3T_DEV void attn_unit(const AttnArgs &a, int t, int r, float (*ps)[16], float (*ob)[128], uint16_t *ring,
                       int lane) {
  const KVView &kv = a.kv;
  const int pos = a.tv.pos[t] + a.tv.pos_add, L = pos + 1, seq = a.tv.seq[t];
  const int pages = (L + 15) >> 4, pw = attn_unit_pages(pages, a.pw), nu = (pages + pw - 1) / pw;
  const int g = r / nu, j = r - g * nu;
  const int p0 = j * pw, np = min(pw, pages - p0);
  const int nh = a.nh;
  uint16_t *kb = kv.k + a.layer * kv.layer_stride;
  uint16_t *vb = kv.v + a.layer * kv.layer_stride;
  const int *pt = kv.page_table + (size_t)seq * kv.pt_stride;
  const int my_page = lane < np ? pt[p0 + lane] : 0;
  const size_t head_off = (size_t)g * 16 * 128, page_elems = (size_t)kv.n_kv * 16 * 128;
  // pages 0 and 1 of the unit in flight before the q loads
#pragma unroll
  for (int i = 0; i < kAttnStages - 1; i++) {
    if (i < np) {
      const size_t off = (size_t)__shfl_sync(0xffffffffu, my_page, i) * page_elems + head_off;
      issue_page(ring + i * 2 * kPageElems, ring + (i * 2 + 1) * kPageElems, kb + off, vb + off,
                 L - (p0 + i) * 16, lane);
    }
    cp_async_commit();
  }
  // q fragments: lane (g, t) < 8 rows holds head g's dims [8(t + 4kp), +8)
  uint4 qf[4];
  {
    const int gq = lane >> 2, tq = lane & 3;
    const uint16_t *qrow = a.q + (size_t)t * nh * 128 + (2 * g + (gq & 1)) * 128;
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const uint4 v = *reinterpret_cast<const uint4 *>(qrow + 8 * (tq + 4 * q));
      qf[q] = gq < 2 ? v : make_uint4(0u, 0u, 0u, 0u);
    }
  }
  AttnAcc A;
  A.m[0] = A.m[1] = -FLT_MAX;
  A.l[0] = A.l[1] = 0.f;
#pragma unroll
  for (int dt = 0; dt < 8; dt++) A.c[dt][0] = A.c[dt][1] = A.c[dt][2] = A.c[dt][3] = 0.f;
  for (int i = 0; i < np; i++) {
    const int nx = i + kAttnStages - 1;  // page to start now, into the slot page i - 1 used
    if (nx < np) {
      const int sl = nx % kAttnStages;
      const size_t off = (size_t)__shfl_sync(0xffffffffu, my_page, nx) * page_elems + head_off;
      issue_page(ring + sl * 2 * kPageElems, ring + (sl * 2 + 1) * kPageElems, kb + off, vb + off,
                 L - (p0 + nx) * 16, lane);
    }
    cp_async_commit();
    cp_async_wait<kAttnStages - 1>();  // this lane's copies of page i have landed
    __syncwarp();                      // ... and every lane's
    const int sl = i % kAttnStages, key0 = (p0 + i) * 16;
    attn_page(A, ring + sl * 2 * kPageElems, ring + (sl * 2 + 1) * kPageElems, qf, min(16, L - key0), a.scale, ps,
              lane);
  }
  // O^T from the accumulators (lanes t == 0) through shared memory: lane
  // l < 16 then holds dims 8l..8l+7 of both heads in o[h][e]
  A.l[0] = warp_sum(A.l[0]);
  A.l[1] = warp_sum(A.l[1]);
  if ((lane & 3) == 0) {
    const int gg = lane >> 2;
#pragma unroll
    for (int dt = 0; dt < 8; dt++) {
      ob[0][16 * dt + gg] = A.c[dt][0];
      ob[1][16 * dt + gg] = A.c[dt][1];
      ob[0][16 * dt + 8 + gg] = A.c[dt][2];
      ob[1][16 * dt + 8 + gg] = A.c[dt][3];
    }
  }
  __syncwarp();
  float o[2][8];
#pragma unroll
  for (int h = 0; h < 2; h++)
#pragma unroll
    for (int e = 0; e < 8; e++) o[h][e] = ob[h][8 * (lane & 15) + e];
  __syncwarp();  // ob is rewritten by the warp's next unit
  uint16_t *out = a.out + (size_t)t * nh * 128 + 2 * g * 128;
  if (nu == 1) {
    if (lane < 16) {
      store_bf16x8(out + 8 * lane, o[0], 1.f / A.l[0]);
      store_bf16x8(out + 128 + 8 * lane, o[1], 1.f / A.l[1]);
    }
    return;
  }
  float *P0 = a.ws.part + ((size_t)t * kv.n_kv + g) * kAttnMaxUnits * 2 * kPart;
  float *P = P0 + (size_t)j * 2 * kPart;
  if (lane < 16) {
#pragma unroll
    for (int h = 0; h < 2; h++) {
      *reinterpret_cast<float4 *>(P + h * kPart + 8 * lane) = make_float4(o[h][0], o[h][1], o[h][2], o[h][3]);
      *reinterpret_cast<float4 *>(P + h * kPart + 8 * lane + 4) = make_float4(o[h][4], o[h][5], o[h][6], o[h][7]);
    }
  }
  if (lane == 0) {
    P[128] = A.m[0];
    P[129] = A.l[0];
    P[kPart + 128] = A.m[1];
    P[kPart + 129] = A.l[1];
  }
  __threadfence();
  __syncwarp();
  int last = 0;
  if (lane == 0) last = atomicAdd(&a.ws.counters[t * kv.n_kv + g], 1) == nu - 1;
  last = __shfl_sync(0xffffffffu, last, 0);
  if (!last) return;
  __threadfence();
  // merge the units in order: lane handles head lane >> 4, dims 8(lane & 15) + [0, 8)
  const int h = lane >> 4, d0 = 8 * (lane & 15);
  float M = -FLT_MAX, Ls = 0.f, acc[8];
#pragma unroll
  for (int e = 0; e < 8; e++) acc[e] = 0.f;
  for (int s0 = 0; s0 < nu; s0 += 4) {  // four partials' loads in flight at a time
    float ms[4], ls[4];
    float4 o0[4], o1[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
      if (s0 + i < nu) {
        const float *Ps = P0 + (size_t)(s0 + i) * 2 * kPart + h * kPart;
        ms[i] = __ldcg(Ps + 128);
        ls[i] = __ldcg(Ps + 129);
        o0[i] = __ldcg(reinterpret_cast<const float4 *>(Ps + d0));
        o1[i] = __ldcg(reinterpret_cast<const float4 *>(Ps + d0 + 4));
      }
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
      if (s0 + i < nu) {
        const float Mn = fmaxf(M, ms[i]), fa = expf(M - Mn), fb = expf(ms[i] - Mn);
        Ls = Ls * fa + ls[i] * fb;
        const float ov[8] = {o0[i].x, o0[i].y, o0[i].z, o0[i].w, o1[i].x, o1[i].y, o1[i].z, o1[i].w};
#pragma unroll
        for (int e = 0; e < 8; e++) acc[e] = acc[e] * fa + ov[e] * fb;
        M = Mn;
      }
    }
  }
  store_bf16x8(out + h * 128 + d0, acc, 1.f / Ls);
  if (lane == 0) a.ws.counters[t * kv.n_kv + g] = 0;
}

// A group of kAttnWarps warps (tid 0..127, `sync` its barrier): numbers the
// units of the launch (host-written metadata only, so this part may run
// before the dependency wait) ...
template <class Sync>
Q3T_DEV void d_attn_number(const AttnArgs &a, int tid, AttnSmem &S, Sync sync) {
  const int w = tid >> 5, lane = tid & 31;
  int ntok = *a.tv.ntok;
  ntok = ntok < kAttnMaxTok ? ntok : kAttnMaxTok;
  if (w == 0) {
    int carry = 0;
    for (int base = 0; base < ntok; base += 32) {
      const int t = base + lane;
      int n = 0;
      if (t < ntok) {
        const int pages = (a.tv.pos[t] + a.tv.pos_add + 16) >> 4;
        const int pw = attn_unit_pages(pages, a.pw);
        n = (pages + pw - 1) / pw * a.kv.n_kv;
      }
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, n, o);
        if (lane >= o) n += v;
      }
      if (t < ntok) S.pre[t + 1] = carry + n;
      carry += __shfl_sync(0xffffffffu, n, 31);
    }
    if (lane == 0) S.pre[0] = 0;
  }
  sync();
}

// ... then its warps take units warp0 + w, + nwarps, ...
template <class Sync>
Q3T_DEV void d_attn_run(const AttnArgs &a, int tid, int warp0, int nwarps, AttnSmem &S, uint16_t *ring, Sync sync) {
  const int w = tid >> 5, lane = tid & 31;
  int ntok = *a.tv.ntok;
  ntok = ntok < kAttnMaxTok ? ntok : kAttnMaxTok;
  const int total = S.pre[ntok];
  for (int u = warp0 + w; u < total; u += nwarps) {
    int lo = 0, hi = ntok;  // largest t with pre[t] <= u
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (S.pre[mid] <= u)
        lo = mid;
      else
        hi = mid;
    }
    attn_unit(a, lo, u - S.pre[lo], S.ps[w], S.ob[w], ring + (size_t)w * kAttnStages * 2 * kPageElems, lane);
  }
  sync();  // S is reused by the caller's next item
}

template <class Sync>
Q3T_DEV void d_attn(const AttnArgs &a, int tid, int warp0, int nwarps, AttnSmem &S, uint16_t *ring, Sync sync) {
  d_attn_number(a, tid, S, sync);
  d_attn_run(a, tid, warp0, nwarps, S, ring, sync);
}

// ---------------------------------------------------------------------------
// Sampling (sampling.rs:33-150) of token row t: reduce the logits partials,
// repetition penalty (gather the original logits, scatter-ADD so duplicates
// accumulate), suppress list, greedy argmax (first index on ties) or
// temperature / top-k / top-p / categorical; teacher forcing; history / EOS.
// Block-wide.  lg/sv/si: shared arrays of kSampleMaxV entries; rv/ri: 32.
// ---------------------------------------------------------------------------

Q3T_DEV uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

Q3T_DEV void bitonic_desc(float *v, int *ix, int n) {
  for (int k = 2; k <= n; k <<= 1)
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int l = i ^ j;
        if (l > i) {
          const bool up = (i & k) == 0;
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

Q3T_DEV void d_sample(const SampleArgs &a, int t, float *lg, float *sv, int *si, float *rv, int *ri) {
  if (t >= *a.ntok) return;
  const int s = a.slot[t];
  const SampleParams P = a.params[s * 2 + a.use_pred_params];
  const int V = a.V, tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  float *row = a.logits + (size_t)t * a.ldl;
  for (int i = tid; i < V; i += blockDim.x) {
    float v = 0.f;
    for (int sp = 0; sp < a.part.splits; sp++) v += a.part.p[sp * a.part.stride + (size_t)t * a.part.ld + i];
    lg[i] = v;
    row[i] = v;
  }
  __syncthreads();
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
    const int64_t *sl = a.suppress + (size_t)s * a.suppress_ld;
    const int ns = a.n_sup ? a.n_sup[s] : a.n_suppress;
    for (int i = tid; i < ns; i += blockDim.x) {
      const int64_t id = sl[i];
      if (id >= 0 && id < V) lg[id] = -INFINITY;
    }
    __syncthreads();
  }
  int tok = 0;
  if (a.kept && !P.do_sample) {
    for (int i = tid; i < V; i += blockDim.x) a.kept[(size_t)t * a.ldl + i] = isfinite(lg[i]) ? 1 : 0;
  }
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
      tok = bi == 0x7fffffff ? 0 : bi;  // a fully masked row: argmax returns index 0
    }
  } else {
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
    if (a.kept) {
      for (int i = tid; i < V; i += blockDim.x) a.kept[(size_t)t * a.ldl + i] = isfinite(lg[i]) ? 1 : 0;
    }
    if (tid == 0) {
      float mx = -INFINITY;
      for (int i = 0; i < V; i++) mx = fmaxf(mx, lg[i]);
      double sum = 0.0;
      for (int i = 0; i < V; i++) sum += expf(lg[i] - mx);
      const uint64_t step = (uint64_t)(a.step_seed + (a.seed_p ? *a.seed_p : 0));
      const uint64_t r = mix64(P.seed ^ mix64(step * 131ull + (uint64_t)a.col) ^ ((uint64_t)s << 40));
      const double u = a.u ? a.u[t] : (double)(r >> 11) * (1.0 / 9007199254740992.0);
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
      if (f < a.force_on[s] && f < a.max_frames) tok = (int)a.forced[((size_t)s * a.max_frames + f) * a.G + a.col];
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
  __syncthreads();
}

}  // namespace q3t

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
Q3T_DEV float4 part4(const Part &P, int t, int n) {
  float4 a = *reinterpret_cast<const float4 *>(P.p + (size_t)t * P.ld + n);
  for (int s = 1; s < P.splits; s++) {
    const float4 b = *reinterpret_cast<const float4 *>(P.p + s * P.stride + (size_t)t * P.ld + n);
    a.x += b.x;
    a.y += b.y;
    a.z += b.z;
    a.w += b.w;
  }
  return a;
}

Q3T_DEV size_t page_elem(const KVView &kv, int seq, int pos, int h) {
  const int page = kv.page_table[(size_t)seq * kv.pt_stride + (pos >> 4)];
  return (((size_t)page * kv.n_kv + h) * 16 + (pos & 15)) * 128;
}

// q_norm / k_norm + rotate-half RoPE (attention.rs:49-69, 126-134): one warp
// per head, lane l holds dims [4l, 4l+4); the partner of dim d is d +- 64,
// i.e. lane l ^ 16.
Q3T_DEV void norm_rope_lane(float4 v, const float *__restrict__ gm, float eps, int lane, int pos,
                            const float *__restrict__ inv_freq, float out[4]) {
  const float ss = warp_sum(v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w);
  const float rms = sqrtf(ss / 128.f + eps);
  float e[4] = {v.x / rms * gm[lane * 4 + 0], v.y / rms * gm[lane * 4 + 1], v.z / rms * gm[lane * 4 + 2],
                v.w / rms * gm[lane * 4 + 3]};
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const float p = __shfl_xor_sync(0xffffffffu, e[i], 16);
    const int d = lane * 4 + i;
    float s, c;
    sincosf((float)pos * inv_freq[d & 63], &s, &c);
    out[i] = d < 64 ? e[i] * c - p * s : e[i] * c + p * s;
  }
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
  const int r = t * a.row_mul + a.row_add;
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
// Skinny GEMM item on the tensor cores (m16n8k16): 8 warps = 8 row blocks
// (128 output rows) x one K chunk of 16*FR x up to 64 tokens.  Weights are
// fragment-packed (one 512-byte A fragment per 16x16 tile, rb-major); the
// X chunk is staged once in shared memory for the 8 warps; partial sums are
// written with plain stores to P[split][token][row].
// ---------------------------------------------------------------------------
constexpr int kLinWarps = 8;

Q3T_DEV void lin_item_coords(const LinArgs &a, int item, int &rg, int &ks, int &tc) {
  const int rgn = a.N / (16 * kLinWarps), ksn = a.K / (16 * a.fr);
  rg = item % rgn;
  ks = (item / rgn) % ksn;
  tc = item / (rgn * ksn);
}

template <int FR>
Q3T_DEV void d_linear_load(const LinArgs &a, int item, uint4 *frag) {
  int rg, ks, tc;
  lin_item_coords(a, item, rg, ks, tc);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rb = rg * kLinWarps + warp;
  const uint4 *wp = a.W + ((size_t)rb * (a.K >> 4) + ks * FR) * 32 + lane;
#pragma unroll
  for (int i = 0; i < FR; i++) frag[i] = ldg_stream(wp + i * 32);
}

template <int NT, int FR>
Q3T_DEV void d_linear_compute(const LinArgs &a, int item, const uint4 *frag, uint16_t *xs) {
  constexpr int kc = FR * 16, ldsx = kc + 8, c8n = kc >> 3;
  int rg, ks, tc;
  lin_item_coords(a, item, rg, ks, tc);
  const int tok_base = tc * 64, k0 = ks * kc;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int ntok = *a.ntok - tok_base;
  ntok = ntok < 0 ? 0 : (ntok > NT * 8 ? NT * 8 : ntok);
  for (int idx = threadIdx.x; idx < NT * 8 * c8n; idx += blockDim.x) {
    const int r = idx / c8n, c8 = (idx - r * c8n) * 8;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (r < ntok) v = *reinterpret_cast<const uint4 *>(a.X + (size_t)(tok_base + r) * a.ldx + k0 + c8);
    *reinterpret_cast<uint4 *>(xs + r * ldsx + c8) = v;
  }
  __syncthreads();
  float acc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; j++) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int i = 0; i < FR; i++) {
#pragma unroll
    for (int j = 0; j < NT; j++) {
      const uint16_t *xr = xs + (j * 8 + g) * ldsx + i * 16 + 2 * t;
      const uint32_t b0 = *reinterpret_cast<const uint32_t *>(xr);
      const uint32_t b1 = *reinterpret_cast<const uint32_t *>(xr + 8);
      mma_16816(acc[j], frag[i].x, frag[i].y, frag[i].z, frag[i].w, b0, b1);
    }
  }
  const int row = (rg * kLinWarps + warp) * 16 + g;
  float *Y = a.P + ks * a.pstride;
#pragma unroll
  for (int j = 0; j < NT; j++) {
    const int tk = j * 8 + 2 * t;
    if (tk < ntok) {
      float *y = Y + (size_t)(tok_base + tk) * a.ldy + row;
      y[0] = acc[j][0];
      y[8] = acc[j][2];
    }
    if (tk + 1 < ntok) {
      float *y = Y + (size_t)(tok_base + tk + 1) * a.ldy + row;
      y[0] = acc[j][1];
      y[8] = acc[j][3];
    }
  }
  __syncthreads();  // xs is reused by the next item
}

// ---------------------------------------------------------------------------
// q/k RMSNorm + RoPE + bf16 q out + K/V append for token t (non-fused path,
// used when a batch holds several tokens of one sequence).
// ---------------------------------------------------------------------------
Q3T_DEV void d_qkv_post(const QkvArgs &a, int t) {
  if (t >= *a.tv.ntok) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int pos = a.tv.pos[t] + a.tv.pos_add, seq = a.tv.seq[t];
  const int nh = a.nh, nkv = a.nkv;
  for (int w = warp; w < nh + 2 * nkv; w += nw) {
    if (w < nh + nkv) {
      const bool isq = w < nh;
      const int h = isq ? w : w - nh;
      const float4 v = part4(a.qkv, t, (isq ? h : nh + h) * 128 + lane * 4);
      float o[4];
      norm_rope_lane(v, isq ? a.q_norm : a.k_norm, a.eps, lane, pos, a.inv_freq, o);
      uint2 p;
      p.x = pack_bf16x2(o[0], o[1]);
      p.y = pack_bf16x2(o[2], o[3]);
      if (isq)
        *reinterpret_cast<uint2 *>(a.qout + (size_t)t * nh * 128 + h * 128 + lane * 4) = p;
      else
        *reinterpret_cast<uint2 *>(a.kv.k + a.layer * a.kv.layer_stride + page_elem(a.kv, seq, pos, h) + lane * 4) = p;
    } else {
      const int h = w - nh - nkv;
      const float4 v = part4(a.qkv, t, (nh + nkv + h) * 128 + lane * 4);
      uint2 p;
      p.x = pack_bf16x2(v.x, v.y);
      p.y = pack_bf16x2(v.z, v.w);
      *reinterpret_cast<uint2 *>(a.kv.v + a.layer * a.kv.layer_stride + page_elem(a.kv, seq, pos, h) + lane * 4) = p;
    }
  }
}

// ---------------------------------------------------------------------------
// Split-K flash-decoding GQA attention item (split sp, kv head g, token t)
// (attention.rs:88-123 with the f32 softmax of nn/attention.rs:13-26) on a
// group of exactly 128 threads (tid 0..127); `sync` is the group barrier.
// Both query heads 2g, 2g+1 share every K/V row read.  Splits of `chunk`
// keys write (o, m, l) partials; the last item of (t, g) to finish merges
// them and resets the counter.  fused: also does the q/k norm + RoPE and the
// K/V append of the new token (one token per sequence in the batch).
// ---------------------------------------------------------------------------
constexpr int kPart = 132;

struct AttnSmem {
  float qs[2][128];
  float sc[2][256];
  float red[2][4];
  float opart[2][2][128];
  int last;
};

template <class Sync>
Q3T_DEV void d_attn(const AttnArgs &a, int sp, int g, int t, int tid, AttnSmem &S, Sync sync) {
  const int w = tid >> 5, lane = tid & 31;
  if (t >= *a.tv.ntok) return;
  const KVView &kv = a.kv;
  const int pos = a.tv.pos[t] + a.tv.pos_add, L = pos + 1, seq = a.tv.seq[t];
  const int nsplit = (L + a.chunk - 1) / a.chunk;
  if (sp >= nsplit) return;
  const int j0 = sp * a.chunk;
  const int n = min(L - j0, a.chunk);
  const int nh = a.nh;
  uint16_t *kb = kv.k + a.layer * kv.layer_stride;
  uint16_t *vb = kv.v + a.layer * kv.layer_stride;
  if (a.fused) {
    if (w < 2) {
      const int h = 2 * g + w;
      const float4 v = part4(a.qkv, t, h * 128 + lane * 4);
      float o[4];
      norm_rope_lane(v, a.q_norm, a.eps, lane, pos, a.inv_freq, o);
#pragma unroll
      for (int i = 0; i < 4; i++) S.qs[w][lane * 4 + i] = bf16_round(o[i]);
    } else if (sp == nsplit - 1) {
      const size_t e = page_elem(kv, seq, pos, g) + lane * 4;
      if (w == 2) {
        const float4 v = part4(a.qkv, t, (nh + g) * 128 + lane * 4);
        float o[4];
        norm_rope_lane(v, a.k_norm, a.eps, lane, pos, a.inv_freq, o);
        uint2 p;
        p.x = pack_bf16x2(o[0], o[1]);
        p.y = pack_bf16x2(o[2], o[3]);
        *reinterpret_cast<uint2 *>(kb + e) = p;
      } else {
        const float4 v = part4(a.qkv, t, (nh + kv.n_kv + g) * 128 + lane * 4);
        uint2 p;
        p.x = pack_bf16x2(v.x, v.y);
        p.y = pack_bf16x2(v.z, v.w);
        *reinterpret_cast<uint2 *>(vb + e) = p;
      }
    }
  } else {
    for (int e = tid; e < 256; e += 128)
      S.qs[e >> 7][e & 127] = bf2f(a.qin[(size_t)t * nh * 128 + (2 * g + (e >> 7)) * 128 + (e & 127)]);
  }
  sync();
  for (int jj = tid; jj < n; jj += 128) {
    const uint4 *kr = reinterpret_cast<const uint4 *>(kb + page_elem(kv, seq, j0 + jj, g));
    float s0 = 0.f, s1 = 0.f;
#pragma unroll 4
    for (int c = 0; c < 16; c++) {
      const uint4 u = kr[c];
      const uint32_t wv[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const float k0v = bf2f(wv[e] & 0xffffu), k1v = bf2f(wv[e] >> 16);
        s0 += S.qs[0][c * 8 + 2 * e] * k0v + S.qs[0][c * 8 + 2 * e + 1] * k1v;
        s1 += S.qs[1][c * 8 + 2 * e] * k0v + S.qs[1][c * 8 + 2 * e + 1] * k1v;
      }
    }
    S.sc[0][jj] = s0 * a.scale;
    S.sc[1][jj] = s1 * a.scale;
  }
  sync();
  float m0 = -FLT_MAX, m1 = -FLT_MAX;
  for (int jj = tid; jj < n; jj += 128) {
    m0 = fmaxf(m0, S.sc[0][jj]);
    m1 = fmaxf(m1, S.sc[1][jj]);
  }
  m0 = warp_max(m0);
  m1 = warp_max(m1);
  if (lane == 0) {
    S.red[0][w] = m0;
    S.red[1][w] = m1;
  }
  sync();
  m0 = fmaxf(fmaxf(S.red[0][0], S.red[0][1]), fmaxf(S.red[0][2], S.red[0][3]));
  m1 = fmaxf(fmaxf(S.red[1][0], S.red[1][1]), fmaxf(S.red[1][2], S.red[1][3]));
  sync();
  float l0 = 0.f, l1 = 0.f;
  for (int jj = tid; jj < n; jj += 128) {
    const float p0 = expf(S.sc[0][jj] - m0), p1 = expf(S.sc[1][jj] - m1);
    S.sc[0][jj] = p0;
    S.sc[1][jj] = p1;
    l0 += p0;
    l1 += p1;
  }
  l0 = warp_sum(l0);
  l1 = warp_sum(l1);
  if (lane == 0) {
    S.red[0][w] = l0;
    S.red[1][w] = l1;
  }
  sync();
  l0 = S.red[0][0] + S.red[0][1] + S.red[0][2] + S.red[0][3];
  l1 = S.red[1][0] + S.red[1][1] + S.red[1][2] + S.red[1][3];
  {
    const int dp = tid & 63, kh = tid >> 6, d = dp * 2;
    float o00 = 0.f, o01 = 0.f, o10 = 0.f, o11 = 0.f;
    for (int jj = kh; jj < n; jj += 2) {
      const uint32_t vv = *reinterpret_cast<const uint32_t *>(vb + page_elem(kv, seq, j0 + jj, g) + d);
      const float v0 = bf2f(vv & 0xffffu), v1 = bf2f(vv >> 16);
      const float p0 = S.sc[0][jj], p1 = S.sc[1][jj];
      o00 += p0 * v0;
      o01 += p0 * v1;
      o10 += p1 * v0;
      o11 += p1 * v1;
    }
    S.opart[kh][0][d] = o00;
    S.opart[kh][0][d + 1] = o01;
    S.opart[kh][1][d] = o10;
    S.opart[kh][1][d + 1] = o11;
  }
  sync();
  const int out_ld = nh * 128;
  if (nsplit == 1) {
    for (int e = tid; e < 256; e += 128) {
      const int h = e >> 7, d = e & 127;
      const float o = S.opart[0][h][d] + S.opart[1][h][d];
      a.out[(size_t)t * out_ld + (2 * g + h) * 128 + d] = f2bf(o / (h ? l1 : l0));
    }
  } else {
    float *P = a.ws.part + (((size_t)t * kv.n_kv + g) * a.ws.max_split + sp) * 2 * kPart;
    for (int e = tid; e < 256; e += 128) {
      const int h = e >> 7, d = e & 127;
      P[h * kPart + d] = S.opart[0][h][d] + S.opart[1][h][d];
    }
    if (tid == 0) {
      P[128] = m0;
      P[129] = l0;
      P[kPart + 128] = m1;
      P[kPart + 129] = l1;
    }
    __threadfence();
    sync();
    if (tid == 0) {
      const int prev = atomicAdd(&a.ws.counters[t * kv.n_kv + g], 1);
      S.last = prev == nsplit - 1;
    }
    sync();
    if (S.last) {
      __threadfence();
      const float *P0 = a.ws.part + ((size_t)t * kv.n_kv + g) * a.ws.max_split * 2 * kPart;
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
        a.out[(size_t)t * out_ld + (2 * g + h) * 128 + d] = f2bf(acc / Ls);
      }
      if (tid == 0) a.ws.counters[t * kv.n_kv + g] = 0;
    }
    sync();
  }
}

// SwiGLU silu(gate) * up of the reduced gate|up partials, 4 columns per thread
Q3T_DEV void d_silu(const SiluArgs &a, int t, int i) {
  if (t >= *a.ntok || i >= a.I) return;
  const float4 g = part4(a.gu, t, i);
  const float4 u = part4(a.gu, t, a.I + i);
  uint2 p;
  p.x = pack_bf16x2(silu(g.x) * u.x, silu(g.y) * u.y);
  p.y = pack_bf16x2(silu(g.z) * u.z, silu(g.w) * u.w);
  *reinterpret_cast<uint2 *>(a.out + (size_t)t * a.I + i) = p;
}

// ---------------------------------------------------------------------------
// Sampling (sampling.rs:33-150) of token row t: reduce the logits partials,
// repetition penalty (gather the original logits, scatter-ADD so duplicates
// accumulate), suppress list, greedy argmax (first index on ties) or
// temperature / top-k / top-p / categorical; teacher forcing; history / EOS.
// Block-wide.  lg/sv/si: shared arrays of kSampleMaxV entries; rv/ri: 32.
// ---------------------------------------------------------------------------
constexpr int kSampleMaxV = 4096;

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
    if (tid == 0) {
      float mx = -INFINITY;
      for (int i = 0; i < V; i++) mx = fmaxf(mx, lg[i]);
      double sum = 0.0;
      for (int i = 0; i < V; i++) sum += expf(lg[i] - mx);
      const uint64_t step = (uint64_t)(a.step_seed + (a.seed_p ? *a.seed_p : 0));
      const uint64_t r = mix64(P.seed ^ mix64(step * 131ull + (uint64_t)a.col) ^ ((uint64_t)s << 40));
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

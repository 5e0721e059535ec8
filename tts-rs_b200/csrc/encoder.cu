// Speech-tokenizer encoder of the voice-clone path on the device
// (Qwen3TtsAudioCodecEncoder::encode_reference_prefix,
// tts_qwen3_tts/src/model/codec/network/encoder.rs:121-136, built as
// codec/config.rs:136-346 builds it): 24 kHz samples -> codes
// [n_valid][frames], for the reference-audio prefix of voice-clone prompts.
//
// One waveform per call, f32 throughout, in the reference's order of
// operations:
//   backbone      causal Conv1d (left pad = effective kernel - stride, right
//                 pad to a whole stride window, conv.rs:33-83), then per
//                 stage a residual unit x + conv_out(elu(conv_in(elu(x))))
//                 and ELU + strided downsampling conv; ELU + output conv
//                 (encoder.rs:138-175);
//   transformer   causal GQA layers on [T][H]: LayerNorm, q/k/v projections,
//                 adjacent-pair RoPE from position 0, masked softmax
//                 attention, o projection with LayerScale, LayerNorm, GELU
//                 MLP with LayerScale (encoder.rs:179-288);
//   downsample    stride-2 conv with edge padding (config.rs:155-166);
//   quantizers    semantic then acoustic residual VQ: input_proj (1x1 conv),
//                 per codebook the nearest centroid embed_sum /
//                 clamp_min(cluster_usage, 1e-6) (first index on ties) and
//                 the residual loses it (encoder.rs:290-368, codebook.rs:4-41).
// The kernels are plain CUDA-core loops over [channel][time] rows: the
// encoder runs once per reference clip, off the synthesis hot path, and a
// 2 s clip is a few GMAC.  Activations live in a stream-ordered workspace
// sized per call; weights are uploaded once at load.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.cuh"
#include "engine.h"

namespace q3t {
namespace {

struct EncConv {
  float *w = nullptr, *b = nullptr;
  int ci = 0, co = 0, k = 0, stride = 1;
};

struct EncLayerDev {
  float *ln1_w, *ln1_b, *ln2_w, *ln2_b;
  float *wq, *bq, *wk, *bk, *wv, *bv, *wo, *bo;
  float *attn_scale, *mlp_scale, *fc1, *fc2;
};

// conv.rs:44-64: left pad and right extra of a causal conv (dilation 1)
void conv_padding(int L, int k, int stride, int *left, int *extra) {
  const int eff = k;
  const int pt = eff > stride ? eff - stride : 0;
  const int padded = L + pt;
  const int missing = eff > padded ? eff - padded : 0;
  *left = pt;
  *extra = missing > 0 ? missing : (stride - (padded - eff) % stride) % stride;
}
int conv_len(const EncConv &c, int L) {
  int pl, ex;
  conv_padding(L, c.k, c.stride, &pl, &ex);
  return (L + pl + ex - c.k) / c.stride + 1;
}

// ---------------------------------------------------------------------------
// kernels
// ---------------------------------------------------------------------------
// y[o][t] = b[o] + sum_i sum_j w[o][i][j] * xpad[i][t * stride + j], where
// xpad is x [ci][L] padded on the left by pl (and on the right as needed)
// with zeros (mode 0) or its edge values (mode 1); sums in (i, j) order.
__global__ void k_enc_conv(const float *__restrict__ x, int ci, int L, const float *__restrict__ w,
                           const float *__restrict__ b, int k, int stride, int pl, int mode, int Lo,
                           float *__restrict__ y) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x, o = blockIdx.y;
  if (t >= Lo) return;
  float acc = b ? b[o] : 0.f;
  const float *wo = w + (size_t)o * ci * k;
  for (int i = 0; i < ci; i++) {
    const float *xi = x + (size_t)i * L;
    for (int j = 0; j < k; j++) {
      int s = t * stride + j - pl;
      float v;
      if (s >= 0 && s < L)
        v = xi[s];
      else if (mode == 1)
        v = xi[s < 0 ? 0 : L - 1];
      else
        v = 0.f;
      acc += wo[i * k + j] * v;
    }
  }
  y[(size_t)o * Lo + t] = acc;
}

// burn elu (alpha 1): x > 0 ? x : exp(x) - 1; in place, or out = elu(x)
__global__ void k_elu(const float *__restrict__ x, float *__restrict__ y, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float v = x[i];
    y[i] = v > 0.f ? v : expf(v) - 1.f;
  }
}

__global__ void k_add(float *__restrict__ x, const float *__restrict__ d, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    x[i] += d[i];
}

// y [C][R] = x [R][C] transposed
__global__ void k_transpose(const float *__restrict__ x, int R, int C, float *__restrict__ y) {
  __shared__ float tile[32][33];
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int r = r0 + i, c = c0 + threadIdx.x;
    if (r < R && c < C) tile[i][threadIdx.x] = x[(size_t)r * C + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = c0 + i, r = r0 + threadIdx.x;
    if (r < R && c < C) y[(size_t)c * R + r] = tile[threadIdx.x][i];
  }
}

// burn LayerNorm with bias (biased variance) of each row of x [T][H]
__global__ void k_layer_norm(const float *__restrict__ x, const float *__restrict__ w, const float *__restrict__ b,
                             int H, float eps, float *__restrict__ y) {
  __shared__ float red[33];
  const float *xr = x + (size_t)blockIdx.x * H;
  float *yr = y + (size_t)blockIdx.x * H;
  float s = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) s += xr[i];
  const float mean = block_sum(s, red) / (float)H;
  float v = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) v += (xr[i] - mean) * (xr[i] - mean);
  const float inv = 1.f / sqrtf(block_sum(v, red) / (float)H + eps);
  for (int i = threadIdx.x; i < H; i += blockDim.x) yr[i] = (xr[i] - mean) * inv * w[i] + b[i];
}

// y[s][n] = sum_k x[s][k] W[n][k] (+ bias[n]) for x [S][K], W [N][K]; with
// gelu the result goes through GELU (erf form); 32 x 32 output tiles
__global__ void k_linear(const float *__restrict__ x, const float *__restrict__ W, const float *__restrict__ bias,
                         int S, int K, int N, int gelu, float *__restrict__ y) {
  __shared__ float xs[32][33], ws[32][33];
  const int n = blockIdx.x * 32 + threadIdx.x, s = blockIdx.y * 32 + threadIdx.y;
  float acc = 0.f;
  for (int k0 = 0; k0 < K; k0 += 32) {
    const int xr = blockIdx.y * 32 + threadIdx.y, wr = blockIdx.x * 32 + threadIdx.y, kc = k0 + threadIdx.x;
    xs[threadIdx.y][threadIdx.x] = xr < S && kc < K ? x[(size_t)xr * K + kc] : 0.f;
    ws[threadIdx.y][threadIdx.x] = wr < N && kc < K ? W[(size_t)wr * K + kc] : 0.f;
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 32; kk++) acc += xs[threadIdx.y][kk] * ws[threadIdx.x][kk];
    __syncthreads();
  }
  if (s < S && n < N) {
    float v = acc + (bias ? bias[n] : 0.f);
    if (gelu) v = 0.5f * v * (1.f + erff(v * 0.70710678118654752f));
    y[(size_t)s * N + n] = v;
  }
}

// burn RotaryEncoding on adjacent pairs (theta_i = theta^(-2i/d)) from
// position 0, in place on x [T][nh][hd]
__global__ void k_rope_pairs(float *x, int T, int nh, int hd, float theta) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x, half = hd / 2;
  if (idx >= T * nh * half) return;
  const int i = idx % half, h = (idx / half) % nh, t = idx / (half * nh);
  const float th = 1.0f / expf((float)(2 * i) / (float)hd * logf(theta));
  const float f = (float)t * th, cs = cosf(f), sn = sinf(f);
  float *p = x + ((size_t)t * nh + h) * hd + 2 * i;
  const float x0 = p[0], x1 = p[1];
  p[0] = x0 * cs - x1 * sn;
  p[1] = x1 * cs + x0 * sn;
}

// causal softmax attention (nn/attention.rs:5-27 with the autoregressive
// mask): q [T][nh][hd], k / v [T][nkv][hd] (query head h reads kv head
// h / (nh / nkv)) -> out [T][nh][hd]; one block per (query, head)
__global__ void k_enc_attn(const float *__restrict__ q, const float *__restrict__ k, const float *__restrict__ v,
                           int T, int nh, int nkv, int hd, float scale, float *__restrict__ out) {
  extern __shared__ float sc[];  // [T]
  __shared__ float red[33];
  const int s = blockIdx.x, h = blockIdx.y, g = h / (nh / nkv);
  const float *qs = q + ((size_t)s * nh + h) * hd;
  for (int j = threadIdx.x; j <= s; j += blockDim.x) {
    const float *kj = k + ((size_t)j * nkv + g) * hd;
    float d = 0.f;
    for (int e = 0; e < hd; e++) d += qs[e] * kj[e];
    sc[j] = d * scale;
  }
  __syncthreads();
  float mx = -INFINITY;
  for (int j = threadIdx.x; j <= s; j += blockDim.x) mx = fmaxf(mx, sc[j]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = (int)(threadIdx.x & 31) < (int)((blockDim.x + 31) >> 5) ? red[threadIdx.x & 31] : -INFINITY;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.f;
  for (int j = threadIdx.x; j <= s; j += blockDim.x) {
    const float e = expf(sc[j] - mx);
    sc[j] = e;
    sum += e;
  }
  sum = block_sum(sum, red);
  __syncthreads();
  for (int e = threadIdx.x; e < hd; e += blockDim.x) {
    float o = 0.f;
    for (int j = 0; j <= s; j++) o += sc[j] / sum * v[((size_t)j * nkv + g) * hd + e];
    out[((size_t)s * nh + h) * hd + e] = o;
  }
}

// h[t][c] += o[t][c] * scale[c] (LayerScale residual)
__global__ void k_scale_add(float *__restrict__ h, const float *__restrict__ o, const float *__restrict__ scale,
                            int64_t n, int H) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    h[i] += o[i] * scale[i % H];
}

// r[d][t] = sum_c P[d][c] z[c][t] (the quantizer's input_proj, a 1x1 conv without bias)
__global__ void k_proj(const float *__restrict__ P, const float *__restrict__ z, int H, int T, int vq,
                       float *__restrict__ r) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x, d = blockIdx.y;
  if (t >= T) return;
  float s = 0.f;
  for (int c = 0; c < H; c++) s += P[(size_t)d * H + c] * z[(size_t)c * T + t];
  r[(size_t)d * T + t] = s;
}

// Residual VQ of frame t (one block per frame) over n codebooks of
// centroids cent[l] [cb][vq]: the nearest centroid by squared distance
// (summed over d in order; first index on ties), written to codes[l][t],
// and subtracted from the residual x [vq][T].
constexpr int kRvqThreads = 256;
__global__ void __launch_bounds__(kRvqThreads) k_rvq(float *__restrict__ x, int T, int vq, const float *const *cent,
                                                    int n, int cb, int64_t *__restrict__ codes) {
  extern __shared__ float xs[];  // [vq]
  __shared__ float bv[kRvqThreads / 32];
  __shared__ int bi[kRvqThreads / 32];
  __shared__ int best_s;
  const int t = blockIdx.x, lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (int d = threadIdx.x; d < vq; d += blockDim.x) xs[d] = x[(size_t)d * T + t];
  __syncthreads();
  for (int l = 0; l < n; l++) {
    const float *c = cent[l];
    float best = INFINITY;
    int bj = 0x7fffffff;
    for (int j = threadIdx.x; j < cb; j += blockDim.x) {
      const float *cj = c + (size_t)j * vq;
      float s = 0.f;
      for (int d = 0; d < vq; d++) {
        const float df = xs[d] - cj[d];
        s += df * df;
      }
      if (s < best) {  // j grows within a thread: the first index wins ties
        best = s;
        bj = j;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oj = __shfl_xor_sync(0xffffffffu, bj, o);
      if (ov < best || (ov == best && oj < bj)) {
        best = ov;
        bj = oj;
      }
    }
    if (lane == 0) {
      bv[w] = best;
      bi[w] = bj;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int k = 1; k < kRvqThreads / 32; k++)
        if (bv[k] < best || (bv[k] == best && bi[k] < bj)) {
          best = bv[k];
          bj = bi[k];
        }
      if (bj == 0x7fffffff) bj = 0;  // no finite distance: index 0, as an argmin over NaNs would
      best_s = bj;
      codes[(size_t)l * T + t] = bj;
    }
    __syncthreads();
    const float *cb_row = c + (size_t)best_s * vq;
    for (int d = threadIdx.x; d < vq; d += blockDim.x) xs[d] -= cb_row[d];
    __syncthreads();
  }
  for (int d = threadIdx.x; d < vq; d += blockDim.x) x[(size_t)d * T + t] = xs[d];
}

inline int blocks_for(int64_t n, int per) { return (int)std::min<int64_t>((n + per - 1) / per, 148 * 16); }

}  // namespace
}  // namespace q3t

using namespace q3t;

struct q3t_codec_encoder {
  int device = 0;
  q3t_codec_encoder_config cfg{};
  DevArena ar;
  cudaStream_t st = nullptr;
  EncConv in_conv, out_conv, downsample;
  std::vector<EncConv> res_in, res_out, down;
  std::vector<EncLayerDev> layers;
  float *proj[2] = {nullptr, nullptr};   // input_proj [vq][hidden] of the semantic / acoustic quantizer
  const float **cent_dev[2] = {nullptr, nullptr};  // device arrays of per-codebook centroid pointers
  int n_cb[2] = {0, 0};
};

namespace {

struct Named {
  std::unordered_map<std::string, const q3t_tensor *> by;
  const q3t_tensor *get(const std::string &n, std::initializer_list<int64_t> shape, bool required = true) const {
    auto it = by.find(n);
    if (it == by.end()) {
      if (required) FAIL(Q3T_INVALID_INPUT, "codec encoder: missing tensor %s", n.c_str());
      return nullptr;
    }
    const q3t_tensor *t = it->second;
    int64_t want = 1, have = 1;
    for (int64_t s : shape) want *= s;
    for (int d = 0; d < t->ndim; d++) have *= t->shape[d];
    if (want != have)
      FAIL(Q3T_INVALID_INPUT, "codec encoder: tensor %s has %lld elements, expected %lld", n.c_str(), (long long)have,
           (long long)want);
    if (t->dtype != Q3T_F32 && t->dtype != Q3T_BF16)
      FAIL(Q3T_INVALID_INPUT, "codec encoder: tensor %s has an unsupported dtype", n.c_str());
    return t;
  }
};

// host copy of a tensor as f32 (bf16 widened)
std::vector<float> host_f32(const q3t_tensor *t) {
  int64_t n = 1;
  for (int d = 0; d < t->ndim; d++) n *= t->shape[d];
  std::vector<float> v((size_t)n);
  if (t->dtype == Q3T_F32) {
    memcpy(v.data(), t->data, (size_t)n * 4);
  } else {
    const uint16_t *s = static_cast<const uint16_t *>(t->data);
    for (int64_t i = 0; i < n; i++) {
      const uint32_t u = (uint32_t)s[i] << 16;
      memcpy(&v[(size_t)i], &u, 4);
    }
  }
  return v;
}

float *upload(q3t_codec_encoder *e, const std::vector<float> &v) {
  float *d = e->ar.alloc<float>(v.size());
  CK(cudaMemcpy(d, v.data(), v.size() * 4, cudaMemcpyHostToDevice));
  return d;
}
float *upload(q3t_codec_encoder *e, const q3t_tensor *t) { return t ? upload(e, host_f32(t)) : nullptr; }

EncConv load_conv(q3t_codec_encoder *e, const Named &T, const std::string &name, int ci, int co, int k, int stride,
                  bool bias) {
  EncConv c;
  c.ci = ci;
  c.co = co;
  c.k = k;
  c.stride = stride;
  c.w = upload(e, T.get(name + ".weight", {co, ci, k}));
  if (bias) c.b = upload(e, T.get(name + ".bias", {co}));
  return c;
}

// the encoder's conv: x [ci][L] -> y [co][Lo]
int run_conv(const EncConv &c, const float *x, int L, int mode, float *y, cudaStream_t st) {
  int pl, ex;
  conv_padding(L, c.k, c.stride, &pl, &ex);
  const int Lo = (L + pl + ex - c.k) / c.stride + 1;
  k_enc_conv<<<dim3((Lo + 255) / 256, c.co), 256, 0, st>>>(x, c.ci, L, c.w, c.b, c.k, c.stride, pl, mode, Lo, y);
  note_launch(cudaGetLastError(), "k_enc_conv");
  g_launches++;
  return Lo;
}

void run_linear(const float *x, const float *W, const float *b, int S, int K, int N, int gelu, float *y,
                cudaStream_t st) {
  k_linear<<<dim3((N + 31) / 32, (S + 31) / 32), dim3(32, 32), 0, st>>>(x, W, b, S, K, N, gelu, y);
  note_launch(cudaGetLastError(), "k_linear");
  g_launches++;
}

void check_launch_errors() {
  const char *k = "";
  cudaError_t e = take_launch_error(&k);
  if (e != cudaSuccess) throw CudaFail{e, k};
}

// frames of the encoder for n samples (the backbone, then the stride-2 downsample)
int encoder_frames(const q3t_codec_encoder *e, int64_t n) {
  int L = conv_len(e->in_conv, (int)n);
  for (size_t s = 0; s < e->down.size(); s++) L = conv_len(e->down[s], L);
  L = conv_len(e->out_conv, L);
  return conv_len(e->downsample, L);
}

// backbone + transformer + downsample on the device; returns the hidden
// [hidden][T] in workspace memory (freed by the caller on the stream)
float *encoder_hidden(q3t_codec_encoder *e, const float *wave, int64_t n, int *T_out) {
  const auto &c = e->cfg;
  cudaStream_t st = e->st;
  std::vector<void *> ws;
  auto wsalloc = [&](size_t floats) {
    void *p = nullptr;
    CK(cudaMallocAsync(&p, (floats ? floats : 1) * 4, st));
    ws.push_back(p);
    return static_cast<float *>(p);
  };
  auto wsfree = [&](void *p) {
    for (auto &q : ws)
      if (q == p) {
        CK(cudaFreeAsync(q, st));
        q = nullptr;
      }
  };
  int L = (int)n, C = c.audio_channels;
  // the largest activation: any conv output or input of the backbone
  float *x = wsalloc((size_t)n * C);
  CK(cudaMemcpyAsync(x, wave, (size_t)n * C * 4, cudaMemcpyHostToDevice, st));
  auto conv_to_new = [&](const EncConv &cv, float *in, int Lin, int mode, int *Lout) {
    const int Lo = conv_len(cv, Lin);
    float *y = wsalloc((size_t)cv.co * Lo);
    run_conv(cv, in, Lin, mode, y, st);
    *Lout = Lo;
    return y;
  };
  auto elu = [&](const float *in, float *out, int64_t cnt) {
    k_elu<<<blocks_for(cnt, 256), 256, 0, st>>>(in, out, cnt);
    note_launch(cudaGetLastError(), "k_elu");
    g_launches++;
  };
  {
    int Lo;
    float *y = conv_to_new(e->in_conv, x, L, 0, &Lo);
    wsfree(x);
    x = y;
    L = Lo;
    C = e->in_conv.co;
  }
  for (size_t s = 0; s < e->down.size(); s++) {
    // resnet: x + conv_out(elu(conv_in(elu(x))))
    const int64_t cnt = (int64_t)C * L;
    float *h = wsalloc((size_t)cnt);
    elu(x, h, cnt);
    int Lm;
    float *m = conv_to_new(e->res_in[s], h, L, 0, &Lm);
    elu(m, m, (int64_t)e->res_in[s].co * Lm);
    run_conv(e->res_out[s], m, Lm, 0, h, st);
    k_add<<<blocks_for(cnt, 256), 256, 0, st>>>(x, h, cnt);
    note_launch(cudaGetLastError(), "k_add");
    g_launches++;
    wsfree(m);
    wsfree(h);
    elu(x, x, cnt);
    int Lo;
    float *y = conv_to_new(e->down[s], x, L, 0, &Lo);
    wsfree(x);
    x = y;
    L = Lo;
    C = e->down[s].co;
  }
  elu(x, x, (int64_t)C * L);
  {
    int Lo;
    float *y = conv_to_new(e->out_conv, x, L, 0, &Lo);
    wsfree(x);
    x = y;
    L = Lo;
    C = e->out_conv.co;
  }
  // transformer on [T][H]
  const int H = c.hidden_size, T = L, nh = c.num_attention_heads, nkv = c.num_key_value_heads, hd = c.head_dim;
  const int qd = nh * hd, kd = nkv * hd, I = c.intermediate_size;
  float *h = wsalloc((size_t)T * H), *nrm = wsalloc((size_t)T * H), *q = wsalloc((size_t)T * qd);
  float *k = wsalloc((size_t)T * kd), *v = wsalloc((size_t)T * kd), *ao = wsalloc((size_t)T * qd);
  float *o = wsalloc((size_t)T * H), *f = wsalloc((size_t)T * I);
  k_transpose<<<dim3((T + 31) / 32, (H + 31) / 32), dim3(32, 8), 0, st>>>(x, H, T, h);
  note_launch(cudaGetLastError(), "k_transpose");
  g_launches++;
  for (const EncLayerDev &Ly : e->layers) {
    k_layer_norm<<<T, 256, 0, st>>>(h, Ly.ln1_w, Ly.ln1_b, H, c.norm_eps, nrm);
    run_linear(nrm, Ly.wq, Ly.bq, T, H, qd, 0, q, st);
    run_linear(nrm, Ly.wk, Ly.bk, T, H, kd, 0, k, st);
    run_linear(nrm, Ly.wv, Ly.bv, T, H, kd, 0, v, st);
    k_rope_pairs<<<(T * nh * (hd / 2) + 255) / 256, 256, 0, st>>>(q, T, nh, hd, c.rope_theta);
    k_rope_pairs<<<(T * nkv * (hd / 2) + 255) / 256, 256, 0, st>>>(k, T, nkv, hd, c.rope_theta);
    k_enc_attn<<<dim3(T, nh), 128, (size_t)T * 4, st>>>(q, k, v, T, nh, nkv, hd, 1.0f / sqrtf((float)hd), ao);
    run_linear(ao, Ly.wo, Ly.bo, T, qd, H, 0, o, st);
    k_scale_add<<<blocks_for((int64_t)T * H, 256), 256, 0, st>>>(h, o, Ly.attn_scale, (int64_t)T * H, H);
    k_layer_norm<<<T, 256, 0, st>>>(h, Ly.ln2_w, Ly.ln2_b, H, c.norm_eps, nrm);
    run_linear(nrm, Ly.fc1, nullptr, T, H, I, 1, f, st);
    run_linear(f, Ly.fc2, nullptr, T, I, H, 0, o, st);
    k_scale_add<<<blocks_for((int64_t)T * H, 256), 256, 0, st>>>(h, o, Ly.mlp_scale, (int64_t)T * H, H);
    note_launch(cudaGetLastError(), "encoder transformer layer");
    g_launches += 12;
  }
  k_transpose<<<dim3((H + 31) / 32, (T + 31) / 32), dim3(32, 8), 0, st>>>(h, T, H, x);
  note_launch(cudaGetLastError(), "k_transpose");
  g_launches++;
  for (float *p : {h, nrm, q, k, v, ao, o, f}) wsfree(p);
  // downsample: stride 2, edge padding
  int To;
  float *z = conv_to_new(e->downsample, x, L, 1, &To);
  wsfree(x);
  for (void *p : ws)
    if (p && p != z) CK(cudaFreeAsync(p, st));
  check_launch_errors();
  *T_out = To;
  return z;
}

}  // namespace

extern "C" q3t_status q3t_codec_encoder_load(const q3t_codec_encoder_desc *d, q3t_codec_encoder **out) {
  if (!d || !out || (d->num_tensors > 0 && !d->tensors)) {
    set_error("q3t_codec_encoder_load: null argument");
    return Q3T_INVALID_INPUT;
  }
  *out = nullptr;
  auto *e = new q3t_codec_encoder();
  try {
    const q3t_codec_encoder_config &c = d->config;
    if (c.audio_channels < 1 || c.num_filters < 1 || c.compress < 1 || c.num_ratios < 1 || c.num_ratios > 8 ||
        c.hidden_size < 1 || c.num_attention_heads < 1 || c.num_key_value_heads < 1 ||
        c.num_attention_heads % c.num_key_value_heads || c.head_dim < 2 || c.head_dim % 2 ||
        c.codebook_size < 1 || c.codebook_dim < 1 || c.num_quantizers < c.num_semantic_quantizers ||
        c.num_semantic_quantizers < 0 || c.downsample_factor < 1)
      FAIL(Q3T_INVALID_INPUT, "codec encoder: invalid config");
    e->cfg = c;
    e->device = d->device;
    CK(cudaSetDevice(d->device));
    CK(cudaStreamCreateWithFlags(&e->st, cudaStreamNonBlocking));
    Named T;
    for (int i = 0; i < d->num_tensors; i++) T.by[d->tensors[i].name] = &d->tensors[i];
    const std::string p = "encoder.encoder.layers";
    e->in_conv = load_conv(e, T, p + ".0.conv", c.audio_channels, c.num_filters, c.kernel_size, 1, true);
    int li = 1, scale = 1;
    for (int s = c.num_ratios - 1; s >= 0; s--) {
      const int Cc = scale * c.num_filters, r = c.ratios[s];
      e->res_in.push_back(load_conv(e, T, p + "." + std::to_string(li) + ".conv_in.conv", Cc, Cc / c.compress,
                                    c.residual_kernel_size, 1, true));
      e->res_out.push_back(
          load_conv(e, T, p + "." + std::to_string(li) + ".conv_out.conv", Cc / c.compress, Cc, 1, 1, true));
      e->down.push_back(load_conv(e, T, p + "." + std::to_string(li + 2) + ".conv", Cc, 2 * Cc, 2 * r, r, true));
      li += 3;
      scale *= 2;
    }
    e->out_conv = load_conv(e, T, p + "." + std::to_string(li + 1) + ".conv", scale * c.num_filters, c.hidden_size,
                            c.last_kernel_size, 1, true);
    const int H = c.hidden_size, qd = c.num_attention_heads * c.head_dim, kd = c.num_key_value_heads * c.head_dim;
    for (int l = 0; l < c.num_hidden_layers; l++) {
      const std::string q = "encoder.encoder_transformer.layers." + std::to_string(l) + ".";
      EncLayerDev L;
      L.ln1_w = upload(e, T.get(q + "input_layernorm.weight", {H}));
      L.ln1_b = upload(e, T.get(q + "input_layernorm.bias", {H}));
      L.ln2_w = upload(e, T.get(q + "post_attention_layernorm.weight", {H}));
      L.ln2_b = upload(e, T.get(q + "post_attention_layernorm.bias", {H}));
      L.wq = upload(e, T.get(q + "self_attn.q_proj.weight", {qd, H}));
      L.bq = upload(e, T.get(q + "self_attn.q_proj.bias", {qd}, false));
      L.wk = upload(e, T.get(q + "self_attn.k_proj.weight", {kd, H}));
      L.bk = upload(e, T.get(q + "self_attn.k_proj.bias", {kd}, false));
      L.wv = upload(e, T.get(q + "self_attn.v_proj.weight", {kd, H}));
      L.bv = upload(e, T.get(q + "self_attn.v_proj.bias", {kd}, false));
      L.wo = upload(e, T.get(q + "self_attn.o_proj.weight", {H, qd}));
      L.bo = upload(e, T.get(q + "self_attn.o_proj.bias", {H}, false));
      L.attn_scale = upload(e, T.get(q + "self_attn_layer_scale.scale", {H}));
      L.mlp_scale = upload(e, T.get(q + "mlp_layer_scale.scale", {H}));
      L.fc1 = upload(e, T.get(q + "mlp.fc1.weight", {c.intermediate_size, H}));
      L.fc2 = upload(e, T.get(q + "mlp.fc2.weight", {H, c.intermediate_size}));
      e->layers.push_back(L);
    }
    e->downsample = load_conv(e, T, "encoder.downsample.conv", H, H, 2 * c.downsample_factor, 2, false);
    const int vq = c.codebook_dim, cb = c.codebook_size;
    const int ng[2] = {c.num_semantic_quantizers, c.num_quantizers - c.num_semantic_quantizers};
    const char *grp[2] = {"semantic", "acoustic"};
    for (int g = 0; g < 2; g++) {
      e->n_cb[g] = ng[g];
      if (ng[g] <= 0) continue;
      const std::string q = std::string("encoder.quantizer.") + grp[g] + "_residual_vector_quantizer.";
      e->proj[g] = upload(e, T.get(q + "input_proj.weight", {vq, H, 1}));
      std::vector<const float *> ptrs;
      for (int j = 0; j < ng[g]; j++) {
        const std::string b = q + "layers." + std::to_string(j) + ".codebook.";
        const std::vector<float> es = host_f32(T.get(b + "embed_sum", {cb, vq}));
        const std::vector<float> us = host_f32(T.get(b + "cluster_usage", {cb}));
        std::vector<float> cent((size_t)cb * vq);
        for (int r = 0; r < cb; r++) {  // codebook.rs:4-41: embed_sum / clamp_min(cluster_usage, 1e-6)
          const float u = us[(size_t)r] < 1e-6f ? 1e-6f : us[(size_t)r];
          for (int dd = 0; dd < vq; dd++) cent[(size_t)r * vq + dd] = es[(size_t)r * vq + dd] / u;
        }
        ptrs.push_back(upload(e, cent));
      }
      e->cent_dev[g] = e->ar.alloc<const float *>(ptrs.size());
      CK(cudaMemcpy(e->cent_dev[g], ptrs.data(), ptrs.size() * sizeof(float *), cudaMemcpyHostToDevice));
    }
  } catch (const Status &s) {
    q3t_codec_encoder_free(e);
    return s.code;
  } catch (const CudaFail &cf) {
    set_error("CUDA error %s (%s) in %s", cudaGetErrorName(cf.err), cudaGetErrorString(cf.err), cf.what.c_str());
    q3t_codec_encoder_free(e);
    return Q3T_CUDA_ERROR;
  }
  *out = e;
  return Q3T_OK;
}

void q3t_codec_encoder_free(q3t_codec_encoder *e) {
  if (!e) return;
  cudaSetDevice(e->device);
  if (e->st) {
    cudaStreamSynchronize(e->st);
    cudaStreamDestroy(e->st);
  }
  e->ar.release();
  delete e;
}

template <class F>
static q3t_status enc_guard(F &&f) {
  try {
    f();
    return Q3T_OK;
  } catch (const Status &s) {
    return s.code;
  } catch (const CudaFail &c) {
    set_error("CUDA error %s (%s) in %s", cudaGetErrorName(c.err), cudaGetErrorString(c.err), c.what.c_str());
    return Q3T_CUDA_ERROR;
  } catch (const std::bad_alloc &) {
    set_error("host allocation failed");
    return Q3T_CUDA_ERROR;
  }
}

extern "C" q3t_status q3t_codec_encoder_frames(const q3t_codec_encoder *e, int64_t num_samples, int *frames) {
  if (!e || !frames || num_samples <= 0) {
    set_error("q3t_codec_encoder_frames: null argument or no samples");
    return Q3T_INVALID_INPUT;
  }
  *frames = encoder_frames(e, num_samples);
  return Q3T_OK;
}

extern "C" q3t_status q3t_codec_encoder_hidden(q3t_codec_encoder *e, const float *wave, int64_t num_samples,
                                               float *hidden, int max_frames, int *frames) {
  if (!e || !wave || !hidden || num_samples <= 0 || num_samples > (int64_t)1 << 30) {
    set_error("q3t_codec_encoder_hidden: null argument or sample count outside 1..2^30");
    return Q3T_INVALID_INPUT;
  }
  return enc_guard([&] {
    CK(cudaSetDevice(e->device));
    const int want = encoder_frames(e, num_samples);
    if (want > max_frames) FAIL(Q3T_INVALID_INPUT, "encoder frames %d exceed max_frames %d", want, max_frames);
    int T = 0;
    float *z = encoder_hidden(e, wave, num_samples, &T);
    CK(cudaMemcpyAsync(hidden, z, (size_t)e->cfg.hidden_size * T * 4, cudaMemcpyDeviceToHost, e->st));
    CK(cudaFreeAsync(z, e->st));
    CK(cudaStreamSynchronize(e->st));
    if (frames) *frames = T;
  });
}

extern "C" q3t_status q3t_codec_encode(q3t_codec_encoder *e, const float *wave, int64_t num_samples, int n_valid,
                                       int64_t *codes, int max_frames, int *frames) {
  if (!e || !wave || !codes || num_samples <= 0 || num_samples > (int64_t)1 << 30) {
    set_error("q3t_codec_encode: null argument or sample count outside 1..2^30");
    return Q3T_INVALID_INPUT;
  }
  if (n_valid < e->cfg.num_semantic_quantizers || n_valid < 1 || n_valid > e->cfg.num_quantizers) {
    set_error("q3t_codec_encode: n_valid %d outside %d..%d", n_valid, std::max(1, e->cfg.num_semantic_quantizers),
              e->cfg.num_quantizers);
    return Q3T_INVALID_INPUT;
  }
  return enc_guard([&] {
    CK(cudaSetDevice(e->device));
    const int want = encoder_frames(e, num_samples);
    if (want > max_frames) FAIL(Q3T_INVALID_INPUT, "encoder frames %d exceed max_frames %d", want, max_frames);
    cudaStream_t st = e->st;
    int T = 0;
    float *z = encoder_hidden(e, wave, num_samples, &T);
    const int H = e->cfg.hidden_size, vq = e->cfg.codebook_dim, cb = e->cfg.codebook_size;
    int64_t *dcodes = nullptr;
    float *r = nullptr;
    CK(cudaMallocAsync((void **)&dcodes, (size_t)n_valid * T * 8, st));
    CK(cudaMallocAsync((void **)&r, (size_t)vq * T * 4, st));
    // semantic codes first, then acoustic (encoder.rs:290-317)
    const int want_g[2] = {e->n_cb[0], std::min(n_valid - e->n_cb[0], e->n_cb[1])};
    int row = 0;
    for (int g = 0; g < 2; g++) {
      if (want_g[g] <= 0) continue;
      k_proj<<<dim3((T + 127) / 128, vq), 128, 0, st>>>(e->proj[g], z, H, T, vq, r);
      k_rvq<<<T, kRvqThreads, (size_t)vq * 4, st>>>(r, T, vq, e->cent_dev[g], want_g[g], cb,
                                                    dcodes + (size_t)row * T);
      note_launch(cudaGetLastError(), "k_proj / k_rvq");
      g_launches += 2;
      row += want_g[g];
    }
    check_launch_errors();
    CK(cudaMemcpyAsync(codes, dcodes, (size_t)row * T * 8, cudaMemcpyDeviceToHost, st));
    CK(cudaFreeAsync(dcodes, st));
    CK(cudaFreeAsync(r, st));
    CK(cudaFreeAsync(z, st));
    CK(cudaStreamSynchronize(st));
    if (frames) *frames = T;
  });
}

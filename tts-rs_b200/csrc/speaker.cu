// ECAPA-TDNN speaker encoder of the voice-clone path on the device
// (LoadedQwen3TtsSpeakerEncoder::encode_embedding, tts_qwen3_tts/src/model/
// speaker/infer/mod.rs:11-20): 24 kHz samples -> x-vector [enc_dim].
//
//   log-mel       reflect-padded frames of 1024 samples every 256
//                 (feature.rs:92-115), periodic Hann window, magnitude of
//                 the 1024-point DFT (f64 sums, |X| + 1e-9 under the square
//                 root), area-normalised mel filters from 0 to sr / 2, log
//                 clamped at 1e-5 (feature.rs:32-194);
//   TDNN blocks   reflect padding (half the receptive field on the left),
//                 dilated conv with bias, ReLU (tdnn.rs:16-82);
//   SE-Res2Net    tdnn1, the Res2Net chain over channel groups (y1 = B1(c1),
//                 y_i = B_i(c_i + y_{i-1})), tdnn2, squeeze-excitation
//                 (mean over time, relu, sigmoid gate) on the residual
//                 (res2net.rs:37-119), three blocks;
//   aggregation   the three block outputs concatenated through the MFA
//                 TDNN, attentive statistics pooling (pooling.rs:25-72) and
//                 the final 1x1 conv (network/mod.rs:59-92).
// Plain f32 CUDA-core kernels over [channel][frame] rows, in the reference's
// order of operations: the encoder runs once per reference clip.
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

constexpr int kNfft = 1024, kHop = 256, kPad = (kNfft - kHop) / 2, kBins = kNfft / 2 + 1;

struct Tdnn {
  float *w = nullptr, *b = nullptr;
  int ci = 0, co = 0, k = 1, dil = 1;
};

// One mel frame per block: window, DFT magnitudes (f64 sums over a cos / sin
// table of the 1024 roots), filters, log.  p = the reflect-padded samples.
__global__ void __launch_bounds__(256) k_spk_mel(const float *__restrict__ p, const float *__restrict__ win,
                                                 const double *__restrict__ cs, const double *__restrict__ sn,
                                                 const float *__restrict__ fb, int n_mels, int frames,
                                                 float *__restrict__ out) {
  __shared__ double xw[kNfft];
  __shared__ float mag[kBins];
  const int t = blockIdx.x;
  for (int i = threadIdx.x; i < kNfft; i += blockDim.x) xw[i] = (double)(p[(size_t)t * kHop + i] * win[i]);
  __syncthreads();
  for (int f = threadIdx.x; f < kBins; f += blockDim.x) {
    double re = 0.0, im = 0.0;
    for (int i = 0; i < kNfft; i++) {
      const int r = (f * i) & (kNfft - 1);
      re += xw[i] * cs[r];
      im -= xw[i] * sn[r];
    }
    const float a = (float)re, b = (float)im;
    mag[f] = sqrtf(a * a + b * b + 1e-9f);
  }
  __syncthreads();
  for (int m = threadIdx.x; m < n_mels; m += blockDim.x) {
    float s = 0.f;
    for (int f = 0; f < kBins; f++) s += fb[(size_t)m * kBins + f] * mag[f];
    out[(size_t)m * frames + t] = logf(s > 1e-5f ? s : 1e-5f);
  }
}

constexpr int kTdT = 64, kTdC = 64, kTdK = 8, kTdWs = kTdC + 4;

// Dynamic shared memory of one k_tdnn CTA for a kernel of k taps spanning
// total = dil (k - 1) frames.
inline size_t tdnn_smem(int k, int total) { return sizeof(float) * ((size_t)kTdK * (kTdT + total) + (size_t)kTdK * k * kTdWs); }

// y[o][t] = relu(b[o] + sum_i sum_j w[o][i][j] * xr[i][t + j dil]) with xr the
// reflect padding of x [ci][T] by pl on the left (x[pl], ..., x[1]) and the
// rest on the right (x[T - 2], ...).  A CTA owns 64 channels x 64 frames
// (4 x 4 a thread); input rows of 8 channels with their halo and the
// matching weights are staged in shared memory; every output sums its terms
// in (i, j) order from the bias.
__global__ void __launch_bounds__(256) k_tdnn(const float *__restrict__ x, int ci, int T, const float *__restrict__ w,
                                              const float *__restrict__ b, int co, int k, int dil, int pl,
                                              float *__restrict__ y) {
  extern __shared__ float4 sm4[];
  float *sm = reinterpret_cast<float *>(sm4);
  const int W = kTdT + dil * (k - 1);
  float *ws = sm;                       // [kTdK * k][kTdWs], 16-byte rows
  float *xs = sm + (size_t)kTdK * k * kTdWs;  // [kTdK][W]
  const int t0 = blockIdx.x * kTdT, o0 = blockIdx.y * kTdC;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  float acc[4][4];
#pragma unroll
  for (int a = 0; a < 4; a++) {
    const int o = o0 + ty * 4 + a;
    const float bias = o < co ? b[o] : 0.f;
#pragma unroll
    for (int c = 0; c < 4; c++) acc[a][c] = bias;
  }
  const int kk = kTdK * k;
  for (int i0 = 0; i0 < ci; i0 += kTdK) {
    const int nc = min(kTdK, ci - i0);
    __syncthreads();
    for (int e = threadIdx.x; e < kTdK * W; e += blockDim.x) {
      const int ii = e / W, u0 = e - ii * W;
      float v = 0.f;
      if (ii < nc) {
        int u = t0 + u0 - pl;
        u = u < 0 ? -u : (u >= T ? 2 * T - 2 - u : u);
        u = min(max(u, 0), T - 1);  // only frames past T reach the clamp
        v = x[(size_t)(i0 + ii) * T + u];
      }
      xs[e] = v;
    }
    for (int e = threadIdx.x; e < kk * kTdC; e += blockDim.x) {
      const int oo = e / kk, r = e - oo * kk;  // r = ii k + j: contiguous in w
      float v = 0.f;
      if (r < nc * k && o0 + oo < co) v = w[((size_t)(o0 + oo) * ci + i0) * k + r];
      ws[r * kTdWs + oo] = v;
    }
    __syncthreads();
    for (int ii = 0; ii < nc; ii++)
      for (int j = 0; j < k; j++) {
        const float4 wv = *reinterpret_cast<const float4 *>(ws + (ii * k + j) * kTdWs + ty * 4);
        const float *xr = xs + ii * W + j * dil + tx;
        float xv[4];
#pragma unroll
        for (int c = 0; c < 4; c++) xv[c] = xr[16 * c];
#pragma unroll
        for (int c = 0; c < 4; c++) {
          acc[0][c] += wv.x * xv[c];
          acc[1][c] += wv.y * xv[c];
          acc[2][c] += wv.z * xv[c];
          acc[3][c] += wv.w * xv[c];
        }
      }
  }
#pragma unroll
  for (int a = 0; a < 4; a++) {
    const int o = o0 + ty * 4 + a;
    if (o >= co) continue;
#pragma unroll
    for (int c = 0; c < 4; c++) {
      const int t = t0 + tx + 16 * c;
      if (t < T) y[(size_t)o * T + t] = acc[a][c] > 0.f ? acc[a][c] : 0.f;
    }
  }
}

__global__ void k_add2(const float *__restrict__ a, const float *__restrict__ b, float *__restrict__ y, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    y[i] = a[i] + (b ? b[i] : 0.f);
}

// squeeze-excitation gate of one block: m = mean_t h (a warp per channel),
// z = relu(W1 m + b1), gate = sigmoid(W2 z + b2); one CTA, C <= 4096
__global__ void __launch_bounds__(1024) k_se_gate(const float *__restrict__ h, int C, int T,
                                                  const float *__restrict__ w1, const float *__restrict__ b1,
                                                  const float *__restrict__ w2, const float *__restrict__ b2, int se,
                                                  float *__restrict__ gate /* [C] */) {
  __shared__ float m[4096], z[1024];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int c = warp; c < C; c += nw) {
    float s = 0.f;
    for (int t = lane; t < T; t += 32) s += h[(size_t)c * T + t];
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) m[c] = s / (float)T;
  }
  __syncthreads();
  for (int j = threadIdx.x; j < se; j += blockDim.x) {
    float s = b1[j];
    for (int c = 0; c < C; c++) s += w1[(size_t)j * C + c] * m[c];
    z[j] = s > 0.f ? s : 0.f;
  }
  __syncthreads();
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    float s = b2[c];
    for (int j = 0; j < se; j++) s += w2[(size_t)c * se + j] * z[j];
    gate[c] = 1.f / (1.f + expf(-s));
  }
}

// x[c][t] += h[c][t] * gate[c] (the SE block's residual, res2net.rs:117)
__global__ void k_se_apply(float *__restrict__ x, const float *__restrict__ h, const float *__restrict__ gate, int T,
                           int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    x[i] += h[i] * gate[i / T];
}

// attentive statistics pooling, first half: per channel mean and standard
// deviation over time, and ain = [h; mean; std] broadcast over time
__global__ void k_asp_stats(const float *__restrict__ h, int C4, int T, float *__restrict__ ain) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C4) return;
  float s1 = 0.f, s2 = 0.f;
  for (int t = 0; t < T; t++) {
    const float v = h[(size_t)c * T + t];
    s1 += v;
    s2 += v * v;
  }
  const float mu = s1 / (float)T, var = s2 / (float)T - mu * mu;
  const float sd = sqrtf((var > 0.f ? var : 0.f) + 1e-5f);
  for (int t = 0; t < T; t++) {
    ain[(size_t)c * T + t] = h[(size_t)c * T + t];
    ain[(size_t)(C4 + c) * T + t] = mu;
    ain[(size_t)(2 * C4 + c) * T + t] = sd;
  }
}

__global__ void k_tanh(float *x, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    x[i] = tanhf(x[i]);
}

// second half, one thread per channel c: scores b[c] + W[c] . a[:, t],
// softmax over t, the weighted mean and standard deviation of h[c]
__global__ void k_asp_pool(const float *__restrict__ h, const float *__restrict__ a, int A, int C4, int T,
                           const float *__restrict__ w, const float *__restrict__ b, float *__restrict__ sc,
                           float *__restrict__ pooled) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C4) return;
  float *s = sc + (size_t)c * T;
  float mx = -INFINITY;
  for (int t = 0; t < T; t++) {
    float v = b[c];
    for (int j = 0; j < A; j++) v += w[(size_t)c * A + j] * a[(size_t)j * T + t];
    s[t] = v;
    mx = v > mx ? v : mx;
  }
  float z = 0.f;
  for (int t = 0; t < T; t++) {
    s[t] = expf(s[t] - mx);
    z += s[t];
  }
  float wm = 0.f, w2 = 0.f;
  for (int t = 0; t < T; t++) {
    const float p = s[t] / z, v = h[(size_t)c * T + t];
    wm += v * p;
    w2 += v * v * p;
  }
  const float wv = w2 - wm * wm;
  pooled[c] = wm;
  pooled[C4 + c] = sqrtf((wv > 0.f ? wv : 0.f) + 1e-5f);
}

// emb[o] = b[o] + W[o] . pooled (the final 1x1 conv)
__global__ void k_spk_fc(const float *__restrict__ pooled, int K, const float *__restrict__ w,
                         const float *__restrict__ b, int N, float *__restrict__ emb) {
  const int o = blockIdx.x * blockDim.x + threadIdx.x;
  if (o >= N) return;
  float v = b[o];
  for (int c = 0; c < K; c++) v += w[(size_t)o * K + c] * pooled[c];
  emb[o] = v;
}

inline int grid_for(int64_t n, int per) { return (int)std::min<int64_t>((n + per - 1) / per, 148 * 16); }

}  // namespace
}  // namespace q3t

using namespace q3t;

struct q3t_speaker_encoder {
  int device = 0;
  q3t_speaker_encoder_config cfg{};
  DevArena ar;
  cudaStream_t st = nullptr;
  float *win = nullptr, *fb = nullptr;
  double *cs = nullptr, *sn = nullptr;
  Tdnn block0, mfa, asp_tdnn;
  struct Se {
    Tdnn tdnn1, tdnn2;
    std::vector<Tdnn> res;
    float *w1, *b1, *w2, *b2;
  } se[3];
  float *asp_w = nullptr, *asp_b = nullptr, *fc_w = nullptr, *fc_b = nullptr;
};

namespace {

struct SpkNamed {
  std::unordered_map<std::string, const q3t_tensor *> by;
  const q3t_tensor *get(const std::string &n, std::initializer_list<int64_t> shape) const {
    auto it = by.find(n);
    if (it == by.end()) FAIL(Q3T_INVALID_INPUT, "speaker encoder: missing tensor %s", n.c_str());
    const q3t_tensor *t = it->second;
    int64_t want = 1, have = 1;
    for (int64_t s : shape) want *= s;
    for (int d = 0; d < t->ndim; d++) have *= t->shape[d];
    if (want != have)
      FAIL(Q3T_INVALID_INPUT, "speaker encoder: tensor %s has %lld elements, expected %lld", n.c_str(),
           (long long)have, (long long)want);
    if (t->dtype != Q3T_F32 && t->dtype != Q3T_BF16)
      FAIL(Q3T_INVALID_INPUT, "speaker encoder: tensor %s has an unsupported dtype", n.c_str());
    return t;
  }
};

template <class T>
T *spk_upload(q3t_speaker_encoder *e, const std::vector<T> &v) {
  T *d = e->ar.alloc<T>(v.size());
  CK(cudaMemcpy(d, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice));
  return d;
}

float *spk_upload(q3t_speaker_encoder *e, const q3t_tensor *t) {
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
  return spk_upload(e, v);
}

Tdnn load_tdnn(q3t_speaker_encoder *e, const SpkNamed &T, const std::string &name, int ci, int co, int k, int dil) {
  Tdnn t;
  t.ci = ci;
  t.co = co;
  t.k = k;
  t.dil = dil;
  if (tdnn_smem(k, dil * (k - 1)) > 48 * 1024)
    FAIL(Q3T_INVALID_INPUT, "speaker encoder: %s spans too many frames (kernel %d, dilation %d)", name.c_str(), k, dil);
  t.w = spk_upload(e, T.get(name + ".weight", {co, ci, k}));
  t.b = spk_upload(e, T.get(name + ".bias", {co}));
  return t;
}

void run_tdnn(const Tdnn &b, const float *x, int T, float *y, cudaStream_t st) {
  const int total = b.dil * (b.k - 1), pl = total / 2;
  k_tdnn<<<dim3((T + kTdT - 1) / kTdT, (b.co + kTdC - 1) / kTdC), 256, tdnn_smem(b.k, total), st>>>(
      x, b.ci, T, b.w, b.b, b.co, b.k, b.dil, pl, y);
  note_launch(cudaGetLastError(), "k_tdnn");
  g_launches++;
}

int spk_frames(int64_t n) { return (int)((n + 2 * kPad - kNfft) / kHop + 1); }

// the log-mel features [n_mels][frames] of samples [n] into device memory
float *spk_mel(q3t_speaker_encoder *e, const float *samples, int64_t n, int *frames_out) {
  const int frames = spk_frames(n), plen = (int)n + 2 * kPad;
  std::vector<float> p((size_t)plen);
  for (int i = 0; i < kPad; i++) {  // left: samples[pad], ..., samples[1] (feature.rs:100-102)
    const int idx = kPad - i;
    p[(size_t)i] = samples[idx < n - 1 ? idx : n - 1];
  }
  memcpy(p.data() + kPad, samples, (size_t)n * 4);
  for (int i = 0; i < kPad; i++) {  // right: samples[n - 2 - i], saturating (feature.rs:104-109)
    int64_t idx = n - 2 - i;
    idx = idx < 0 ? 0 : (idx > n - 1 ? n - 1 : idx);
    p[(size_t)kPad + n + i] = samples[idx];
  }
  cudaStream_t st = e->st;
  float *dp = nullptr, *mel = nullptr;
  CK(cudaMallocAsync((void **)&dp, (size_t)plen * 4, st));
  CK(cudaMallocAsync((void **)&mel, (size_t)e->cfg.mel_dim * frames * 4, st));
  CK(cudaMemcpyAsync(dp, p.data(), (size_t)plen * 4, cudaMemcpyHostToDevice, st));
  k_spk_mel<<<frames, 256, 0, st>>>(dp, e->win, e->cs, e->sn, e->fb, e->cfg.mel_dim, frames, mel);
  note_launch(cudaGetLastError(), "k_spk_mel");
  g_launches++;
  CK(cudaFreeAsync(dp, st));
  CK(cudaStreamSynchronize(st));  // the host padding buffer goes out of scope
  *frames_out = frames;
  return mel;
}

void spk_forward(q3t_speaker_encoder *e, const float *mel, int T, float *emb_host) {
  const auto &c = e->cfg;
  cudaStream_t st = e->st;
  const int C = c.channels[1], C4 = c.channels[4], A = c.attention_channels, cs = C / c.res2net_scale;
  // reflect padding needs T > half the receptive field of every block
  // (the reference's slices reject shorter inputs, tdnn.rs:45-82)
  std::vector<const Tdnn *> all = {&e->block0, &e->mfa, &e->asp_tdnn};
  for (const auto &B : e->se) all.push_back(&B.res[0]);
  for (const Tdnn *b : all) {
    const int total = b->dil * (b->k - 1), pl = total / 2, pr = total - pl;
    if ((pl > 0 && T < pl + 1) || (pr > 0 && T < pr + 1))
      FAIL(Q3T_INVALID_INPUT, "speaker encoder: %d frames are too few for the reflect padding", T);
  }
  std::vector<void *> ws;
  auto wsalloc = [&](size_t floats) {
    void *p = nullptr;
    CK(cudaMallocAsync(&p, (floats ? floats : 1) * 4, st));
    ws.push_back(p);
    return static_cast<float *>(p);
  };
  float *x = wsalloc((size_t)C * T), *cat = wsalloc((size_t)3 * C * T), *h = wsalloc((size_t)C * T);
  float *g = wsalloc((size_t)C * T), *in = wsalloc((size_t)cs * T), *scr = wsalloc((size_t)C);
  run_tdnn(e->block0, mel, T, x, st);
  for (int i = 0; i < 3; i++) {  // network/mod.rs:75-92
    const auto &B = e->se[i];
    run_tdnn(B.tdnn1, x, T, h, st);
    CK(cudaMemcpyAsync(g, h, (size_t)cs * T * 4, cudaMemcpyDeviceToDevice, st));
    for (int s = 1; s < c.res2net_scale; s++) {
      k_add2<<<grid_for((int64_t)cs * T, 256), 256, 0, st>>>(h + (size_t)s * cs * T,
                                                             s > 1 ? g + (size_t)(s - 1) * cs * T : nullptr, in,
                                                             (int64_t)cs * T);
      note_launch(cudaGetLastError(), "k_add2");
      g_launches++;
      run_tdnn(B.res[s - 1], in, T, g + (size_t)s * cs * T, st);
    }
    run_tdnn(B.tdnn2, g, T, h, st);
    k_se_gate<<<1, 1024, 0, st>>>(h, C, T, B.w1, B.b1, B.w2, B.b2, c.se_channels, scr);
    k_se_apply<<<grid_for((int64_t)C * T, 256), 256, 0, st>>>(x, h, scr, T, (int64_t)C * T);
    note_launch(cudaGetLastError(), "k_se_gate / k_se_apply");
    g_launches += 2;
    CK(cudaMemcpyAsync(cat + (size_t)i * C * T, x, (size_t)C * T * 4, cudaMemcpyDeviceToDevice, st));
  }
  float *hm = wsalloc((size_t)C4 * T), *ain = wsalloc((size_t)3 * C4 * T), *a = wsalloc((size_t)A * T);
  float *sc = wsalloc((size_t)C4 * T), *pooled = wsalloc((size_t)2 * C4), *emb = wsalloc((size_t)c.enc_dim);
  run_tdnn(e->mfa, cat, T, hm, st);
  k_asp_stats<<<(C4 + 127) / 128, 128, 0, st>>>(hm, C4, T, ain);
  run_tdnn(e->asp_tdnn, ain, T, a, st);
  k_tanh<<<grid_for((int64_t)A * T, 256), 256, 0, st>>>(a, (int64_t)A * T);
  k_asp_pool<<<(C4 + 127) / 128, 128, 0, st>>>(hm, a, A, C4, T, e->asp_w, e->asp_b, sc, pooled);
  k_spk_fc<<<(c.enc_dim + 127) / 128, 128, 0, st>>>(pooled, 2 * C4, e->fc_w, e->fc_b, c.enc_dim, emb);
  note_launch(cudaGetLastError(), "speaker encoder pooling");
  g_launches += 4;
  const char *kn = "";
  const cudaError_t le = take_launch_error(&kn);
  if (le != cudaSuccess) throw CudaFail{le, kn};
  CK(cudaMemcpyAsync(emb_host, emb, (size_t)c.enc_dim * 4, cudaMemcpyDeviceToHost, st));
  for (void *p : ws) CK(cudaFreeAsync(p, st));
  CK(cudaStreamSynchronize(st));
}

template <class F>
q3t_status spk_guard(F &&f) {
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

}  // namespace

extern "C" q3t_status q3t_speaker_encoder_load(const q3t_speaker_encoder_desc *d, q3t_speaker_encoder **out) {
  if (!d || !out || (d->num_tensors > 0 && !d->tensors)) {
    set_error("q3t_speaker_encoder_load: null argument");
    return Q3T_INVALID_INPUT;
  }
  *out = nullptr;
  auto *e = new q3t_speaker_encoder();
  const q3t_status rc = spk_guard([&] {
    const q3t_speaker_encoder_config &c = d->config;
    bool ok = c.mel_dim > 0 && c.enc_dim > 0 && c.attention_channels > 0 && c.se_channels > 0 &&
              c.se_channels <= 1024 &&
              c.res2net_scale >= 2 && c.sample_rate > 0 && c.channels[1] % c.res2net_scale == 0 &&
              c.channels[1] == c.channels[2] && c.channels[1] == c.channels[3] && c.channels[1] <= 4096;
    for (int i = 0; i < 5; i++) ok = ok && c.channels[i] > 0 && c.kernel_sizes[i] > 0 && c.dilations[i] > 0;
    if (!ok) FAIL(Q3T_INVALID_INPUT, "speaker encoder: invalid config");
    e->cfg = c;
    e->device = d->device;
    CK(cudaSetDevice(d->device));
    CK(cudaStreamCreateWithFlags(&e->st, cudaStreamNonBlocking));
    SpkNamed T;
    for (int i = 0; i < d->num_tensors; i++) T.by[d->tensors[i].name] = &d->tensors[i];
    const std::string p = "speaker_encoder";
    const int C = c.channels[1], cs = C / c.res2net_scale;
    e->block0 = load_tdnn(e, T, p + ".blocks.0.conv", c.mel_dim, c.channels[0], c.kernel_sizes[0], c.dilations[0]);
    if (c.channels[0] != C) FAIL(Q3T_INVALID_INPUT, "speaker encoder: block 0 width must equal the SE blocks'");
    for (int i = 1; i < 4; i++) {
      const std::string b = p + ".blocks." + std::to_string(i);
      auto &B = e->se[i - 1];
      B.tdnn1 = load_tdnn(e, T, b + ".tdnn1.conv", C, C, 1, 1);
      for (int j = 0; j < c.res2net_scale - 1; j++)
        B.res.push_back(load_tdnn(e, T, b + ".res2net_block.blocks." + std::to_string(j) + ".conv", cs, cs,
                                  c.kernel_sizes[i], c.dilations[i]));
      B.tdnn2 = load_tdnn(e, T, b + ".tdnn2.conv", C, C, 1, 1);
      B.w1 = spk_upload(e, T.get(b + ".se_block.conv1.weight", {c.se_channels, C, 1}));
      B.b1 = spk_upload(e, T.get(b + ".se_block.conv1.bias", {c.se_channels}));
      B.w2 = spk_upload(e, T.get(b + ".se_block.conv2.weight", {C, c.se_channels, 1}));
      B.b2 = spk_upload(e, T.get(b + ".se_block.conv2.bias", {C}));
    }
    const int C4 = c.channels[4];
    e->mfa = load_tdnn(e, T, p + ".mfa.conv", 3 * C, C4, c.kernel_sizes[4], c.dilations[4]);
    e->asp_tdnn = load_tdnn(e, T, p + ".asp.tdnn.conv", 3 * C4, c.attention_channels, 1, 1);
    e->asp_w = spk_upload(e, T.get(p + ".asp.conv.weight", {C4, c.attention_channels, 1}));
    e->asp_b = spk_upload(e, T.get(p + ".asp.conv.bias", {C4}));
    e->fc_w = spk_upload(e, T.get(p + ".fc.weight", {c.enc_dim, 2 * C4, 1}));
    e->fc_b = spk_upload(e, T.get(p + ".fc.bias", {c.enc_dim}));
    // periodic Hann window (feature.rs:135-142) and the mel filterbank
    // (feature.rs:156-194), f32 on the host as the reference builds them
    std::vector<float> win(kNfft), fb((size_t)c.mel_dim * kBins, 0.f), hz((size_t)c.mel_dim + 2);
    for (int i = 0; i < kNfft; i++) win[(size_t)i] = 0.5f - 0.5f * cosf(2.0f * (float)M_PI * (float)i / (float)kNfft);
    auto hz_to_mel = [](float f) { return 2595.0f * log10f(1.0f + f / 700.0f); };
    auto mel_to_hz = [](float m) { return 700.0f * (powf(10.0f, m / 2595.0f) - 1.0f); };
    const float mn = hz_to_mel(0.0f), mx = hz_to_mel((float)c.sample_rate / 2.0f);
    for (int i = 0; i <= c.mel_dim + 1; i++)
      hz[(size_t)i] = mel_to_hz(mn + (mx - mn) * (float)i / (float)(c.mel_dim + 1));
    for (int m = 0; m < c.mel_dim; m++) {
      const float l = hz[(size_t)m], ce = hz[(size_t)m + 1], r = hz[(size_t)m + 2];
      for (int f = 0; f < kBins; f++) {
        const float fq = (float)f * (float)c.sample_rate / (float)kNfft;
        float v = 0.f;
        if (fq >= l && fq <= ce && ce > l)
          v = (fq - l) / (ce - l);
        else if (fq > ce && fq <= r && r > ce)
          v = (r - fq) / (r - ce);
        fb[(size_t)m * kBins + f] = v;
      }
      const float bw = hz[(size_t)m + 2] - hz[(size_t)m];
      if (bw > 0.f)
        for (int f = 0; f < kBins; f++) fb[(size_t)m * kBins + f] *= 2.0f / bw;
    }
    std::vector<double> cs_t(kNfft), sn_t(kNfft);
    for (int r = 0; r < kNfft; r++) {  // the 1024 roots exp(-2 pi i r / 1024) as cos / sin
      cs_t[(size_t)r] = cos(2.0 * M_PI * r / kNfft);
      sn_t[(size_t)r] = sin(2.0 * M_PI * r / kNfft);
    }
    e->win = spk_upload(e, win);
    e->fb = spk_upload(e, fb);
    e->cs = spk_upload(e, cs_t);
    e->sn = spk_upload(e, sn_t);
  });
  if (rc != Q3T_OK) {
    q3t_speaker_encoder_free(e);
    return rc;
  }
  *out = e;
  return Q3T_OK;
}

void q3t_speaker_encoder_free(q3t_speaker_encoder *e) {
  if (!e) return;
  cudaSetDevice(e->device);
  if (e->st) {
    cudaStreamSynchronize(e->st);
    cudaStreamDestroy(e->st);
  }
  e->ar.release();
  delete e;
}

extern "C" q3t_status q3t_speaker_mel(q3t_speaker_encoder *e, const float *samples, int64_t num_samples,
                                      float *mel, int max_frames, int *frames) {
  if (!e || !samples || !mel || num_samples < kNfft - 2 * kPad || num_samples > (int64_t)1 << 28) {
    set_error("q3t_speaker_mel: null argument or sample count outside %d..2^28", kNfft - 2 * kPad);
    return Q3T_INVALID_INPUT;
  }
  return spk_guard([&] {
    CK(cudaSetDevice(e->device));
    if (spk_frames(num_samples) > max_frames)
      FAIL(Q3T_INVALID_INPUT, "speaker mel: %d frames exceed max_frames %d", spk_frames(num_samples), max_frames);
    int T = 0;
    float *d = spk_mel(e, samples, num_samples, &T);
    CK(cudaMemcpyAsync(mel, d, (size_t)e->cfg.mel_dim * T * 4, cudaMemcpyDeviceToHost, e->st));
    CK(cudaFreeAsync(d, e->st));
    CK(cudaStreamSynchronize(e->st));
    if (frames) *frames = T;
  });
}

extern "C" q3t_status q3t_speaker_embed(q3t_speaker_encoder *e, const float *samples, int64_t num_samples,
                                        float *embedding) {
  if (!e || !samples || !embedding || num_samples < kNfft - 2 * kPad || num_samples > (int64_t)1 << 28) {
    set_error("q3t_speaker_embed: null argument or sample count outside %d..2^28", kNfft - 2 * kPad);
    return Q3T_INVALID_INPUT;
  }
  return spk_guard([&] {
    CK(cudaSetDevice(e->device));
    int T = 0;
    float *mel = spk_mel(e, samples, num_samples, &T);
    try {
      spk_forward(e, mel, T, embedding);
    } catch (...) {
      cudaFreeAsync(mel, e->st);
      cudaStreamSynchronize(e->st);
      throw;
    }
    CK(cudaFreeAsync(mel, e->st));
    CK(cudaStreamSynchronize(e->st));
  });
}

/*
 * CPU oracle for the Qwen3-TTS synthesis hot path — TEST INFRASTRUCTURE ONLY.
 *
 * This is a plain-C restatement of the reference's math (onenewcode/tts-rs,
 * Rust on Burn 0.21).  It exists to check the CUDA library and to serve as
 * the timed CPU baseline; the product never links, loads or calls it.
 *
 * Parity status:
 *   - pinned: greedy/suppress and top-k=1 sampling KATs
 *     (tts_qwen3_tts/src/model/talker/infer/sampling.rs:165-219), KV-cache
 *     reset/append KATs (talker/network/kv.rs:220-273), pad_1d constant/edge
 *     KATs (codec/network/conv.rs:94-140), attention shape KAT
 *     (model/nn/attention.rs:37-79);
 *   - parity unpinned: transformer / attention / RoPE / MLP / code-predictor
 *     / codec-decoder numerics.  The reference cannot be compiled here (no
 *     Rust toolchain, Burn not vendored) and ships no golden vectors, so
 *     these are a line-by-line restatement of the cited Rust, nothing more.
 *
 * Precision model: talker/predictor weights are bf16 values held in f32;
 * every Linear input is rounded to bf16 and K/V/Q are stored as bf16 (the
 * reference's bf16 runtime dtype); accumulation, norms, softmax are f32
 * (model/nn/attention.rs:13-26 promotes attention to f32).  The codec is
 * pure f32 (the reference f32 codec output is the comparison target).
 */
#ifndef Q3T_ORACLE_H
#define Q3T_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------- transformer stacks (talker / code predictor) ---------- */
typedef struct {
  int hidden, inter, n_layers, n_heads, n_kv, head_dim;
  float eps, theta;
} orc_lm_cfg;

typedef struct {
  const float *in_norm, *post_norm;       /* [hidden] */
  const float *wq, *wk, *wv, *wo;         /* PyTorch layout [out][in] */
  const float *q_norm, *k_norm;           /* [head_dim] */
  const float *w_gate, *w_up, *w_down;    /* [out][in] */
} orc_layer;

typedef struct {
  orc_lm_cfg cfg;
  const orc_layer *layers;                /* n_layers entries */
  const float *final_norm;                /* [hidden] */
} orc_stack;

/* Dense autoregressive cache for one layer, batch 1: [n_kv][cap][head_dim]
 * (talker/network/kv.rs:5-161).  k/v owned by the caller. */
typedef struct {
  float *k, *v;
  int len, cap, n_kv, head_dim;
} orc_kv;

void orc_set_threads(int n);
int orc_get_threads(void);

float orc_bf16_round(float x);
void orc_bf16_round_array(float *x, int64_t n);

/* kv.rs:56-161: append S new steps k_new/v_new [n_kv][S][hd], sliding when
 * full; writes the valid slice [n_kv][len][hd] to k_out/v_out (may be NULL)
 * and returns its length. */
int orc_kv_forward(orc_kv *c, const float *k_new, const float *v_new, int S,
                   float *k_out, float *v_out);
/* kv.rs:46-53 */
void orc_kv_reset_preserve(orc_kv *c);

/* layer.rs / model.rs / predictor.rs: runs S tokens through every layer of
 * the stack, positions = cache.len + s, causal mask iff the caches were
 * empty (model.rs:44-56, infer/mod.rs:555-558).  out = final RMSNorm output
 * [S][hidden] (f32). */
void orc_stack_forward(const orc_stack *st, orc_kv *caches, const float *x,
                       int S, float *out);

/* y[n] = sum_k W[n][k] * bf16(x[k]) for S rows; W [N][K] */
void orc_linear(const float *W, const float *bias, const float *x, int S,
                int K, int N, float *y);

/* session_seed.rs:668-679 + mlp.rs:36-40: text embedding -> fc1 + b1 -> silu
 * (bf16) -> fc2 + b2 (bf16); out [n][H] */
void orc_text_project(const float *emb, const float *w1, const float *b1, const float *w2,
                      const float *b2, int Ht, int H, const int64_t *ids, int n, float *out);

/* --------------------------- sampling ----------------------------------- */
typedef struct {
  int do_sample;
  float temperature;
  int top_k;          /* <= 0 : none */
  float top_p;
  float repetition_penalty; /* <= 0 or NaN : none */
} orc_sampling;

/* sampling.rs:128-150 — in-place on logits[V] */
void orc_apply_repetition_penalty(float *logits, int V, const int64_t *hist,
                                  int n_hist, float penalty);
int orc_repetition_penalty_enabled(float penalty);
/* sampling.rs:33-99; u = uniform [0,1) draw used by the categorical step */
int64_t orc_sample_token(const float *logits, int V, const orc_sampling *s,
                         const int64_t *suppress, int n_suppress, float u);
/* session_seed.rs:144-149 */
int orc_build_suppress_ids(int vocab, int64_t eos, int64_t *out);

/* ------------------------- talker generator ------------------------------ */
typedef struct {
  orc_stack talker, predictor;
  const float *codec_head;        /* [vocab][hidden] */
  const float *talker_codec_emb;  /* [vocab][hidden] */
  const float *const *cp_codec_emb; /* n_groups-1 x [cp_vocab][hidden] */
  const float *const *lm_heads;     /* n_groups-1 x [cp_vocab][cp_hidden] */
  int vocab, cp_vocab, n_groups;
} orc_talker;

typedef struct orc_gen orc_gen;

/* infer/mod.rs:69-188.  inputs [S][hidden]; trailing [T_tr][hidden]; pad
 * [hidden]; eos < 0 means None. */
orc_gen *orc_gen_start(const orc_talker *m, const float *inputs, int S,
                       const float *trailing, int trailing_len,
                       const float *pad, const orc_sampling *talker_s,
                       const orc_sampling *cp_s, int max_new_tokens,
                       int64_t eos, const int64_t *suppress, int n_suppress,
                       int64_t forced_first, float *first_logits, int *status);
/* infer/mod.rs:190-299.  forced: NULL or [n_groups] codes that replace the
 * sampled ones (teacher forcing; forced[0] is the code that was sampled by
 * the previous call).  Dumps: talker_logits [vocab] (the next talker token's
 * logits), cp_logits [(n_groups-1)][cp_vocab].  u: n_groups uniforms.
 * Returns 1 = advanced, 2 = finished, 0 = already finished (None), <0 error. */
int orc_gen_step(orc_gen *g, const int64_t *forced_codes, const float *u,
                 float *talker_logits, float *cp_logits, float *hidden_out);
int orc_gen_num_frames(const orc_gen *g);
void orc_gen_codes(const orc_gen *g, int64_t *out); /* [n_groups][T] */
void orc_gen_free(orc_gen *g);

/* one code-predictor frame (infer/mod.rs:434-535) on its own: hidden [hidden],
 * code0 -> codes[n_groups]; logits dump [(n_groups-1)][cp_vocab] */
void orc_predict_frame(const orc_talker *m, const float *hidden, int64_t code0,
                       const orc_sampling *s, const int64_t *forced,
                       const float *u, int64_t *codes, float *logits);

/* infer/mod.rs:343-383: codes[n_groups] -> embedding sum (+ extra row) */
void orc_codec_group_embedding(const orc_talker *m, const int64_t *codes,
                               const float *extra, float *out);

/* ---------------------------- codec decoder ------------------------------ */
typedef struct {
  const float *w1, *b1;      /* conv k7 dil d: [C][C][7], [C] */
  const float *w2, *b2;      /* conv k1: [C][C][1], [C] */
  const float *a1_alpha, *a1_beta, *a2_alpha, *a2_beta; /* [C] */
} orc_resunit;

typedef struct {
  const float *snake_alpha, *snake_beta; /* [Cin] */
  const float *wt, *bt;                  /* ConvT [Cin][Cout][2r], [Cout] */
  orc_resunit ru[3];
} orc_wave_stage;

typedef struct {
  const float *wt, *bt;           /* ConvT [C][C][r], [C] */
  const float *dw_w, *dw_b;       /* depthwise [C][1][7], [C] */
  const float *ln_w, *ln_b;       /* [C] */
  const float *pw1_w, *pw1_b;     /* [4C][C], [4C] */
  const float *pw2_w, *pw2_b;     /* [C][4C], [C] */
  const float *gamma;             /* [C] */
} orc_convnext;

typedef struct {
  const float *in_norm, *post_norm;
  const float *wq, *wk, *wv, *wo;
  const float *attn_scale, *mlp_scale;
  const float *w_gate, *w_up, *w_down;
} orc_codec_layer;

typedef struct {
  /* config (codec/config.rs:50-76) */
  int n_q, n_semantic, codebook_size, codebook_dim, latent, decoder_dim;
  int hidden, inter, n_layers, n_heads, n_kv, head_dim;
  float eps, theta;
  int n_up; int up_ratio[4];
  int n_stage; int rates[8];
  /* weights */
  const float *const *emb_sum;   /* n_q x [codebook_size][codebook_dim/2] */
  const float *const *usage;     /* n_q x [codebook_size] */
  const float *first_out_proj;   /* [codebook_dim][codebook_dim/2][1] */
  const float *rest_out_proj;
  const float *pre_conv_w, *pre_conv_b;  /* [latent][codebook_dim][3] */
  const float *in_proj_w, *in_proj_b;    /* [hidden][latent] */
  const float *out_proj_w, *out_proj_b;  /* [latent][hidden] */
  const float *final_norm;               /* [hidden] */
  const orc_codec_layer *layers;
  const orc_convnext *up;
  const float *in_conv_w, *in_conv_b;    /* [decoder_dim][latent][7] */
  const orc_wave_stage *stages;
  const float *out_alpha, *out_beta;     /* [decoder_dim >> n_stage] */
  const float *out_conv_w, *out_conv_b;  /* [1][C][7], [1] */
} orc_codec;

/* number of output samples for T frames (decoder.rs:250-278, conv.rs:19-31) */
int64_t orc_codec_out_len(const orc_codec *c, int T);
/* codes [B][n_q][T] -> wave [B][out_len]; returns 0 or <0 on bad input */
int orc_codec_decode(const orc_codec *c, const int64_t *codes, int B, int T,
                     float *wave);
/* intermediate taps of one batch item, written channel-major [C][L]:
 * 0 = quantizer out, 1 = pre_conv out, 2 = pre_transformer out,
 * 3 = after the ConvNeXt upsamplers, 4 = wave input conv,
 * 5.. 4+n_stage = after each wave stage, 5+n_stage = final clamped wave.
 * out may be NULL to query the size; returns C*L or <0 on bad input. */
int64_t orc_codec_decode_tap(const orc_codec *c, const int64_t *codes, int T,
                             int tap, float *out);

/* codec/network/conv.rs:71-83 pad_1d (mode 0 = constant 0, 1 = edge) */
void orc_pad_1d(const float *x, int C, int L, int left, int right, int mode,
                float *out);
/* codec/network/conv.rs:44-64 */
void orc_conv1d_padding(int L, int k, int dil, int stride, int *pad_total,
                        int *extra);
/* codec/infer/mod.rs:80-90 */
void orc_to_pcm(const float *x, int64_t n, int16_t *out);

/* nn/attention.rs:5-27 on [H][S][D] f32 tensors, mask [S][L] (1 = masked) */
void orc_sdpa(const float *q, const float *k, const float *v,
              const uint8_t *mask, int H, int S, int L, int D, float scale,
              float *out);

/* ------------------------------------------------------------------------ */
/* Codec encoder (voice-clone reference audio): codec/network/encoder.rs,    */
/* codec/config.rs:136-346                                                   */
/* ------------------------------------------------------------------------ */
typedef struct {
  const float *w, *b; /* Conv1d weight [co][ci][k], bias [co] (nullable) */
  int ci, co, k, stride;
} orc_conv;

typedef struct {
  const float *ln1_w, *ln1_b, *ln2_w, *ln2_b;               /* [H] */
  const float *wq, *bq, *wk, *bk, *wv, *bv, *wo, *bo;       /* [out][in], biases nullable */
  const float *attn_scale, *mlp_scale;                      /* LayerScale [H] */
  const float *fc1, *fc2;                                   /* [inter][H], [H][inter] */
} orc_enc_layer;

typedef struct {
  const float *in_proj;             /* Conv1d k1 [vq][H][1], no bias */
  const float *const *embed_sum;    /* n_layers x [codebook_size][vq] */
  const float *const *usage;        /* n_layers x [codebook_size] */
  int n_layers;
} orc_enc_rvq;

typedef struct {
  int hidden, n_layers, n_heads, n_kv, head_dim, inter, codebook_size, vq_dim;
  float norm_eps, theta;
  int n_stages;
  orc_conv in_conv;                 /* audio -> num_filters, constant pad */
  orc_conv res_in[8], res_out[8];   /* per stage: resnet k_res (C -> C/compress) and k1 back */
  orc_conv down[8];                 /* per stage: C -> 2C, kernel 2r, stride r */
  orc_conv out_conv;                /* -> hidden, last_kernel_size */
  const orc_enc_layer *layers;
  orc_conv downsample;              /* hidden -> hidden, stride 2, edge pad, no bias */
  orc_enc_rvq semantic, acoustic;
} orc_codec_encoder;

/* Qwen3TtsAudioCodecEncoder::encode_reference_prefix (encoder.rs:121-136):
 * wave [n] (one channel) -> codes [n_valid][T] (semantic layers first, then
 * n_valid - n_semantic acoustic ones).  Returns T, or < 0 on bad input or
 * when the codes would not fit max_frames. */
int orc_codec_encode(const orc_codec_encoder *e, const float *wave, int n, int n_valid, int64_t *codes,
                     int max_frames);
/* the hidden [hidden][T] the quantizers read (after the stride-2
 * downsample); returns T or < 0 */
int orc_codec_encoder_hidden(const orc_codec_encoder *e, const float *wave, int n, float *out, int max_frames);
/* one residual vector quantizer's encode (encoder.rs:319-368) on x [vq][T]
 * (already through input_proj): codes [n_layers][T]; x is left holding the
 * final residual */
void orc_rvq_encode(const float *const *embed_sum, const float *const *usage, int n_layers, int codebook_size,
                    int vq, float *x, int T, int64_t *codes);

/* ------------------------------------------------------------------------ */
/* Speaker encoder (voice-clone x-vector): model/speaker/{infer,network}     */
/* ------------------------------------------------------------------------ */
/* speaker/infer/feature.rs: log-mel features of n samples (n >= 256):
 * reflect-padded STFT (n_fft 1024, hop 256, periodic Hann window; the DFT
 * rustfft 6.4.1 computes), magnitudes, mel filters with area normalisation,
 * ln(max(., 1e-5)) -> out [n_mels][frames].  Returns frames, < 0 on bad input
 * or when they would not fit max_frames. */
int orc_speaker_mel(const float *samples, int n, int sample_rate, int n_mels, float *out, int max_frames);

typedef struct {
  const float *w, *b; /* Conv1d [co][ci][k], bias [co] */
  int ci, co, k, dil;
} orc_tdnn;           /* reflect pad, conv, ReLU (speaker/network/tdnn.rs) */

typedef struct {
  orc_tdnn tdnn1, tdnn2;     /* k1 */
  orc_tdnn res[15];          /* scale - 1 Res2Net branches */
  int scale;
  const float *se_w1, *se_b1, *se_w2, *se_b2; /* [se][C][1], [se], [C][se][1], [C] */
  int se_ch;
} orc_se_block;

typedef struct {
  int mel_dim, enc_dim, sample_rate;
  int channels[5];
  orc_tdnn block0;
  orc_se_block se[3];
  orc_tdnn mfa;
  orc_tdnn asp_tdnn;               /* 3C -> attention channels, k1 */
  const float *asp_w, *asp_b;      /* [C][att][1], [C] */
  const float *fc_w, *fc_b;        /* [enc_dim][2C][1], [enc_dim] */
} orc_speaker;

/* SpeakerEncoderNetwork::forward (network/mod.rs:71-99) on mel [mel_dim][T]
 * -> emb [enc_dim]; < 0 on bad input */
int orc_speaker_forward(const orc_speaker *s, const float *mel, int T, float *emb);
/* encode_embedding (infer/mod.rs:11-20): samples -> emb [enc_dim] */
int orc_speaker_embed(const orc_speaker *s, const float *samples, int n, float *emb);

#ifdef __cplusplus
}
#endif
#endif

/*
 * q3t.h — C ABI of the B200 (sm_100a) Qwen3-TTS synthesis hot path.
 *
 * Drop-in boundary for the `tts_qwen3_tts` driver of onenewcode/tts-rs: the
 * Rust driver keeps its surface (surface/mod.rs), package loading and
 * request compiler, and replaces three things with calls into this library:
 *   - the Burn weight load        (tts_qwen3_tts/src/loading/runtime.rs:131-156)
 *   - TalkerGenerator start/step/finalize
 *                                 (tts_qwen3_tts/src/model/talker/infer/mod.rs:69-311)
 *   - decode_waveform + to_pcm    (tts_qwen3_tts/src/model/codec/infer/mod.rs:61-111)
 * and gains a ragged continuous-batching scheduler (no reference counterpart:
 * the reference is batch-1, talker/infer/mod.rs:92-96).
 *
 * Conventions: plain pointers and sizes; host buffers are owned by the
 * caller and copied on entry/exit; every device buffer (weights, KV pages,
 * activations, workspaces) is owned by the library and freed by *_free.
 * Every call returns a q3t_status; q3t_last_error() gives the message of the
 * last failure on the calling thread.  A model handle is immutable after load
 * and may be shared by threads; sessions and batches are single-threaded.
 */
#ifndef Q3T_H
#define Q3T_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define Q3T_ABI_VERSION 1

/* Status codes.  The first four mirror Qwen3TtsInferenceError variants
 * (tts_qwen3_tts/src/error.rs:64-101) so the Rust side maps them 1:1. */
typedef enum {
  Q3T_OK = 0,
  Q3T_INVALID_INPUT = 1,   /* QwenTtsInferenceError::InvalidInput */
  Q3T_RUNTIME_LOAD = 2,    /* QwenTtsInferenceError::RuntimeLoad (missing / bad tensor) */
  Q3T_TENSOR_READ = 3,     /* QwenTtsInferenceError::TensorRead (device -> host read failed) */
  Q3T_DEVICE_TIMEOUT = 4,  /* a bounded device-side wait gave up */
  Q3T_OUT_OF_PAGES = 5,    /* KV page pool exhausted (the reference slides; see q3t_session_desc) */
  Q3T_CUDA_ERROR = 6       /* CUDA runtime error (message has the CUDA error string) */
} q3t_status;

typedef enum { Q3T_F32 = 0, Q3T_BF16 = 1 } q3t_dtype;

/* Decoder-stack hyper-parameters (tts_qwen3_tts/src/model/talker/config.rs:18-61).
 * Kernels are specialised for head_dim 128, hidden % 256 == 0, intermediate % 256 == 0. */
typedef struct {
  int hidden_size;
  int intermediate_size;
  int num_hidden_layers;
  int num_attention_heads;
  int num_key_value_heads;
  int head_dim;
  int vocab_size;
  float rms_norm_eps;
  float rope_theta;
} q3t_lm_config;

typedef struct {
  q3t_lm_config talker;      /* talker_config */
  q3t_lm_config predictor;   /* talker_config.code_predictor_config */
  int num_code_groups;       /* 16 */
} q3t_talker_config;

/* Speech-tokenizer decoder config (tts_qwen3_tts/src/model/codec/config.rs:50-76). */
typedef struct {
  int num_quantizers;            /* 16 */
  int num_semantic_quantizers;   /* 1 */
  int codebook_size;             /* 2048 */
  int codebook_dim;              /* 512 (tables are codebook_dim / 2 wide) */
  int latent_dim;                /* 1024 */
  int decoder_dim;               /* 1536 */
  int hidden_size;               /* pre-transformer width, 512 */
  int intermediate_size;         /* 1024 */
  int num_hidden_layers;         /* 8 */
  int num_attention_heads;       /* 16 */
  int num_key_value_heads;       /* 16 */
  int head_dim;                  /* 64 */
  float rms_norm_eps;            /* 1e-5 */
  float rope_theta;              /* 1e4 */
  int num_upsampling_ratios;
  int upsampling_ratios[4];      /* [2, 2] */
  int num_upsample_rates;
  int upsample_rates[8];         /* [8, 5, 4, 3] */
  int output_sample_rate;        /* 24000 */
} q3t_codec_config;

/* One named tensor in PyTorch layout (Linear [out,in], Conv1d [out,in/g,k],
 * ConvTranspose1d [in,out,k]).  Names are the checkpoint names the reference
 * loads (talker/weights.rs:14, codec/weights.rs:13-33), e.g.
 * "talker.model.layers.0.self_attn.q_proj.weight" or
 * "decoder.quantizer.rvq_rest.vq.layers.3._codebook.embedding_sum". */
typedef struct {
  const char *name;
  int dtype;                 /* q3t_dtype of `data` (host memory) */
  int ndim;
  int64_t shape[4];
  const void *data;
} q3t_tensor;

typedef struct {
  int device;                /* CUDA device ordinal */
  q3t_talker_config talker;
  int has_talker;            /* 0: codec-only model */
  q3t_codec_config codec;
  int has_codec;             /* 0: talker-only model */
  const q3t_tensor *tensors;
  int num_tensors;
  int64_t kv_pages;          /* talker KV pool size in 16-token pages (0: 8192) */
  int max_active;            /* max requests in one batched step, 1..64 (0: 64) */
} q3t_model_desc;

typedef struct q3t_model q3t_model;

/* Replaces loading/runtime.rs:131-156 (safetensors -> Burn with the bf16
 * load-time cast): copies every tensor into device memory (bf16 for the
 * linears, with their TMA descriptors; f32 for norms and codec tables). */
q3t_status q3t_model_load(const q3t_model_desc *desc, q3t_model **out);
void q3t_model_free(q3t_model *model);

/* Sampling (tts_qwen3_tts/src/model/talker/infer/sampling.rs:12-31).
 * top_k <= 0: none; repetition_penalty <= 0, NaN or 1: none.  seed drives the
 * on-device categorical draw (Burn's RNG stream is not reproducible). */
typedef struct {
  int do_sample;
  float temperature;
  int top_k;
  float top_p;
  float repetition_penalty;
  uint64_t seed;
} q3t_sampling;

/* TalkerGeneratorStart (talker/infer/mod.rs:49-60).  Positions are
 * arange(prompt_len) in all three MRoPE rows (session_seed.rs:90-92), so
 * they are implied.  The attention mask is all ones in the reference. */
typedef struct {
  const float *inputs_embeds;   /* [prompt_len][hidden] */
  int prompt_len;
  const float *trailing_text;   /* [trailing_len][hidden], trailing_len > 0 */
  int trailing_len;
  const float *pad_embed;       /* [hidden] */
  q3t_sampling talker_sampling;
  q3t_sampling predictor_sampling;
  int max_new_tokens;           /* > 0 (infer/mod.rs:86-91) */
  int64_t eos_token_id;         /* < 0: None */
  const int64_t *suppress_ids;  /* applied to the first talker token only */
  int num_suppress;
  /* teacher forcing (tests; absent in the reference): >= 0 replaces the
   * first sampled talker token; first_logits (nullable) receives its logits */
  int64_t forced_first_token;
  float *first_logits;          /* [vocab] */
} q3t_session_desc;

typedef struct q3t_session q3t_session;

/* TalkerGenerator::start (infer/mod.rs:69-188): prefill + first sample. */
q3t_status q3t_session_start(q3t_model *model, const q3t_session_desc *desc,
                             q3t_session **out);
/* TalkerGenerator::step (infer/mod.rs:190-299).  *state: 0 = None (already
 * finished), 1 = advanced, 2 = finished.  INVALID_INPUT for "EOS before any
 * audio codec token" (:197-202). */
q3t_status q3t_session_step(q3t_session *s, int *state);
/* Teacher-forced step: codes[num_code_groups] replace the sampled codes of
 * this frame (codes[0] the talker token, codes[1..] the predictor's); the
 * logits computed on the way are written out (nullable):
 * talker_logits [vocab] = the next talker token's logits (after the
 * repetition penalty), predictor_logits [num_code_groups-1][cp_vocab],
 * hidden [hidden] = the talker's new last hidden state. */
q3t_status q3t_session_step_forced(q3t_session *s, const int64_t *codes,
                                   float *talker_logits, float *predictor_logits,
                                   float *hidden, int *state);
/* TalkerGenerator::finalize (infer/mod.rs:301-311): codes [G][T] (pass
 * out = NULL to query T).  INVALID_INPUT if no codec tokens were generated. */
q3t_status q3t_session_codes(q3t_session *s, int64_t *out, int *num_frames);
/* SessionImpl::finish (execution/loaded_model.rs:112-152) without the
 * voice-clone prefix: codec-decodes the generated codes; wave (nullable)
 * receives f32 samples, pcm (nullable) the i16 PCM of Waveform::to_pcm.  An
 * in-context voice-clone session instead decodes [clip codes, generated
 * codes] with q3t_codec_decode and drops the first clip_frames * n /
 * (clip_frames + T) samples, as :115-135 do. */
q3t_status q3t_session_finish(q3t_session *s, float *wave, int16_t *pcm,
                              int64_t capacity, int64_t *num_samples);
/* Isolated talker decode step (decode_step + codec_head, infer/mod.rs:
 * 410-432 and 268-273): inputs_embeds [hidden] at position = cache length;
 * appends K/V; writes logits [vocab] and hidden [hidden] (nullable). */
q3t_status q3t_session_decode_embeds(q3t_session *s, const float *inputs_embeds,
                                     float *logits, float *hidden);
/* Test hook: overwrite the talker KV cache with `len` positions of bf16 K/V,
 * k/v laid out [num_layers][num_kv_heads][len][head_dim] (bit patterns),
 * and set the session's current hidden state [hidden] (nullable). */
q3t_status q3t_session_load_kv(q3t_session *s, const uint16_t *k, const uint16_t *v,
                               int len, const float *hidden);
/* Device time (ms) of the last step / decode call on this session. */
q3t_status q3t_session_last_ms(q3t_session *s, float *ms);
void q3t_session_free(q3t_session *s);

/* Speech-tokenizer encoder of the voice-clone path (codec/config.rs:79-121,
 * built as config.rs:136-346 builds it).  ratios are the tokenizer's
 * upsampling_ratios; the encoder downsamples by them in reverse order. */
typedef struct {
  int audio_channels;            /* 1 */
  int num_filters;               /* 64 */
  int kernel_size;               /* 7 */
  int residual_kernel_size;      /* 3 */
  int last_kernel_size;          /* 3 */
  int compress;                  /* 2 */
  int num_ratios;
  int ratios[8];                 /* [8, 6, 5, 4] */
  int hidden_size;               /* 512 */
  int num_hidden_layers;         /* 8 */
  int num_attention_heads;       /* 8 */
  int num_key_value_heads;       /* 8 */
  int head_dim;                  /* 64 */
  int intermediate_size;         /* 2048 */
  float norm_eps;                /* 1e-5 */
  float rope_theta;              /* 1e4 */
  int codebook_size;             /* 2048 */
  int codebook_dim;              /* 256 (the quantizers' vector width) */
  int num_quantizers;            /* 32 */
  int num_semantic_quantizers;   /* 1 */
  int downsample_factor;         /* 2 */
} q3t_codec_encoder_config;

typedef struct {
  int device;                    /* CUDA device ordinal */
  q3t_codec_encoder_config config;
  const q3t_tensor *tensors;     /* "encoder.encoder.layers.*", "encoder.encoder_transformer.*",
                                    "encoder.downsample.conv.weight", "encoder.quantizer.*" */
  int num_tensors;
} q3t_codec_encoder_desc;

typedef struct q3t_codec_encoder q3t_codec_encoder;

/* Replaces the Burn load of Qwen3TtsAudioCodecEncoder (codec/weights.rs,
 * codec/config.rs:136-346): weights to device memory as f32, the codebook
 * centroids embed_sum / clamp_min(cluster_usage, 1e-6) computed once. */
q3t_status q3t_codec_encoder_load(const q3t_codec_encoder_desc *desc, q3t_codec_encoder **out);
void q3t_codec_encoder_free(q3t_codec_encoder *enc);
/* Frames the encoder emits for num_samples samples (conv.rs:44-64 lengths). */
q3t_status q3t_codec_encoder_frames(const q3t_codec_encoder *enc, int64_t num_samples, int *frames);
/* Qwen3TtsAudioCodecEncoder::encode_reference_prefix (codec/network/
 * encoder.rs:121-136): wave [num_samples] 24 kHz mono f32 -> codes
 * [n_valid][frames] (semantic codebooks first, then acoustic), n_valid in
 * num_semantic_quantizers..num_quantizers; INVALID_INPUT when the frames
 * exceed max_frames. */
q3t_status q3t_codec_encode(q3t_codec_encoder *enc, const float *wave, int64_t num_samples, int n_valid,
                            int64_t *codes, int max_frames, int *frames);
/* Test hook: the hidden the quantizers read, [hidden_size][frames]. */
q3t_status q3t_codec_encoder_hidden(q3t_codec_encoder *enc, const float *wave, int64_t num_samples,
                                    float *hidden, int max_frames, int *frames);

/* ECAPA-TDNN speaker encoder of the voice-clone path (speaker/config.rs:
 * 18-32).  channels[1..3] are the three SE-Res2Net blocks' width (equal,
 * divisible by res2net_scale, <= 4096) and channels[0] must match it. */
typedef struct {
  int mel_dim;                   /* 128 */
  int enc_dim;                   /* 1024 (the x-vector width) */
  int channels[5];               /* [512, 512, 512, 512, 1536] */
  int kernel_sizes[5];           /* [5, 3, 3, 3, 1] */
  int dilations[5];              /* [1, 2, 3, 4, 1] */
  int attention_channels;        /* 128 */
  int res2net_scale;             /* 8 */
  int se_channels;               /* 128 */
  int sample_rate;               /* 24000 */
} q3t_speaker_encoder_config;

typedef struct {
  int device;                    /* CUDA device ordinal */
  q3t_speaker_encoder_config config;
  const q3t_tensor *tensors;     /* "speaker_encoder.*" (speaker/weights.rs:73) */
  int num_tensors;
} q3t_speaker_encoder_desc;

typedef struct q3t_speaker_encoder q3t_speaker_encoder;

/* Replaces the Burn load of the speaker encoder (speaker/weights.rs): conv
 * weights to device memory as f32, the Hann window and mel filterbank built
 * once. */
q3t_status q3t_speaker_encoder_load(const q3t_speaker_encoder_desc *desc, q3t_speaker_encoder **out);
void q3t_speaker_encoder_free(q3t_speaker_encoder *enc);
/* LoadedQwen3TtsSpeakerEncoder::encode_embedding (speaker/infer/mod.rs:
 * 11-20): samples [num_samples] at sample_rate (>= 256 of them) -> the
 * x-vector embedding [enc_dim] f32.  Clips too short for the TDNN blocks'
 * reflect padding are INVALID_INPUT, as the reference's slices reject them. */
q3t_status q3t_speaker_embed(q3t_speaker_encoder *enc, const float *samples, int64_t num_samples,
                             float *embedding);
/* Test hook: the log-mel features [mel_dim][frames] (feature.rs:32-150),
 * frames = (num_samples + 768 - 1024) / 256 + 1; INVALID_INPUT when they
 * exceed max_frames. */
q3t_status q3t_speaker_mel(q3t_speaker_encoder *enc, const float *samples, int64_t num_samples, float *mel,
                           int max_frames, int *frames);

/* Codec decode (decode_waveform, codec/infer/mod.rs:94-111): codes
 * [B][num_quantizers][T] -> wave [B][n] f32 clamped to [-1, 1] and/or pcm
 * [B][n] i16 (to_pcm, :80-90).  *n = samples per item = (((4T-1)*8-1)*5-1)...
 * for the default config (the transposed convs trim k - stride from both
 * ends, conv.rs:19-31).  Codes outside [0, codebook_size) are INVALID_INPUT. */
q3t_status q3t_codec_decode(q3t_model *model, const int64_t *codes, int B, int T,
                            float *wave, int16_t *pcm, int64_t *n);
q3t_status q3t_codec_out_len(const q3t_model *model, int T, int64_t *n);
/* Device time (ms) of the calling thread's last q3t_codec_decode, from the
 * codes on the device to the samples on the device (CUDA events). */
q3t_status q3t_codec_last_ms(float *ms);

/* No reference counterpart.  q3t_codec_decode that allocates nothing, for
 * callers that may not allocate device memory: a real-time audio thread
 * (cudaMalloc can wait for the whole device) or a host framework whose own
 * allocator owns all device memory.  The codes, every intermediate buffer and
 * the samples use one static 48 MiB device array per process: B x T up to
 * about 26 frames (a 24-frame streaming window at B = 1); larger requests are
 * INVALID_INPUT with the needed size in q3t_last_error().  Runs on `stream`
 * (a cudaStream_t; NULL is the default stream) and blocks: it synchronises
 * `stream` and returns only when wave / pcm (host buffers, nullable) hold the
 * result.  A convolution timeout is read from a word inside the array on
 * `stream` (other decodes running at the same time neither see nor clear
 * it).  The first call on each device looks up the array's address
 * (cudaGetSymbolAddress) with the model's device current; make that first
 * call before any stream capture.  The calling thread's current device is
 * the same on return as on entry.  Calls that overlap in time on one device
 * share the array and race: serialise them. */
q3t_status q3t_codec_decode_static(q3t_model *model, const int64_t *codes, int B, int T,
                                   float *wave, int16_t *pcm, int64_t *n, void *stream);

/* Prompt text projection: project_text_ids
 * (tts_qwen3_tts/src/execution/compiler/session_seed.rs:668-679) =
 * Qwen3TtsTalkerResizeMlp (talker/network/mlp.rs:36-40, config.rs:200-209)
 * over the text embedding: out[i] = linear_fc2(silu(linear_fc1(
 * text_embedding[ids[i]]))) with biases, [n][hidden] f32 rows holding bf16
 * values (the model dtype).  q3t_session_seed assembles a whole prompt seed
 * from these rows on the device.  Needs the optional tensors
 * talker.model.text_embedding.weight [text_vocab][text_hidden] and
 * talker.text_projection.linear_fc{1,2}.{weight,bias} in q3t_model_load;
 * INVALID_INPUT without them or for ids outside [0, text_vocab). */
q3t_status q3t_text_project(q3t_model *model, const int64_t *ids, int n, float *out);
/* text_vocab / text_hidden of the loaded text projection (0 if absent). */
q3t_status q3t_text_dims(const q3t_model *model, int *text_vocab, int *text_hidden);

/* Control token ids of a profile (the reference's ProfileControlIds). */
typedef struct {
  int64_t tts_bos_token_id, tts_eos_token_id, tts_pad_token_id; /* text vocabulary */
  const int64_t *codec_prefix_ids;                               /* talker codec vocabulary */
  int n_codec_prefix;                                            /* >= 2 */
  int64_t codec_pad_id, codec_bos_id;                            /* talker codec vocabulary */
} q3t_seed_controls;

/* The prompt seed of the non-voice-clone recipes, build_non_streaming_seed
 * (session_seed.rs:151-215), computed on the device: with P(ids) the text
 * projection above and E(id) the talker codec embedding,
 *   inputs_embeds = [ P(leading_ids)                      (instruct, nullable)
 *                     P(text_ids[0..3])                   (role)
 *                     P(pad) x (n_codec_prefix - 2), P(bos)  + E(codec_prefix_ids[0..n-1])
 *                     P(text_ids[3..n_text-5])             + E(codec_pad_id)
 *                     P(eos)                               + E(codec_pad_id)
 *                     P(pad)                               + E(codec_bos_id) ]
 * as [rows][hidden] f32 rows holding bf16 values (sums rounded as the
 * reference's bf16 adds), rows = n_leading + 3 + (n_codec_prefix - 1) +
 * (n_text - 8) + 2; pad_embed [hidden] = P(tts_pad), which is also the
 * trailing text hidden of these recipes.  inputs_embeds == NULL only reports
 * *rows; max_rows < rows or n_text < 8, n_codec_prefix < 2 or an id outside
 * its vocabulary is INVALID_INPUT.  The voice-clone recipes' seeds are
 * q3t_session_seed_voice_clone. */
q3t_status q3t_session_seed(q3t_model *model, const int64_t *text_ids, int n_text, const int64_t *leading_ids,
                            int n_leading, const q3t_seed_controls *controls, float *inputs_embeds, int max_rows,
                            int *rows, float *pad_embed);

/* The prompt seed of the voice-clone recipes, build_voice_clone_seed
 * (session_seed.rs:248-322), on the device, from the x-vector of
 * q3t_speaker_embed (speaker [hidden], cast to bf16) and, for the in-context
 * recipe, the reference clip's codes of q3t_codec_encode (ref_codes
 * [num_code_groups][ref_frames], group 0 in the talker codec vocabulary,
 * the others in the predictor's) with its text ids (3 role ids, body, 2
 * trailing ids).  With P and E as in q3t_session_seed and n =
 * n_codec_prefix:
 *   inputs_embeds = [ P(text_ids[0..3])
 *                     P(pad) + E(codec_prefix_ids[i]), i < n - 2
 *                     P(pad) + speaker,  P(bos) + E(codec_pad_id)
 *                     then, ref_text_ids == NULL (x-vector recipe):
 *                       P(body[0]) + E(codec_bos_id)           (if any body)
 *                     else (build_voice_clone_icl_seed, :324-396), with
 *                     text = P(ref body + body + eos), codec = [E(codec_bos_id),
 *                     frame t: sum over groups g of Emb_g(ref_codes[g][t])]:
 *                       text[i] (P(pad) past its end) + codec[i], i < 1 + ref_frames ]
 * trailing_text = P(body[1..]), P(eos) (x-vector), or the text rows past
 * the codec rows, or P(pad) when there are none (in-context); every sum is
 * rounded to bf16 as the reference's bf16 adds, the frame sums group by
 * group.  inputs_embeds == NULL only reports *rows and *trailing_rows;
 * outputs too small, ids outside their vocabularies, n_text < 8,
 * n_ref_text < 5, n_codec_prefix < 2 or an in-context call without codes
 * are INVALID_INPUT. */
q3t_status q3t_session_seed_voice_clone(q3t_model *model, const int64_t *text_ids, int n_text, const float *speaker,
                                        const int64_t *ref_text_ids, int n_ref_text, const int64_t *ref_codes,
                                        int ref_frames, const q3t_seed_controls *controls, float *inputs_embeds,
                                        int max_rows, int *rows, float *trailing_text, int max_trailing,
                                        int *trailing_rows, float *pad_embed);

/* ------------------------------- file IO --------------------------------- */
/* A memory-mapped .safetensors checkpoint whose float tensors (F32 and BF16
 * in place, F16 widened to F32; integer tensors skipped) are listed as
 * q3t_tensor entries by their checkpoint names, ready for q3t_model_load
 * (concatenate the lists of the talker and speech-tokenizer files).  Replaces
 * the SafetensorsStore reads of talker/weights.rs:52-66 and
 * codec/weights.rs:77-81 (driven by loading/runtime.rs:131-156); the key
 * remaps there are Burn module renames, except the codec's legacy
 * `._codebook.` spelling, which q3t_model_load accepts as well as
 * `.codebook.`.  The list stays valid until q3t_tensor_set_free. */
typedef struct q3t_tensor_set q3t_tensor_set;
q3t_status q3t_safetensors_open(const char *path, q3t_tensor_set **out);
q3t_status q3t_tensor_set_list(const q3t_tensor_set *set, const q3t_tensor **tensors, int *num_tensors);
void q3t_tensor_set_free(q3t_tensor_set *set);

/* PcmAudio::write_wav (tts_infer/src/audio.rs:12-49): the RIFF/WAVE image of
 * 16-bit integer PCM (44-byte header, format 1, little-endian samples) into
 * out[capacity]; *size = 44 + 2 * num_samples (out = NULL: size query). */
q3t_status q3t_wav_write(const int16_t *pcm, int64_t num_samples, int sample_rate, int channels, uint8_t *out,
                         int64_t capacity, int64_t *size);

/* decode_reference_audio (execution/reference_audio.rs:17-50, 76-121): a
 * RIFF/WAVE image (integer PCM 16 / 24 / 32-bit, or 32-bit float; the
 * extensible header resolved to its sub-format) -> mono f32 samples, each
 * frame the mean of its channels (integer samples / 2^(bits-1), clamped to
 * [-1, 1]); *n_samples = frames, *sample_rate (nullable) the file's rate
 * (samples = NULL: size query).  Other formats, zero channels, no samples
 * or no complete frame are INVALID_INPUT.  Host code, no GPU. */
q3t_status q3t_wav_read(const uint8_t *bytes, int64_t n_bytes, float *samples, int64_t max_samples,
                        int64_t *n_samples, uint32_t *sample_rate);
/* resample_linear (reference_audio.rs:123-156): linear interpolation from
 * source_rate to target_rate, (n * target + source / 2) / source output
 * samples (at least 1); none for n = 0 or a zero rate, a copy for equal
 * rates or one sample (out = NULL: size query).  Host code, no GPU. */
q3t_status q3t_resample_linear(const float *in, int64_t n, uint32_t source_rate, uint32_t target_rate, float *out,
                               int64_t max_out, int64_t *n_out);

/* ------------------------ ragged continuous batching --------------------- */
typedef struct {
  int max_active;            /* <= model max_active */
  int codec_mode;            /* 0: none, 1: full-sequence decode at retire
                                (reference semantics), 2: chunked streaming */
  int chunk_frames;          /* codec_mode 2: frames emitted per chunk */
  int left_context;          /* codec_mode 2: frames of left context per chunk */
  int keep_output;           /* 1: keep codes/PCM for q3t_batch_take */
} q3t_batch_desc;

typedef struct {
  int active;                /* requests in the decode frame (first token known) */
  int admitted;              /* requests admitted into a slot this step (their prompts run in
                                chunks inside this and the following talker passes) */
  int retired;               /* requests finished this step */
  int64_t frames;            /* frames generated this step */
  int64_t samples;           /* PCM samples emitted this step */
  float device_ms;           /* device time of this step (CUDA events) */
  int64_t kv_tokens;         /* sum over the decode tokens of their KV length */
  int64_t h2d_bytes;         /* host -> device bytes copied during this step */
  int64_t d2h_bytes;         /* device -> host bytes copied during this step */
  float predictor_ms;        /* device time of the frame's code-predictor loop (15 codebooks) */
  float talker_ms;           /* device time of the frame's talker pass (decode tokens and
                                prompt-chunk tokens), codec_head and sampling */
  int prefill_tokens;        /* prompt tokens that ran in this step's talker pass */
  int first_tokens;          /* prompts completed this step (their first token sampled) */
} q3t_step_stats;

typedef struct q3t_batch q3t_batch;

q3t_status q3t_batch_create(q3t_model *model, const q3t_batch_desc *desc, q3t_batch **out);
/* Queue a request; its inputs are copied to device memory now, so a later
 * step finds them resident.  forced_codes (nullable) [max_new_tokens][G]
 * teacher-forces every frame (then EOS is ignored and the request runs
 * max_new_tokens). */
q3t_status q3t_batch_submit(q3t_batch *b, const q3t_session_desc *req,
                            const int64_t *forced_codes, int64_t *request_id);
/* One scheduler iteration: admit queued requests into free slots, one decode
 * frame for every request whose first token is known, with prompt tokens of
 * admitted requests packed into the same talker pass (up to 128 tokens in
 * all; a prompt's first token is sampled in the step its last chunk runs,
 * and it decodes from the next step on), retire finished ones (codec decode
 * per codec_mode). */
q3t_status q3t_batch_step(q3t_batch *b, q3t_step_stats *stats);
/* state: 0 queued, 1 active, 2 finished, 3 failed */
q3t_status q3t_batch_poll(q3t_batch *b, int64_t request_id, int *state, int64_t *frames,
                          int64_t *samples);
/* Copy out (and release) a finished request's codes [G][T], the tokens the
 * sampler picked before teacher forcing replaced them (sampled [G][T], for
 * argmax-agreement checks; nullable) and its samples (codec_mode 1/2). */
q3t_status q3t_batch_take(q3t_batch *b, int64_t request_id, int64_t *codes, int32_t *sampled,
                          int max_frames, float *wave, int64_t max_samples);
q3t_status q3t_batch_pending(q3t_batch *b, int *queued, int *active);
/* Test hook (the per-frame logits of TalkerGenerator::step, infer/mod.rs:
 * 249-283, for one request of a batch): copies the logits of request_id's
 * token in the last decode frame: talker_logits [vocab] (after the repetition
 * penalty) and predictor_logits [num_code_groups - 1][cp_vocab] (nullable
 * each).  INVALID_INPUT if the request was not in that frame.  Valid until
 * the next q3t_batch_step. */
q3t_status q3t_batch_logits(q3t_batch *b, int64_t request_id, float *talker_logits, float *predictor_logits);
/* The CUDA stream (cudaStream_t) the batch's device work is ordered on, for
 * callers that time steps with their own CUDA events.  With codec_mode 2 a
 * step's chunk decodes run on a second, lower-priority stream, overlapped
 * with the next step's frame; the next q3t_batch_step joins them into this
 * stream and counts their samples (a step in which a request finishes joins
 * at once). */
q3t_status q3t_batch_stream(q3t_batch *b, void **stream);
void q3t_batch_free(q3t_batch *b);

/* Test hook of sample_token (tts_qwen3_tts/src/model/talker/infer/sampling.rs:
 * 33-90): runs the device sampler of the decode frames on one row of logits
 * [vocab] (vocab <= 4096) with the suppress list applied, using the given
 * uniform draw u in [0, 1) for the categorical step instead of the on-device
 * counter hash, so a test can compare it with a host restatement fed the
 * same u.  *token receives the pick; kept (nullable) [vocab] receives 1 for
 * every token that is still a candidate after suppress, top-k and top-p. */
q3t_status q3t_sample_logits(q3t_model *model, const float *logits, int vocab, const q3t_sampling *sampling,
                             const int64_t *suppress_ids, int num_suppress, double u, int64_t *token,
                             uint8_t *kept);

/* ------------------------------- misc ----------------------------------- */
/* Struct layout as this library was compiled (no reference counterpart: the
 * reference is one Rust crate, so its structs need no cross-language check).
 * A binding that re-declares the structs above (a Rust `#[repr(C)]` -sys
 * crate, a ctypes mirror) compares its own sizes and offsets with these at
 * start-up or in its tests.  `name` is the C struct name ("q3t_step_stats");
 * fields are numbered in declaration order.  INVALID_INPUT for an unknown
 * struct or an index outside [0, num_fields). */
q3t_status q3t_abi_struct(const char *name, size_t *size, size_t *align, int *num_fields);
q3t_status q3t_abi_field(const char *name, int index, const char **field, size_t *offset,
                         size_t *size);
const char *q3t_last_error(void);
const char *q3t_version(void);
/* Number of kernel launches this thread has issued into the library's
 * streams since load (graph replays count their kernel nodes). */
int64_t q3t_kernel_launches(void);

#ifdef __cplusplus
}
#endif
#endif /* Q3T_H */

// Layout table of the public structs of include/q3t.h (q3t_abi_struct /
// q3t_abi_field): sizeof, alignof and every field's offset and size as this
// compiler laid them out, so a binding in another language (the Rust -sys
// crate, the Python ctypes mirror) can check its own declarations against
// the library it links instead of trusting a copy of the header.
#include <cstddef>
#include <cstring>

#include "../../include/q3t.h"
#include "engine.h"

namespace {

struct FieldRow {
  const char *name;
  size_t offset, size;
};
struct StructRow {
  const char *name;
  size_t size, align;
  const FieldRow *fields;
  int n;
};

#define Q3T_F(S, f) {#f, offsetof(S, f), sizeof(((S *)nullptr)->f)}

const FieldRow k_lm[] = {
    Q3T_F(q3t_lm_config, hidden_size),       Q3T_F(q3t_lm_config, intermediate_size),
    Q3T_F(q3t_lm_config, num_hidden_layers), Q3T_F(q3t_lm_config, num_attention_heads),
    Q3T_F(q3t_lm_config, num_key_value_heads), Q3T_F(q3t_lm_config, head_dim),
    Q3T_F(q3t_lm_config, vocab_size),        Q3T_F(q3t_lm_config, rms_norm_eps),
    Q3T_F(q3t_lm_config, rope_theta),
};
const FieldRow k_talker[] = {
    Q3T_F(q3t_talker_config, talker),
    Q3T_F(q3t_talker_config, predictor),
    Q3T_F(q3t_talker_config, num_code_groups),
};
const FieldRow k_codec[] = {
    Q3T_F(q3t_codec_config, num_quantizers),     Q3T_F(q3t_codec_config, num_semantic_quantizers),
    Q3T_F(q3t_codec_config, codebook_size),      Q3T_F(q3t_codec_config, codebook_dim),
    Q3T_F(q3t_codec_config, latent_dim),         Q3T_F(q3t_codec_config, decoder_dim),
    Q3T_F(q3t_codec_config, hidden_size),        Q3T_F(q3t_codec_config, intermediate_size),
    Q3T_F(q3t_codec_config, num_hidden_layers),  Q3T_F(q3t_codec_config, num_attention_heads),
    Q3T_F(q3t_codec_config, num_key_value_heads), Q3T_F(q3t_codec_config, head_dim),
    Q3T_F(q3t_codec_config, rms_norm_eps),       Q3T_F(q3t_codec_config, rope_theta),
    Q3T_F(q3t_codec_config, num_upsampling_ratios), Q3T_F(q3t_codec_config, upsampling_ratios),
    Q3T_F(q3t_codec_config, num_upsample_rates), Q3T_F(q3t_codec_config, upsample_rates),
    Q3T_F(q3t_codec_config, output_sample_rate),
};
const FieldRow k_tensor[] = {
    Q3T_F(q3t_tensor, name), Q3T_F(q3t_tensor, dtype), Q3T_F(q3t_tensor, ndim),
    Q3T_F(q3t_tensor, shape), Q3T_F(q3t_tensor, data),
};
const FieldRow k_model_desc[] = {
    Q3T_F(q3t_model_desc, device),      Q3T_F(q3t_model_desc, talker),   Q3T_F(q3t_model_desc, has_talker),
    Q3T_F(q3t_model_desc, codec),       Q3T_F(q3t_model_desc, has_codec), Q3T_F(q3t_model_desc, tensors),
    Q3T_F(q3t_model_desc, num_tensors), Q3T_F(q3t_model_desc, kv_pages), Q3T_F(q3t_model_desc, max_active),
};
const FieldRow k_sampling[] = {
    Q3T_F(q3t_sampling, do_sample), Q3T_F(q3t_sampling, temperature),        Q3T_F(q3t_sampling, top_k),
    Q3T_F(q3t_sampling, top_p),     Q3T_F(q3t_sampling, repetition_penalty), Q3T_F(q3t_sampling, seed),
};
const FieldRow k_session_desc[] = {
    Q3T_F(q3t_session_desc, inputs_embeds),      Q3T_F(q3t_session_desc, prompt_len),
    Q3T_F(q3t_session_desc, trailing_text),      Q3T_F(q3t_session_desc, trailing_len),
    Q3T_F(q3t_session_desc, pad_embed),          Q3T_F(q3t_session_desc, talker_sampling),
    Q3T_F(q3t_session_desc, predictor_sampling), Q3T_F(q3t_session_desc, max_new_tokens),
    Q3T_F(q3t_session_desc, eos_token_id),       Q3T_F(q3t_session_desc, suppress_ids),
    Q3T_F(q3t_session_desc, num_suppress),       Q3T_F(q3t_session_desc, forced_first_token),
    Q3T_F(q3t_session_desc, first_logits),
};
const FieldRow k_seed_controls[] = {
    Q3T_F(q3t_seed_controls, tts_bos_token_id), Q3T_F(q3t_seed_controls, tts_eos_token_id),
    Q3T_F(q3t_seed_controls, tts_pad_token_id), Q3T_F(q3t_seed_controls, codec_prefix_ids),
    Q3T_F(q3t_seed_controls, n_codec_prefix),   Q3T_F(q3t_seed_controls, codec_pad_id),
    Q3T_F(q3t_seed_controls, codec_bos_id),
};
const FieldRow k_batch_desc[] = {
    Q3T_F(q3t_batch_desc, max_active),   Q3T_F(q3t_batch_desc, codec_mode), Q3T_F(q3t_batch_desc, chunk_frames),
    Q3T_F(q3t_batch_desc, left_context), Q3T_F(q3t_batch_desc, keep_output),
};
const FieldRow k_step_stats[] = {
    Q3T_F(q3t_step_stats, active),    Q3T_F(q3t_step_stats, admitted),     Q3T_F(q3t_step_stats, retired),
    Q3T_F(q3t_step_stats, frames),    Q3T_F(q3t_step_stats, samples),      Q3T_F(q3t_step_stats, device_ms),
    Q3T_F(q3t_step_stats, kv_tokens), Q3T_F(q3t_step_stats, h2d_bytes),    Q3T_F(q3t_step_stats, d2h_bytes),
    Q3T_F(q3t_step_stats, predictor_ms), Q3T_F(q3t_step_stats, talker_ms), Q3T_F(q3t_step_stats, prefill_tokens),
    Q3T_F(q3t_step_stats, first_tokens),
};
const FieldRow k_enc_config[] = {
    Q3T_F(q3t_codec_encoder_config, audio_channels),      Q3T_F(q3t_codec_encoder_config, num_filters),
    Q3T_F(q3t_codec_encoder_config, kernel_size),         Q3T_F(q3t_codec_encoder_config, residual_kernel_size),
    Q3T_F(q3t_codec_encoder_config, last_kernel_size),    Q3T_F(q3t_codec_encoder_config, compress),
    Q3T_F(q3t_codec_encoder_config, num_ratios),          Q3T_F(q3t_codec_encoder_config, ratios),
    Q3T_F(q3t_codec_encoder_config, hidden_size),         Q3T_F(q3t_codec_encoder_config, num_hidden_layers),
    Q3T_F(q3t_codec_encoder_config, num_attention_heads), Q3T_F(q3t_codec_encoder_config, num_key_value_heads),
    Q3T_F(q3t_codec_encoder_config, head_dim),            Q3T_F(q3t_codec_encoder_config, intermediate_size),
    Q3T_F(q3t_codec_encoder_config, norm_eps),            Q3T_F(q3t_codec_encoder_config, rope_theta),
    Q3T_F(q3t_codec_encoder_config, codebook_size),       Q3T_F(q3t_codec_encoder_config, codebook_dim),
    Q3T_F(q3t_codec_encoder_config, num_quantizers),      Q3T_F(q3t_codec_encoder_config, num_semantic_quantizers),
    Q3T_F(q3t_codec_encoder_config, downsample_factor),
};
const FieldRow k_enc_desc[] = {
    Q3T_F(q3t_codec_encoder_desc, device),  Q3T_F(q3t_codec_encoder_desc, config),
    Q3T_F(q3t_codec_encoder_desc, tensors), Q3T_F(q3t_codec_encoder_desc, num_tensors),
};
const FieldRow k_spk_config[] = {
    Q3T_F(q3t_speaker_encoder_config, mel_dim),       Q3T_F(q3t_speaker_encoder_config, enc_dim),
    Q3T_F(q3t_speaker_encoder_config, channels),      Q3T_F(q3t_speaker_encoder_config, kernel_sizes),
    Q3T_F(q3t_speaker_encoder_config, dilations),     Q3T_F(q3t_speaker_encoder_config, attention_channels),
    Q3T_F(q3t_speaker_encoder_config, res2net_scale), Q3T_F(q3t_speaker_encoder_config, se_channels),
    Q3T_F(q3t_speaker_encoder_config, sample_rate),
};
const FieldRow k_spk_desc[] = {
    Q3T_F(q3t_speaker_encoder_desc, device),  Q3T_F(q3t_speaker_encoder_desc, config),
    Q3T_F(q3t_speaker_encoder_desc, tensors), Q3T_F(q3t_speaker_encoder_desc, num_tensors),
};
#undef Q3T_F

#define Q3T_S(S, table) {#S, sizeof(S), alignof(S), table, (int)(sizeof(table) / sizeof(table[0]))}
const StructRow k_structs[] = {
    Q3T_S(q3t_lm_config, k_lm),
    Q3T_S(q3t_talker_config, k_talker),
    Q3T_S(q3t_codec_config, k_codec),
    Q3T_S(q3t_tensor, k_tensor),
    Q3T_S(q3t_model_desc, k_model_desc),
    Q3T_S(q3t_sampling, k_sampling),
    Q3T_S(q3t_session_desc, k_session_desc),
    Q3T_S(q3t_seed_controls, k_seed_controls),
    Q3T_S(q3t_batch_desc, k_batch_desc),
    Q3T_S(q3t_step_stats, k_step_stats),
    Q3T_S(q3t_codec_encoder_config, k_enc_config),
    Q3T_S(q3t_codec_encoder_desc, k_enc_desc),
    Q3T_S(q3t_speaker_encoder_config, k_spk_config),
    Q3T_S(q3t_speaker_encoder_desc, k_spk_desc),
};
#undef Q3T_S

const StructRow *find_struct(const char *name) {
  if (!name) return nullptr;
  for (const StructRow &s : k_structs)
    if (strcmp(s.name, name) == 0) return &s;
  return nullptr;
}

}  // namespace

extern "C" q3t_status q3t_abi_struct(const char *name, size_t *size, size_t *align, int *num_fields) {
  const StructRow *s = find_struct(name);
  if (!s) {
    q3t::set_error("q3t_abi_struct: unknown struct '%s'", name ? name : "(null)");
    return Q3T_INVALID_INPUT;
  }
  if (size) *size = s->size;
  if (align) *align = s->align;
  if (num_fields) *num_fields = s->n;
  return Q3T_OK;
}

extern "C" q3t_status q3t_abi_field(const char *name, int index, const char **field, size_t *offset,
                                    size_t *size) {
  const StructRow *s = find_struct(name);
  if (!s || index < 0 || index >= s->n) {
    q3t::set_error("q3t_abi_field: no field %d in struct '%s'", index, name ? name : "(null)");
    return Q3T_INVALID_INPUT;
  }
  if (field) *field = s->fields[index].name;
  if (offset) *offset = s->fields[index].offset;
  if (size) *size = s->fields[index].size;
  return Q3T_OK;
}

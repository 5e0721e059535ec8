// Speech-tokenizer decoder (codec) entry points used by the engine.
#pragma once
#include <vector>

#include "engine.h"

namespace q3t {

CodecModel *codec_load(q3t_model *m, const q3t_model_desc *desc, cudaStream_t st);
void codec_free(CodecModel *c);
void codec_out_len(const CodecModel *c, int T, int64_t *n);
// codes [B][n_q][T] (host) -> wave / pcm [B][n] (host, nullable)
void codec_decode_host_codes(q3t_model *m, const int64_t *codes, int B, int T, float *wave, int16_t *pcm,
                             cudaStream_t st);
// chunked streaming decode inside a batch (codec_mode 2)
void codec_stream_init(q3t_model *m, q3t_batch *b);
void codec_stream_step(q3t_model *m, q3t_batch *b, const std::vector<Req *> &act, int64_t *samples);
// completes the streaming codec work still in flight; samples (nullable) counts what it emitted
void codec_stream_join(q3t_batch *b, int64_t *samples);
// launches the decode of the windows the last codec_stream_step gathered (no-op if none)
void codec_stream_launch(q3t_batch *b);
void codec_stream_free(q3t_batch *b);

}  // namespace q3t

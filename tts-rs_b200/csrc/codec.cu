// Speech-tokenizer decoder (placeholder until the codec kernels land).
#include "codec.cuh"

namespace q3t {

struct CodecModel {
  int dummy;
};

CodecModel *codec_load(q3t_model *, const q3t_model_desc *, cudaStream_t) {
  FAIL(Q3T_INVALID_INPUT, "codec decoder not available in this build");
}
void codec_free(CodecModel *c) { delete c; }
void codec_out_len(const CodecModel *, int, int64_t *n) { *n = 0; }
void codec_decode_host_codes(q3t_model *, const int64_t *, int, int, float *, int16_t *, cudaStream_t) {
  FAIL(Q3T_INVALID_INPUT, "codec decoder not available in this build");
}
void codec_stream_init(q3t_model *, q3t_batch *) {}
void codec_stream_step(q3t_model *, q3t_batch *, const std::vector<Req *> &, int64_t *) {}
void codec_stream_free(q3t_batch *) {}

}  // namespace q3t

using namespace q3t;

extern "C" q3t_status q3t_codec_out_len(const q3t_model *m, int T, int64_t *n) {
  if (!m || !n || T <= 0 || !m->has_codec || !m->codec) {
    set_error("q3t_codec_out_len: model has no codec or T <= 0");
    return Q3T_INVALID_INPUT;
  }
  codec_out_len(m->codec, T, n);
  return Q3T_OK;
}

extern "C" q3t_status q3t_codec_decode(q3t_model *, const int64_t *, int, int, float *, int16_t *, int64_t *) {
  set_error("codec decoder not available in this build");
  return Q3T_INVALID_INPUT;
}

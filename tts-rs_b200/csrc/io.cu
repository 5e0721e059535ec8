// Host-side model and audio IO of the C ABI:
//  - a safetensors reader that hands checkpoint tensors to q3t_model_load
//    (the reads of burn_store's SafetensorsStore in
//    tts_qwen3_tts/src/model/talker/weights.rs:52-66 and
//    codec/weights.rs:77-81, driven by loading/runtime.rs:131-156);
//  - the WAV image of 16-bit PCM (PcmAudio::write_wav,
//    tts_infer/src/audio.rs:12-49, which writes hound's canonical RIFF
//    layout for integer 16-bit samples);
//  - the voice-clone reference audio in front of the encoders: a WAV image
//    decoded to mono f32 (decode_reference_audio,
//    tts_qwen3_tts/src/execution/reference_audio.rs:17-50, 76-121) and the
//    linear resampler (resample_linear, :123-156).
//
// safetensors layout: u64 little-endian header length N, N bytes of JSON
// {name: {"dtype", "shape", "data_offsets": [begin, end]}, "__metadata__":
// {...}}, then the raw little-endian tensor bytes (offsets relative to the
// end of the header).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstring>
#include <string>
#include <vector>

#include "engine.h"

struct q3t_tensor_set {
  void *map = nullptr;
  size_t map_len = 0;
  std::vector<std::string> names;
  std::vector<q3t_tensor> tensors;
  std::vector<std::vector<float>> converted;  // F16 tensors widened to f32
};

namespace q3t {
namespace {

// Minimal JSON reader for the safetensors header: objects, arrays, strings,
// integers and the literals; anything malformed throws.
struct Json {
  const char *p, *end;
  [[noreturn]] void bad(const char *what) { FAIL(Q3T_RUNTIME_LOAD, "safetensors header: %s", what); }
  void ws() {
    while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) p++;
  }
  bool eat(char c) {
    ws();
    if (p < end && *p == c) {
      p++;
      return true;
    }
    return false;
  }
  void need(char c) {
    if (!eat(c)) bad("unexpected character");
  }
  std::string str() {
    need('"');
    std::string s;
    while (p < end && *p != '"') {
      if (*p == '\\') {
        if (++p >= end) bad("bad escape");
        switch (*p) {
          case 'n': s += '\n'; break;
          case 't': s += '\t'; break;
          case 'r': s += '\r'; break;
          case 'b': s += '\b'; break;
          case 'f': s += '\f'; break;
          case 'u': {  // keep ASCII, replace the rest (tensor names are ASCII)
            if (end - p < 5) bad("bad \\u escape");
            const unsigned v = (unsigned)strtoul(std::string(p + 1, p + 5).c_str(), nullptr, 16);
            s += v < 128 ? (char)v : '?';
            p += 4;
            break;
          }
          default: s += *p; break;
        }
        p++;
      } else {
        s += *p++;
      }
    }
    if (p >= end) bad("unterminated string");
    p++;
    return s;
  }
  long long integer() {  // parsed from a bounded copy: the header is not NUL-terminated
    ws();
    char buf[24];
    size_t k = 0;
    while (p + k < end && k < sizeof buf - 1 && (p[k] == '-' || (p[k] >= '0' && p[k] <= '9'))) {
      buf[k] = p[k];
      k++;
    }
    buf[k] = 0;
    char *e = nullptr;
    errno = 0;
    const long long v = strtoll(buf, &e, 10);
    if (e == buf || errno == ERANGE || (size_t)(e - buf) != k) bad("number expected");
    p += k;
    return v;
  }
  void skip() {  // any value
    ws();
    if (p >= end) bad("value expected");
    if (*p == '"') {
      str();
    } else if (*p == '{') {
      p++;
      if (eat('}')) return;
      do {
        str();
        need(':');
        skip();
      } while (eat(','));
      need('}');
    } else if (*p == '[') {
      p++;
      if (eat(']')) return;
      do skip();
      while (eat(','));
      need(']');
    } else {
      while (p < end && *p != ',' && *p != '}' && *p != ']' && *p != ' ' && *p != '\n') p++;
    }
  }
};

float half_to_float(uint16_t h) {
  const uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 31, m = h & 1023;
  uint32_t u;
  if (e == 0) {
    if (m == 0) {
      u = s;
    } else {  // subnormal: renormalise
      int k = -1;
      uint32_t mm = m;
      do {
        k++;
        mm <<= 1;
      } while (!(mm & 1024));
      u = s | ((uint32_t)(127 - 15 - k) << 23) | ((mm & 1023) << 13);
    }
  } else if (e == 31) {
    u = s | 0x7f800000u | (m << 13);
  } else {
    u = s | ((e + 127 - 15) << 23) | (m << 13);
  }
  float f;
  memcpy(&f, &u, 4);
  return f;
}

void parse(q3t_tensor_set *s, const unsigned char *base, size_t len) {
  if (len < 8) FAIL(Q3T_RUNTIME_LOAD, "safetensors: file shorter than its header length");
  uint64_t n = 0;
  for (int i = 0; i < 8; i++) n |= (uint64_t)base[i] << (8 * i);
  if (n > len - 8) FAIL(Q3T_RUNTIME_LOAD, "safetensors: header length %llu beyond the file", (unsigned long long)n);
  const unsigned char *data = base + 8 + n;
  const size_t data_len = len - 8 - n;
  Json j{reinterpret_cast<const char *>(base + 8), reinterpret_cast<const char *>(base + 8 + n)};
  j.need('{');
  if (j.eat('}')) return;
  struct Entry {
    std::string name, dtype;
    std::vector<long long> shape;
    long long b = -1, e = -1;
  };
  std::vector<Entry> entries;
  do {
    Entry en;
    en.name = j.str();
    j.need(':');
    if (en.name == "__metadata__") {
      j.skip();
      continue;
    }
    j.need('{');
    if (!j.eat('}')) {
      do {
        const std::string key = j.str();
        j.need(':');
        if (key == "dtype") {
          en.dtype = j.str();
        } else if (key == "shape") {
          j.need('[');
          if (!j.eat(']')) {
            do en.shape.push_back(j.integer());
            while (j.eat(','));
            j.need(']');
          }
        } else if (key == "data_offsets") {
          j.need('[');
          en.b = j.integer();
          j.need(',');
          en.e = j.integer();
          j.need(']');
        } else {
          j.skip();
        }
      } while (j.eat(','));
      j.need('}');
    }
    entries.push_back(en);
  } while (j.eat(','));
  j.need('}');
  for (const Entry &en : entries) {
    int esz = 0, dtype = -1;
    if (en.dtype == "F32") esz = 4, dtype = Q3T_F32;
    else if (en.dtype == "BF16") esz = 2, dtype = Q3T_BF16;
    else if (en.dtype == "F16") esz = 2, dtype = Q3T_F32;  // widened below
    else continue;  // integer / other tensors are not weights of this path
    if (en.shape.size() > 4) FAIL(Q3T_RUNTIME_LOAD, "safetensors: tensor %s has rank > 4", en.name.c_str());
    long long numel = 1;
    for (long long d : en.shape) {
      if (d < 0) FAIL(Q3T_RUNTIME_LOAD, "safetensors: tensor %s has a negative dimension", en.name.c_str());
      if (d > 0 && numel > (1LL << 40) / d)
        FAIL(Q3T_RUNTIME_LOAD, "safetensors: tensor %s has more than 2^40 elements", en.name.c_str());
      numel *= d;
    }
    if (en.b < 0 || en.e < en.b || (size_t)en.e > data_len || en.e - en.b != numel * esz)
      FAIL(Q3T_RUNTIME_LOAD, "safetensors: tensor %s has bad data offsets", en.name.c_str());
    q3t_tensor t{};
    t.dtype = dtype;
    t.ndim = (int)en.shape.size();
    for (int i = 0; i < t.ndim; i++) t.shape[i] = en.shape[i];
    const unsigned char *src = data + en.b;
    if (en.dtype == "F16") {
      s->converted.emplace_back((size_t)numel);
      std::vector<float> &f = s->converted.back();
      for (long long i = 0; i < numel; i++) {
        uint16_t h;
        memcpy(&h, src + 2 * i, 2);
        f[i] = half_to_float(h);
      }
      t.data = f.data();
    } else {
      t.data = src;
    }
    s->names.push_back(en.name);
    s->tensors.push_back(t);
  }
  for (size_t i = 0; i < s->tensors.size(); i++) s->tensors[i].name = s->names[i].c_str();
}

template <class F>
q3t_status io_guard(F &&f) {
  try {
    f();
    return Q3T_OK;
  } catch (const Status &st) {
    return st.code;
  } catch (const std::bad_alloc &) {
    set_error("host allocation failed");
    return Q3T_RUNTIME_LOAD;
  }
}

void put_u32(unsigned char *p, uint32_t v) {
  for (int i = 0; i < 4; i++) p[i] = (unsigned char)(v >> (8 * i));
}
void put_u16(unsigned char *p, uint16_t v) {
  p[0] = (unsigned char)v;
  p[1] = (unsigned char)(v >> 8);
}
uint32_t get_u32(const unsigned char *p) {
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
uint16_t get_u16(const unsigned char *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

// The fields of a WAVE file that the decoder reads (hound's WavSpec plus
// where the sample bytes are).
struct WavInfo {
  int format = 0;  // 1 integer PCM, 3 IEEE float (WAVE_FORMAT_EXTENSIBLE resolved to its sub-format)
  int channels = 0, bits = 0, block_align = 0;
  uint32_t rate = 0;
  const unsigned char *data = nullptr;
  uint64_t data_len = 0;
};

// RIFF/WAVE chunk walk: "fmt " (16 bytes, or 40 with the extensible
// sub-format GUID) and "data"; other chunks are skipped, chunks are padded
// to even sizes.
void parse_wav(const unsigned char *b, uint64_t n, WavInfo *w) {
  if (n < 12 || memcmp(b, "RIFF", 4) || memcmp(b + 8, "WAVE", 4))
    FAIL(Q3T_INVALID_INPUT, "not a RIFF/WAVE image");
  bool have_fmt = false, have_data = false;
  for (uint64_t off = 12; off + 8 <= n && !have_data;) {
    const unsigned char *c = b + off;
    const uint64_t len = get_u32(c + 4);
    if (off + 8 + len > n) FAIL(Q3T_INVALID_INPUT, "wav chunk of %llu bytes runs past the image", (unsigned long long)len);
    if (!memcmp(c, "fmt ", 4)) {
      if (len < 16) FAIL(Q3T_INVALID_INPUT, "wav fmt chunk of %llu bytes", (unsigned long long)len);
      w->format = get_u16(c + 8);
      w->channels = get_u16(c + 10);
      w->rate = get_u32(c + 12);
      w->block_align = get_u16(c + 20);
      w->bits = get_u16(c + 22);
      if (w->format == 0xFFFE) {  // WAVE_FORMAT_EXTENSIBLE: the GUID's first two bytes are the format tag
        if (len < 40) FAIL(Q3T_INVALID_INPUT, "wav extensible fmt chunk of %llu bytes", (unsigned long long)len);
        w->format = get_u16(c + 8 + 24);
      }
      have_fmt = true;
    } else if (!memcmp(c, "data", 4)) {
      if (!have_fmt) FAIL(Q3T_INVALID_INPUT, "wav data chunk before its fmt chunk");
      w->data = c + 8;
      w->data_len = len;
      have_data = true;
    }
    off += 8 + len + (len & 1);
  }
  if (!have_fmt || !have_data) FAIL(Q3T_INVALID_INPUT, "wav image without %s chunk", have_fmt ? "a data" : "a fmt");
}

}  // namespace
}  // namespace q3t

using namespace q3t;

extern "C" q3t_status q3t_safetensors_open(const char *path, q3t_tensor_set **out) {
  if (!path || !out) {
    set_error("q3t_safetensors_open: null argument");
    return Q3T_INVALID_INPUT;
  }
  *out = nullptr;
  auto *s = new q3t_tensor_set();
  const q3t_status rc = io_guard([&] {
    const int fd = open(path, O_RDONLY);
    if (fd < 0) FAIL(Q3T_RUNTIME_LOAD, "cannot open %s", path);
    struct stat st;
    if (fstat(fd, &st) != 0) {
      close(fd);
      FAIL(Q3T_RUNTIME_LOAD, "cannot stat %s", path);
    }
    s->map_len = (size_t)st.st_size;
    s->map = s->map_len ? mmap(nullptr, s->map_len, PROT_READ, MAP_PRIVATE, fd, 0) : nullptr;
    close(fd);
    if (s->map_len && s->map == MAP_FAILED) {
      s->map = nullptr;
      FAIL(Q3T_RUNTIME_LOAD, "cannot map %s", path);
    }
    parse(s, static_cast<const unsigned char *>(s->map), s->map_len);
  });
  if (rc != Q3T_OK) {
    q3t_tensor_set_free(s);
    return rc;
  }
  *out = s;
  return Q3T_OK;
}

extern "C" q3t_status q3t_tensor_set_list(const q3t_tensor_set *s, const q3t_tensor **tensors, int *num_tensors) {
  if (!s || !tensors || !num_tensors) {
    set_error("q3t_tensor_set_list: null argument");
    return Q3T_INVALID_INPUT;
  }
  *tensors = s->tensors.empty() ? nullptr : s->tensors.data();
  *num_tensors = (int)s->tensors.size();
  return Q3T_OK;
}

extern "C" void q3t_tensor_set_free(q3t_tensor_set *s) {
  if (!s) return;
  if (s->map) munmap(s->map, s->map_len);
  delete s;
}

extern "C" q3t_status q3t_wav_write(const int16_t *pcm, int64_t num_samples, int sample_rate, int channels,
                                    uint8_t *out, int64_t capacity, int64_t *size) {
  if ((num_samples > 0 && !pcm) || num_samples < 0 || sample_rate <= 0 || channels < 1 || channels > 2 || !size) {
    set_error("q3t_wav_write: bad argument");
    return Q3T_INVALID_INPUT;
  }
  if (num_samples % channels) {
    set_error("q3t_wav_write: %lld samples is not a whole number of %d-channel frames", (long long)num_samples,
              channels);
    return Q3T_INVALID_INPUT;
  }
  const int64_t data = num_samples * 2;
  if (data > 0xffffffffLL - 36) {
    set_error("q3t_wav_write: %lld samples exceed the RIFF size field", (long long)num_samples);
    return Q3T_INVALID_INPUT;
  }
  *size = 44 + data;
  if (!out) return Q3T_OK;  // size query
  if (capacity < *size) {
    set_error("q3t_wav_write: buffer holds %lld bytes, need %lld", (long long)capacity, (long long)*size);
    return Q3T_INVALID_INPUT;
  }
  memcpy(out, "RIFF", 4);
  put_u32(out + 4, (uint32_t)(36 + data));
  memcpy(out + 8, "WAVEfmt ", 8);
  put_u32(out + 16, 16);  // PCM format chunk
  put_u16(out + 20, 1);   // WAVE_FORMAT_PCM
  put_u16(out + 22, (uint16_t)channels);
  put_u32(out + 24, (uint32_t)sample_rate);
  put_u32(out + 28, (uint32_t)(sample_rate * channels * 2));  // byte rate
  put_u16(out + 32, (uint16_t)(channels * 2));                // block align
  put_u16(out + 34, 16);                                      // bits per sample
  memcpy(out + 36, "data", 4);
  put_u32(out + 40, (uint32_t)data);
  for (int64_t i = 0; i < num_samples; i++) put_u16(out + 44 + 2 * i, (uint16_t)pcm[i]);
  return Q3T_OK;
}

extern "C" q3t_status q3t_wav_read(const uint8_t *bytes, int64_t n_bytes, float *samples, int64_t max_samples,
                                   int64_t *n_samples, uint32_t *sample_rate) {
  if (!bytes || n_bytes < 0 || !n_samples) {
    set_error("q3t_wav_read: bad argument");
    return Q3T_INVALID_INPUT;
  }
  return io_guard([&] {
    WavInfo w;
    parse_wav(bytes, (uint64_t)n_bytes, &w);
    if (w.channels == 0) FAIL(Q3T_INVALID_INPUT, "wav has zero channels");
    // read_wav_samples (reference_audio.rs:76-96): float 32, integer 16 / 24 / 32
    const bool flt = w.format == 3 && w.bits == 32;
    const bool pcm = w.format == 1 && (w.bits == 16 || w.bits == 24 || w.bits == 32);
    if (!flt && !pcm) FAIL(Q3T_INVALID_INPUT, "unsupported wav format: tag %d / %d-bit", w.format, w.bits);
    const int bps = w.bits / 8;
    if (w.block_align != w.channels * bps)
      FAIL(Q3T_INVALID_INPUT, "wav block align %d is not %d channels x %d bytes", w.block_align, w.channels, bps);
    const uint64_t total = w.data_len / (uint64_t)bps;  // interleaved samples
    if (total == 0) FAIL(Q3T_INVALID_INPUT, "wav contains no audio samples");
    const uint64_t frames = total / (uint64_t)w.channels;  // mixdown_to_mono keeps whole frames (:114-121)
    if (frames == 0) FAIL(Q3T_INVALID_INPUT, "wav contains no complete audio frames");
    *n_samples = (int64_t)frames;
    if (sample_rate) *sample_rate = w.rate;
    if (!samples) return;  // size query
    if (max_samples < (int64_t)frames)
      FAIL(Q3T_INVALID_INPUT, "wav has %llu frames, the output holds %lld", (unsigned long long)frames,
           (long long)max_samples);
    // integer samples: (value as f32 / 2^(bits-1)).clamp(-1, 1) (:98-112)
    const float scale = w.bits == 16 ? 32768.0f : (w.bits == 24 ? 8388608.0f : 2147483648.0f);
    auto sample = [&](uint64_t i) -> float {
      const unsigned char *p = w.data + i * (uint64_t)bps;
      if (flt) {
        const uint32_t u = get_u32(p);
        float f;
        memcpy(&f, &u, 4);
        return f;
      }
      int32_t v;
      if (bps == 2)
        v = (int16_t)get_u16(p);
      else if (bps == 3)
        v = (int32_t)((uint32_t)p[0] << 8 | (uint32_t)p[1] << 16 | (uint32_t)p[2] << 24) >> 8;
      else
        v = (int32_t)get_u32(p);
      const float x = (float)v / scale;
      return x < -1.0f ? -1.0f : (x > 1.0f ? 1.0f : x);
    };
    const float ch = (float)w.channels;
    for (uint64_t f = 0; f < frames; f++) {
      float acc = -0.0f;  // f32 Sum starts from -0.0
      for (int c = 0; c < w.channels; c++) acc += sample(f * (uint64_t)w.channels + (uint64_t)c);
      samples[f] = acc / ch;
    }
  });
}

extern "C" q3t_status q3t_resample_linear(const float *in, int64_t n, uint32_t source_rate, uint32_t target_rate,
                                          float *out, int64_t max_out, int64_t *n_out) {
  if ((n > 0 && !in) || n < 0 || !n_out) {
    set_error("q3t_resample_linear: bad argument");
    return Q3T_INVALID_INPUT;
  }
  // resample_linear (reference_audio.rs:123-156): no output for an empty
  // input or a zero rate, a copy for equal rates or a single sample
  const uint64_t src = (uint64_t)source_rate, dst = (uint64_t)target_rate;
  uint64_t len = 0;
  if (n > 0 && src > 0 && dst > 0) {
    if (src == dst || n == 1) {
      len = (uint64_t)n;
    } else {
      const unsigned __int128 num = (unsigned __int128)(uint64_t)n * dst + src / 2;
      const unsigned __int128 q = num / src;
      if (q > (unsigned __int128)((uint64_t)1 << 40)) {
        set_error("q3t_resample_linear: output of %llu+ samples", (unsigned long long)((uint64_t)1 << 40));
        return Q3T_INVALID_INPUT;
      }
      len = q == 0 ? 1 : (uint64_t)q;
    }
  }
  *n_out = (int64_t)len;
  if (!out || len == 0) return Q3T_OK;  // size query / empty
  if (max_out < (int64_t)len) {
    set_error("q3t_resample_linear: %llu output samples, the output holds %lld", (unsigned long long)len,
              (long long)max_out);
    return Q3T_INVALID_INPUT;
  }
  if (src == dst || n == 1) {
    memcpy(out, in, (size_t)len * sizeof(float));
    return Q3T_OK;
  }
  const float dst_f = (float)target_rate;
  const uint64_t last = (uint64_t)n - 1;
  for (uint64_t i = 0; i < len; i++) {
    const unsigned __int128 pos = (unsigned __int128)i * src;  // saturating u64 in the reference, never reached
    const uint64_t left = (uint64_t)(pos / dst), right = left + 1 < last ? left + 1 : last;
    const float mix = (float)(uint32_t)(pos % dst) / dst_f;
    const float a = in[left] * (1.0f - mix), b = in[right] * mix;
    out[i] = a + b;
  }
  return Q3T_OK;
}

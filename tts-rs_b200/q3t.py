"""Python host mirror of the q3t C ABI (include/q3t.h) via ctypes.

Mirrors the reference driver's hot-path API shape:
  Model(...)              ~ loading/runtime.rs:131-156 (weights -> device, bf16 cast)
  Model.session(...)      ~ TalkerGenerator::start   (talker/infer/mod.rs:69-188)
  Session.step()          ~ TalkerGenerator::step    (:190-299)
  Session.codes()         ~ TalkerGenerator::finalize (:301-311)
  Session.finish()        ~ SessionImpl::finish      (execution/loaded_model.rs:112-152)
  Model.codec_decode(...) ~ decode_waveform + to_pcm (codec/infer/mod.rs:61-111)
  Model.batch(...)        ragged continuous batching (new; the reference is batch 1)

The CUDA library must be present: there is no CPU fallback.  Errors raise
Q3TError with the status code and q3t_last_error().
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libq3t_b200.so")
_LIB = None

OK, INVALID_INPUT, RUNTIME_LOAD, TENSOR_READ, DEVICE_TIMEOUT, OUT_OF_PAGES, CUDA_ERROR = range(7)
STATUS_NAMES = ["OK", "INVALID_INPUT", "RUNTIME_LOAD", "TENSOR_READ", "DEVICE_TIMEOUT",
                "OUT_OF_PAGES", "CUDA_ERROR"]


class Q3TError(RuntimeError):
    def __init__(self, status, message):
        self.status = status
        super().__init__(f"{STATUS_NAMES[status] if 0 <= status < len(STATUS_NAMES) else status}: {message}")


class LMConfig(C.Structure):
    _fields_ = [("hidden_size", C.c_int), ("intermediate_size", C.c_int),
                ("num_hidden_layers", C.c_int), ("num_attention_heads", C.c_int),
                ("num_key_value_heads", C.c_int), ("head_dim", C.c_int), ("vocab_size", C.c_int),
                ("rms_norm_eps", C.c_float), ("rope_theta", C.c_float)]


class TalkerConfig(C.Structure):
    _fields_ = [("talker", LMConfig), ("predictor", LMConfig), ("num_code_groups", C.c_int)]


class CodecConfig(C.Structure):
    _fields_ = [(n, C.c_int) for n in (
        "num_quantizers", "num_semantic_quantizers", "codebook_size", "codebook_dim",
        "latent_dim", "decoder_dim", "hidden_size", "intermediate_size", "num_hidden_layers",
        "num_attention_heads", "num_key_value_heads", "head_dim")] + [
        ("rms_norm_eps", C.c_float), ("rope_theta", C.c_float),
        ("num_upsampling_ratios", C.c_int), ("upsampling_ratios", C.c_int * 4),
        ("num_upsample_rates", C.c_int), ("upsample_rates", C.c_int * 8),
        ("output_sample_rate", C.c_int)]


class Tensor(C.Structure):
    _fields_ = [("name", C.c_char_p), ("dtype", C.c_int), ("ndim", C.c_int),
                ("shape", C.c_int64 * 4), ("data", C.c_void_p)]


class ModelDesc(C.Structure):
    _fields_ = [("device", C.c_int), ("talker", TalkerConfig), ("has_talker", C.c_int),
                ("codec", CodecConfig), ("has_codec", C.c_int),
                ("tensors", C.POINTER(Tensor)), ("num_tensors", C.c_int),
                ("kv_pages", C.c_int64), ("max_active", C.c_int)]


class Sampling(C.Structure):
    _fields_ = [("do_sample", C.c_int), ("temperature", C.c_float), ("top_k", C.c_int),
                ("top_p", C.c_float), ("repetition_penalty", C.c_float), ("seed", C.c_uint64)]


class SessionDesc(C.Structure):
    _fields_ = [("inputs_embeds", C.POINTER(C.c_float)), ("prompt_len", C.c_int),
                ("trailing_text", C.POINTER(C.c_float)), ("trailing_len", C.c_int),
                ("pad_embed", C.POINTER(C.c_float)), ("talker_sampling", Sampling),
                ("predictor_sampling", Sampling), ("max_new_tokens", C.c_int),
                ("eos_token_id", C.c_int64), ("suppress_ids", C.POINTER(C.c_int64)),
                ("num_suppress", C.c_int), ("forced_first_token", C.c_int64),
                ("first_logits", C.POINTER(C.c_float))]


class BatchDesc(C.Structure):
    _fields_ = [("max_active", C.c_int), ("codec_mode", C.c_int), ("chunk_frames", C.c_int),
                ("left_context", C.c_int), ("keep_output", C.c_int)]


class StepStats(C.Structure):
    _fields_ = [("active", C.c_int), ("admitted", C.c_int), ("retired", C.c_int),
                ("frames", C.c_int64), ("samples", C.c_int64), ("device_ms", C.c_float),
                ("kv_tokens", C.c_int64), ("h2d_bytes", C.c_int64), ("d2h_bytes", C.c_int64),
                ("predictor_ms", C.c_float), ("talker_ms", C.c_float),
                ("prefill_tokens", C.c_int), ("first_tokens", C.c_int)]


class CodecEncoderConfig(C.Structure):
    _fields_ = [(n, C.c_int) for n in (
        "audio_channels", "num_filters", "kernel_size", "residual_kernel_size", "last_kernel_size",
        "compress", "num_ratios")] + [("ratios", C.c_int * 8)] + [(n, C.c_int) for n in (
        "hidden_size", "num_hidden_layers", "num_attention_heads", "num_key_value_heads", "head_dim",
        "intermediate_size")] + [("norm_eps", C.c_float), ("rope_theta", C.c_float)] + [(n, C.c_int) for n in (
        "codebook_size", "codebook_dim", "num_quantizers", "num_semantic_quantizers", "downsample_factor")]


class CodecEncoderDesc(C.Structure):
    _fields_ = [("device", C.c_int), ("config", CodecEncoderConfig), ("tensors", C.POINTER(Tensor)),
                ("num_tensors", C.c_int)]


class SpeakerEncoderConfig(C.Structure):
    _fields_ = [("mel_dim", C.c_int), ("enc_dim", C.c_int), ("channels", C.c_int * 5),
                ("kernel_sizes", C.c_int * 5), ("dilations", C.c_int * 5)] + [(n, C.c_int) for n in (
        "attention_channels", "res2net_scale", "se_channels", "sample_rate")]


class SpeakerEncoderDesc(C.Structure):
    _fields_ = [("device", C.c_int), ("config", SpeakerEncoderConfig), ("tensors", C.POINTER(Tensor)),
                ("num_tensors", C.c_int)]


EXPORTS = [
    "q3t_model_load", "q3t_model_free", "q3t_session_start", "q3t_session_step",
    "q3t_session_step_forced", "q3t_session_codes", "q3t_session_finish",
    "q3t_session_decode_embeds", "q3t_session_load_kv", "q3t_session_last_ms",
    "q3t_session_free", "q3t_codec_decode", "q3t_codec_out_len", "q3t_codec_decode_static",
    "q3t_batch_create",
    "q3t_batch_submit", "q3t_batch_step", "q3t_batch_poll", "q3t_batch_take",
    "q3t_batch_pending", "q3t_batch_stream", "q3t_batch_free", "q3t_last_error", "q3t_version",
    "q3t_kernel_launches", "q3t_text_project", "q3t_text_dims",
    "q3t_safetensors_open", "q3t_tensor_set_list", "q3t_tensor_set_free", "q3t_wav_write",
    "q3t_codec_last_ms", "q3t_session_seed", "q3t_abi_struct", "q3t_abi_field",
    "q3t_sample_logits", "q3t_batch_logits", "q3t_codec_encoder_load", "q3t_codec_encoder_free",
    "q3t_codec_encoder_frames", "q3t_codec_encode", "q3t_codec_encoder_hidden",
    "q3t_speaker_encoder_load", "q3t_speaker_encoder_free", "q3t_speaker_embed", "q3t_speaker_mel",
    "q3t_session_seed_voice_clone", "q3t_wav_read", "q3t_resample_linear",
]


class SeedControls(C.Structure):
    """q3t_seed_controls: a profile's control ids (ProfileControlIds)."""
    _fields_ = [("tts_bos_token_id", C.c_int64), ("tts_eos_token_id", C.c_int64),
                ("tts_pad_token_id", C.c_int64), ("codec_prefix_ids", C.POINTER(C.c_int64)),
                ("n_codec_prefix", C.c_int), ("codec_pad_id", C.c_int64), ("codec_bos_id", C.c_int64)]

_F = C.POINTER(C.c_float)
_I64 = C.POINTER(C.c_int64)


def lib():
    """Load the in-tree CUDA library; raises if it has not been built."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `make -C tts-rs_b200` "
                               "(there is no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        L.q3t_last_error.restype = C.c_char_p
        L.q3t_version.restype = C.c_char_p
        L.q3t_kernel_launches.restype = C.c_int64
        L.q3t_model_load.argtypes = [C.POINTER(ModelDesc), C.POINTER(C.c_void_p)]
        L.q3t_model_free.argtypes = [C.c_void_p]
        L.q3t_model_free.restype = None
        L.q3t_session_start.argtypes = [C.c_void_p, C.POINTER(SessionDesc), C.POINTER(C.c_void_p)]
        L.q3t_session_step.argtypes = [C.c_void_p, C.POINTER(C.c_int)]
        L.q3t_session_step_forced.argtypes = [C.c_void_p, _I64, _F, _F, _F, C.POINTER(C.c_int)]
        L.q3t_session_codes.argtypes = [C.c_void_p, _I64, C.POINTER(C.c_int)]
        L.q3t_session_finish.argtypes = [C.c_void_p, _F, C.POINTER(C.c_int16), C.c_int64, _I64]
        L.q3t_session_decode_embeds.argtypes = [C.c_void_p, _F, _F, _F]
        L.q3t_session_load_kv.argtypes = [C.c_void_p, C.POINTER(C.c_uint16), C.POINTER(C.c_uint16),
                                          C.c_int, _F]
        L.q3t_session_last_ms.argtypes = [C.c_void_p, _F]
        L.q3t_session_free.argtypes = [C.c_void_p]
        L.q3t_session_free.restype = None
        L.q3t_codec_decode.argtypes = [C.c_void_p, _I64, C.c_int, C.c_int, _F, C.POINTER(C.c_int16), _I64]
        L.q3t_codec_out_len.argtypes = [C.c_void_p, C.c_int, _I64]
        L.q3t_codec_last_ms.argtypes = [_F]
        L.q3t_codec_decode_static.argtypes = [C.c_void_p, _I64, C.c_int, C.c_int, _F,
                                              C.POINTER(C.c_int16), _I64, C.c_void_p]
        L.q3t_batch_create.argtypes = [C.c_void_p, C.POINTER(BatchDesc), C.POINTER(C.c_void_p)]
        L.q3t_batch_submit.argtypes = [C.c_void_p, C.POINTER(SessionDesc), _I64, _I64]
        L.q3t_batch_step.argtypes = [C.c_void_p, C.POINTER(StepStats)]
        L.q3t_batch_poll.argtypes = [C.c_void_p, C.c_int64, C.POINTER(C.c_int), _I64, _I64]
        L.q3t_batch_take.argtypes = [C.c_void_p, C.c_int64, _I64, C.POINTER(C.c_int32), C.c_int, _F,
                                     C.c_int64]
        L.q3t_batch_pending.argtypes = [C.c_void_p, C.POINTER(C.c_int), C.POINTER(C.c_int)]
        L.q3t_batch_logits.argtypes = [C.c_void_p, C.c_int64, _F, _F]
        L.q3t_batch_stream.argtypes = [C.c_void_p, C.POINTER(C.c_void_p)]
        L.q3t_batch_free.argtypes = [C.c_void_p]
        L.q3t_batch_free.restype = None
        L.q3t_text_project.argtypes = [C.c_void_p, _I64, C.c_int, _F]
        L.q3t_text_dims.argtypes = [C.c_void_p, C.POINTER(C.c_int), C.POINTER(C.c_int)]
        L.q3t_session_seed_voice_clone.argtypes = [C.c_void_p, _I64, C.c_int, _F, _I64, C.c_int, _I64, C.c_int,
                                                   C.POINTER(SeedControls), _F, C.c_int, C.POINTER(C.c_int), _F,
                                                   C.c_int, C.POINTER(C.c_int), _F]
        L.q3t_session_seed.argtypes = [C.c_void_p, _I64, C.c_int, _I64, C.c_int, C.POINTER(SeedControls), _F,
                                       C.c_int, C.POINTER(C.c_int), _F]
        L.q3t_safetensors_open.argtypes = [C.c_char_p, C.POINTER(C.c_void_p)]
        L.q3t_tensor_set_list.argtypes = [C.c_void_p, C.POINTER(C.POINTER(Tensor)), C.POINTER(C.c_int)]
        L.q3t_tensor_set_free.argtypes = [C.c_void_p]
        L.q3t_tensor_set_free.restype = None
        L.q3t_wav_read.argtypes = [C.POINTER(C.c_uint8), C.c_int64, _F, C.c_int64, C.POINTER(C.c_int64),
                                   C.POINTER(C.c_uint32)]
        L.q3t_resample_linear.argtypes = [_F, C.c_int64, C.c_uint32, C.c_uint32, _F, C.c_int64,
                                          C.POINTER(C.c_int64)]
        L.q3t_wav_write.argtypes = [C.POINTER(C.c_int16), C.c_int64, C.c_int, C.c_int, C.POINTER(C.c_uint8),
                                    C.c_int64, _I64]
        L.q3t_sample_logits.argtypes = [C.c_void_p, _F, C.c_int, C.POINTER(Sampling), _I64, C.c_int, C.c_double,
                                        _I64, C.POINTER(C.c_uint8)]
        L.q3t_codec_encoder_load.argtypes = [C.POINTER(CodecEncoderDesc), C.POINTER(C.c_void_p)]
        L.q3t_codec_encoder_free.argtypes = [C.c_void_p]
        L.q3t_codec_encoder_free.restype = None
        L.q3t_codec_encoder_frames.argtypes = [C.c_void_p, C.c_int64, C.POINTER(C.c_int)]
        L.q3t_codec_encode.argtypes = [C.c_void_p, _F, C.c_int64, C.c_int, _I64, C.c_int, C.POINTER(C.c_int)]
        L.q3t_codec_encoder_hidden.argtypes = [C.c_void_p, _F, C.c_int64, _F, C.c_int, C.POINTER(C.c_int)]
        L.q3t_speaker_encoder_load.argtypes = [C.POINTER(SpeakerEncoderDesc), C.POINTER(C.c_void_p)]
        L.q3t_speaker_encoder_free.argtypes = [C.c_void_p]
        L.q3t_speaker_encoder_free.restype = None
        L.q3t_speaker_embed.argtypes = [C.c_void_p, _F, C.c_int64, _F]
        L.q3t_speaker_mel.argtypes = [C.c_void_p, _F, C.c_int64, _F, C.c_int, C.POINTER(C.c_int)]
        L.q3t_abi_struct.argtypes = [C.c_char_p, C.POINTER(C.c_size_t), C.POINTER(C.c_size_t),
                                     C.POINTER(C.c_int)]
        L.q3t_abi_field.argtypes = [C.c_char_p, C.c_int, C.POINTER(C.c_char_p), C.POINTER(C.c_size_t),
                                    C.POINTER(C.c_size_t)]
        _LIB = L
    return _LIB


def abi_layout(name):
    """(size, align, [(field, offset, size), ...]) of a public struct as the
    library was compiled (q3t_abi_struct / q3t_abi_field); no GPU needed."""
    L = lib()
    size, align, n = C.c_size_t(), C.c_size_t(), C.c_int()
    check(L.q3t_abi_struct(name.encode(), C.byref(size), C.byref(align), C.byref(n)))
    fields = []
    for i in range(n.value):
        f, off, fs = C.c_char_p(), C.c_size_t(), C.c_size_t()
        check(L.q3t_abi_field(name.encode(), i, C.byref(f), C.byref(off), C.byref(fs)))
        fields.append((f.value.decode(), off.value, fs.value))
    return size.value, align.value, fields


# ctypes mirrors of the public structs, by their C names
STRUCTS = {"q3t_lm_config": LMConfig, "q3t_talker_config": TalkerConfig, "q3t_codec_config": CodecConfig,
           "q3t_tensor": Tensor, "q3t_model_desc": ModelDesc, "q3t_sampling": Sampling,
           "q3t_session_desc": SessionDesc, "q3t_seed_controls": SeedControls, "q3t_batch_desc": BatchDesc,
           "q3t_step_stats": StepStats, "q3t_codec_encoder_config": CodecEncoderConfig,
           "q3t_codec_encoder_desc": CodecEncoderDesc, "q3t_speaker_encoder_config": SpeakerEncoderConfig,
           "q3t_speaker_encoder_desc": SpeakerEncoderDesc}


def check(rc):
    if rc != OK:
        raise Q3TError(rc, lib().q3t_last_error().decode(errors="replace"))


def _fp(a):
    return None if a is None else a.ctypes.data_as(_F)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def sampling(do_sample=False, temperature=1.0, top_k=0, top_p=1.0, repetition_penalty=0.0, seed=0):
    return Sampling(int(do_sample), float(temperature), int(top_k or 0), float(top_p),
                    float(repetition_penalty or 0.0), int(seed))


def _lm(c) -> LMConfig:
    return LMConfig(c.hidden, c.inter, c.n_layers, c.n_heads, c.n_kv, c.head_dim, c.vocab,
                    c.eps, c.theta)


def codec_config(c) -> CodecConfig:
    cc = CodecConfig(c.n_q, c.n_semantic, c.codebook_size, c.codebook_dim, c.latent,
                     c.decoder_dim, c.hidden, c.inter, c.n_layers, c.n_heads, c.n_kv, c.head_dim)
    cc.rms_norm_eps, cc.rope_theta = c.eps, c.theta
    cc.num_upsampling_ratios = len(c.up_ratios)
    for i, r in enumerate(c.up_ratios):
        cc.upsampling_ratios[i] = r
    cc.num_upsample_rates = len(c.rates)
    for i, r in enumerate(c.rates):
        cc.upsample_rates[i] = r
    cc.output_sample_rate = c.sample_rate
    return cc


def codec_encoder_config(c) -> CodecEncoderConfig:
    """q3t_codec_encoder_config from a synthetic.CodecEncoderConfig."""
    e = CodecEncoderConfig()
    e.audio_channels, e.num_filters, e.kernel_size = c.audio_channels, c.num_filters, c.kernel_size
    e.residual_kernel_size, e.last_kernel_size, e.compress = c.residual_kernel_size, c.last_kernel_size, c.compress
    e.num_ratios = len(c.upsampling_ratios)
    for i, r in enumerate(c.upsampling_ratios):
        e.ratios[i] = r
    e.hidden_size, e.num_hidden_layers, e.num_attention_heads = c.hidden, c.n_layers, c.n_heads
    e.num_key_value_heads, e.head_dim, e.intermediate_size = c.n_kv, c.head_dim, c.inter
    e.norm_eps, e.rope_theta = c.norm_eps, c.theta
    e.codebook_size, e.codebook_dim, e.num_quantizers = c.codebook_size, c.vq_dim, c.n_q
    e.num_semantic_quantizers, e.downsample_factor = c.n_semantic, c.downsample_factor
    return e


class CodecEncoder:
    """Speech-tokenizer encoder of the voice-clone path on the device
    (q3t_codec_encoder_*; Qwen3TtsAudioCodecEncoder::encode_reference_prefix,
    codec/network/encoder.rs:121-136).  Weights map checkpoint names to float
    arrays (synthetic.codec_encoder_tensor_specs names)."""

    def __init__(self, cfg, weights, device=0):
        L = lib()
        keep, tens = [], []
        for name, arr in weights.items():
            a = _f32(arr)
            nb = name.encode()
            keep += [a, nb]
            tens.append(Tensor(nb, 0, a.ndim, (C.c_int64 * 4)(*(list(a.shape) + [0] * (4 - a.ndim))),
                               a.ctypes.data))
        arr = (Tensor * max(1, len(tens)))(*tens)
        d = CodecEncoderDesc(device, codec_encoder_config(cfg), arr, len(tens))
        h = C.c_void_p()
        check(L.q3t_codec_encoder_load(C.byref(d), C.byref(h)))
        self.h, self.cfg = h, cfg

    def frames(self, n):
        f = C.c_int()
        check(lib().q3t_codec_encoder_frames(self.h, int(n), C.byref(f)))
        return f.value

    def encode(self, wave, n_valid=None):
        """wave [n] f32 -> codes [n_valid][frames] (n_valid defaults to all codebooks)."""
        wave = _f32(wave)
        n_valid = self.cfg.n_q if n_valid is None else n_valid
        T = self.frames(len(wave))
        codes = np.zeros((n_valid, T), np.int64)
        got = C.c_int()
        check(lib().q3t_codec_encode(self.h, _fp(wave), len(wave), n_valid, codes.ctypes.data_as(_I64), T,
                                     C.byref(got)))
        assert got.value == T
        return codes

    def hidden(self, wave):
        """The hidden [hidden][frames] the quantizers read."""
        wave = _f32(wave)
        T = self.frames(len(wave))
        out = np.zeros((self.cfg.hidden, T), np.float32)
        got = C.c_int()
        check(lib().q3t_codec_encoder_hidden(self.h, _fp(wave), len(wave), _fp(out), T, C.byref(got)))
        assert got.value == T
        return out

    def close(self):
        if getattr(self, "h", None):
            lib().q3t_codec_encoder_free(self.h)
            self.h = None

    def __del__(self):
        self.close()


def speaker_encoder_config(c) -> SpeakerEncoderConfig:
    """q3t_speaker_encoder_config from a synthetic.SpeakerEncoderConfig."""
    e = SpeakerEncoderConfig()
    e.mel_dim, e.enc_dim = c.mel_dim, c.enc_dim
    for i in range(5):
        e.channels[i], e.kernel_sizes[i], e.dilations[i] = c.enc_channels[i], c.enc_kernel_sizes[i], c.enc_dilations[i]
    e.attention_channels, e.res2net_scale = c.enc_attention_channels, c.enc_res2net_scale
    e.se_channels, e.sample_rate = c.enc_se_channels, c.sample_rate
    return e


class SpeakerEncoder:
    """ECAPA-TDNN speaker encoder of the voice-clone path on the device
    (q3t_speaker_*; LoadedQwen3TtsSpeakerEncoder::encode_embedding,
    speaker/infer/mod.rs:11-20).  Weights map checkpoint names to float
    arrays (synthetic.speaker_tensor_specs names)."""

    def __init__(self, cfg, weights, device=0):
        L = lib()
        keep, tens = [], []
        for name, arr in weights.items():
            a = _f32(arr)
            nb = name.encode()
            keep += [a, nb]
            tens.append(Tensor(nb, 0, a.ndim, (C.c_int64 * 4)(*(list(a.shape) + [0] * (4 - a.ndim))),
                               a.ctypes.data))
        arr = (Tensor * max(1, len(tens)))(*tens)
        d = SpeakerEncoderDesc(device, speaker_encoder_config(cfg), arr, len(tens))
        h = C.c_void_p()
        check(L.q3t_speaker_encoder_load(C.byref(d), C.byref(h)))
        self.h, self.cfg = h, cfg

    def embed(self, samples):
        """samples [n] f32 at the config's sample rate -> x-vector [enc_dim]."""
        x = _f32(samples)
        out = np.zeros(self.cfg.enc_dim, np.float32)
        check(lib().q3t_speaker_embed(self.h, _fp(x), len(x), _fp(out)))
        return out

    def mel(self, samples):
        """The log-mel features [mel_dim][frames] the network reads."""
        x = _f32(samples)
        T = max(self.cfg.frames(len(x)), 1)
        out = np.zeros((self.cfg.mel_dim, T), np.float32)
        got = C.c_int()
        check(lib().q3t_speaker_mel(self.h, _fp(x), len(x), _fp(out), T, C.byref(got)))
        assert got.value == T
        return out

    def close(self):
        if getattr(self, "h", None):
            lib().q3t_speaker_encoder_free(self.h)
            self.h = None

    def __del__(self):
        self.close()


class TensorSet:
    """A memory-mapped .safetensors checkpoint (q3t_safetensors_open): its
    float tensors by checkpoint name, ready for Model(tensor_sets=[...])."""

    def __init__(self, path):
        h = C.c_void_p()
        check(lib().q3t_safetensors_open(os.fsencode(path), C.byref(h)))
        self.h = h

    def tensors(self):
        """[(name, dtype, shape)] of the listed tensors (dtype 0 = f32, 1 = bf16)."""
        p, n = C.POINTER(Tensor)(), C.c_int()
        check(lib().q3t_tensor_set_list(self.h, C.byref(p), C.byref(n)))
        return [(p[i].name.decode(), p[i].dtype, tuple(p[i].shape[:p[i].ndim])) for i in range(n.value)]

    def raw(self):
        p, n = C.POINTER(Tensor)(), C.c_int()
        check(lib().q3t_tensor_set_list(self.h, C.byref(p), C.byref(n)))
        return [p[i] for i in range(n.value)]

    def close(self):
        if getattr(self, "h", None):
            lib().q3t_tensor_set_free(self.h)
            self.h = None

    def __del__(self):
        self.close()


def wav_bytes(pcm, sample_rate=24000, channels=1):
    """PcmAudio::write_wav: the RIFF/WAVE image of int16 samples."""
    pcm = np.ascontiguousarray(pcm, np.int16)
    size = C.c_int64()
    pp = pcm.ctypes.data_as(C.POINTER(C.c_int16)) if pcm.size else None
    check(lib().q3t_wav_write(pp, pcm.size, sample_rate, channels, None, 0, C.byref(size)))
    out = np.zeros(size.value, np.uint8)
    check(lib().q3t_wav_write(pp, pcm.size, sample_rate, channels, out.ctypes.data_as(C.POINTER(C.c_uint8)),
                              size.value, C.byref(size)))
    return out.tobytes()


def wav_read(data):
    """decode_reference_audio on a WAV image: (mono f32 samples, sample rate)."""
    buf = np.frombuffer(bytes(data), np.uint8)
    bp = buf.ctypes.data_as(C.POINTER(C.c_uint8))
    n, rate = C.c_int64(), C.c_uint32()
    check(lib().q3t_wav_read(bp, buf.size, None, 0, C.byref(n), C.byref(rate)))
    out = np.zeros(n.value, np.float32)
    check(lib().q3t_wav_read(bp, buf.size, _fp(out), n.value, C.byref(n), C.byref(rate)))
    return out, rate.value


def resample_linear(samples, source_rate, target_rate):
    """resample_linear: linear interpolation to target_rate (f32)."""
    x = _f32(np.asarray(samples).reshape(-1))
    n = C.c_int64()
    xp = _fp(x) if x.size else None
    check(lib().q3t_resample_linear(xp, x.size, int(source_rate), int(target_rate), None, 0, C.byref(n)))
    out = np.zeros(n.value, np.float32)
    check(lib().q3t_resample_linear(xp, x.size, int(source_rate), int(target_rate),
                                    _fp(out) if out.size else None, n.value, C.byref(n)))
    return out


class Model:
    """A loaded Qwen3-TTS model on one GPU (talker + code predictor and/or
    codec decoder).  Weight dicts map checkpoint names to float32 arrays."""

    def __init__(self, talker_cfg=None, talker_weights=None, codec_cfg=None, codec_weights=None,
                 device=0, kv_pages=0, max_active=0, tensor_sets=()):
        L = lib()
        keep, tens = [], []
        for ts in tensor_sets:
            tens.extend(ts.raw())
        for wdict in (talker_weights or {}), (codec_weights or {}):
            for name, arr in wdict.items():
                a = _f32(arr)
                keep.append(a)
                nb = name.encode()
                keep.append(nb)
                t = Tensor(nb, 0, a.ndim, (C.c_int64 * 4)(*(list(a.shape) + [0] * (4 - a.ndim))),
                           a.ctypes.data)
                tens.append(t)
        arr = (Tensor * max(1, len(tens)))(*tens)
        d = ModelDesc()
        d.device = device
        d.has_talker = int(talker_cfg is not None)
        if talker_cfg is not None:
            d.talker = TalkerConfig(_lm(talker_cfg.talker), _lm(talker_cfg.predictor), talker_cfg.n_groups)
        d.has_codec = int(codec_cfg is not None)
        if codec_cfg is not None:
            d.codec = codec_config(codec_cfg)
        d.tensors = arr
        d.num_tensors = len(tens)
        d.kv_pages = kv_pages
        d.max_active = max_active
        h = C.c_void_p()
        check(L.q3t_model_load(C.byref(d), C.byref(h)))
        self.h = h
        self.talker_cfg, self.codec_cfg = talker_cfg, codec_cfg

    def close(self):
        if getattr(self, "h", None):
            lib().q3t_model_free(self.h)
            self.h = None

    def __del__(self):
        self.close()

    # -- sessions -------------------------------------------------------------
    def session(self, prompt, trailing, pad, talker_sampling=None, predictor_sampling=None,
                max_new_tokens=64, eos=-1, suppress=None, forced_first=-1, first_logits=False):
        return Session(self, prompt, trailing, pad, talker_sampling, predictor_sampling,
                       max_new_tokens, eos, suppress, forced_first, first_logits)

    # -- codec ------------------------------------------------------------------
    def codec_out_len(self, T):
        n = C.c_int64()
        check(lib().q3t_codec_out_len(self.h, T, C.byref(n)))
        return n.value

    def codec_decode(self, codes, pcm=False):
        codes = np.ascontiguousarray(codes, np.int64)
        B, _, T = codes.shape
        n = self.codec_out_len(T)
        wave = np.zeros((B, n), np.float32)
        p = np.zeros((B, n), np.int16) if pcm else None
        nn = C.c_int64()
        check(lib().q3t_codec_decode(self.h, codes.ctypes.data_as(_I64), B, T, _fp(wave),
                                     None if p is None else p.ctypes.data_as(C.POINTER(C.c_int16)),
                                     C.byref(nn)))
        return (wave, p) if pcm else wave

    def text_project(self, ids):
        """project_text_ids on the device: [n][hidden] f32 rows (bf16 values)."""
        ids = np.ascontiguousarray(ids, np.int64)
        out = np.zeros((len(ids), self.talker_cfg.talker.hidden), np.float32)
        check(lib().q3t_text_project(self.h, ids.ctypes.data_as(_I64) if len(ids) else None, len(ids), _fp(out)))
        return out

    def session_seed(self, text_ids, controls, leading_ids=None):
        """build_non_streaming_seed on the device: (inputs_embeds [rows][hidden],
        tts_pad embedding [hidden]); controls: dict of q3t_seed_controls fields
        with codec_prefix_ids as a sequence."""
        text_ids = np.ascontiguousarray(text_ids, np.int64)
        lead = None if leading_ids is None else np.ascontiguousarray(leading_ids, np.int64)
        cp = np.ascontiguousarray(controls["codec_prefix_ids"], np.int64)
        ctl = SeedControls(controls["tts_bos_token_id"], controls["tts_eos_token_id"], controls["tts_pad_token_id"],
                           cp.ctypes.data_as(_I64), len(cp), controls["codec_pad_id"], controls["codec_bos_id"])
        args = (self.h, text_ids.ctypes.data_as(_I64), len(text_ids),
                None if lead is None else lead.ctypes.data_as(_I64), 0 if lead is None else len(lead),
                C.byref(ctl))
        rows = C.c_int()
        check(lib().q3t_session_seed(*args, None, 0, C.byref(rows), None))
        H = self.talker_cfg.talker.hidden
        out = np.zeros((rows.value, H), np.float32)
        pad = np.zeros(H, np.float32)
        check(lib().q3t_session_seed(*args, _fp(out), rows.value, C.byref(rows), _fp(pad)))
        return out, pad

    def session_seed_voice_clone(self, text_ids, controls, speaker, ref_text_ids=None, ref_codes=None):
        """build_voice_clone_seed on the device: (inputs_embeds [rows][hidden],
        trailing text [rows][hidden], tts_pad embedding [hidden]); speaker =
        the x-vector [hidden]; ref_text_ids / ref_codes [groups][frames] select
        the in-context recipe."""
        text_ids = np.ascontiguousarray(text_ids, np.int64)
        spk = _f32(np.asarray(speaker).reshape(-1))
        rt = None if ref_text_ids is None else np.ascontiguousarray(ref_text_ids, np.int64)
        rc = None if ref_codes is None else np.ascontiguousarray(ref_codes, np.int64)
        cp = np.ascontiguousarray(controls["codec_prefix_ids"], np.int64)
        ctl = SeedControls(controls["tts_bos_token_id"], controls["tts_eos_token_id"], controls["tts_pad_token_id"],
                           cp.ctypes.data_as(_I64), len(cp), controls["codec_pad_id"], controls["codec_bos_id"])
        head = (self.h, text_ids.ctypes.data_as(_I64), len(text_ids), _fp(spk),
                None if rt is None else rt.ctypes.data_as(_I64), 0 if rt is None else len(rt),
                None if rc is None else rc.ctypes.data_as(_I64), 0 if rc is None else rc.shape[-1], C.byref(ctl))
        rows, trows = C.c_int(), C.c_int()
        check(lib().q3t_session_seed_voice_clone(*head, None, 0, C.byref(rows), None, 0, C.byref(trows), None))
        H = self.talker_cfg.talker.hidden
        out = np.zeros((rows.value, H), np.float32)
        tr = np.zeros((trows.value, H), np.float32)
        pad = np.zeros(H, np.float32)
        check(lib().q3t_session_seed_voice_clone(*head, _fp(out), rows.value, C.byref(rows), _fp(tr), trows.value,
                                                 C.byref(trows), _fp(pad)))
        return out, tr, pad

    @staticmethod
    def codec_last_ms():
        """Device time (ms) of this thread's last codec decode."""
        ms = C.c_float()
        check(lib().q3t_codec_last_ms(C.byref(ms)))
        return ms.value

    def sample_logits(self, logits, sampling, u, suppress=None):
        """The device sampler on one row with the uniform draw u: (token, kept mask)."""
        lg = _f32(logits)
        sup = None if suppress is None else np.ascontiguousarray(suppress, np.int64)
        tok = C.c_int64()
        kept = np.zeros(lg.shape[0], np.uint8)
        check(lib().q3t_sample_logits(self.h, _fp(lg), lg.shape[0], C.byref(sampling),
                                      None if sup is None else sup.ctypes.data_as(_I64),
                                      0 if sup is None else sup.shape[0], float(u), C.byref(tok),
                                      kept.ctypes.data_as(C.POINTER(C.c_uint8))))
        return tok.value, kept.astype(bool)

    def batch(self, max_active=64, codec_mode=0, chunk_frames=16, left_context=8, keep_output=1):
        return Batch(self, max_active, codec_mode, chunk_frames, left_context, keep_output)


def _session_desc(model, prompt, trailing, pad, ts, cs, max_new, eos, suppress, forced_first,
                  first_logits_buf, keep):
    prompt, trailing, pad = _f32(prompt), _f32(trailing), _f32(pad)
    sup = np.ascontiguousarray(suppress if suppress is not None else [], np.int64)
    keep += [prompt, trailing, pad, sup]
    d = SessionDesc()
    d.inputs_embeds = _fp(prompt)
    d.prompt_len = prompt.shape[0]
    d.trailing_text = _fp(trailing)
    d.trailing_len = trailing.shape[0]
    d.pad_embed = _fp(pad)
    d.talker_sampling = ts or sampling()
    d.predictor_sampling = cs or sampling()
    d.max_new_tokens = max_new
    d.eos_token_id = eos
    d.suppress_ids = sup.ctypes.data_as(_I64) if len(sup) else None
    d.num_suppress = len(sup)
    d.forced_first_token = forced_first
    d.first_logits = _fp(first_logits_buf)
    return d


class Session:
    def __init__(self, model, prompt, trailing, pad, ts, cs, max_new, eos, suppress, forced_first,
                 want_first_logits):
        self.model = model
        tc = model.talker_cfg
        self._keep = []
        self.first_logits = np.zeros(tc.talker.vocab, np.float32) if want_first_logits else None
        d = _session_desc(model, prompt, trailing, pad, ts, cs, max_new, eos, suppress,
                          forced_first, self.first_logits, self._keep)
        h = C.c_void_p()
        check(lib().q3t_session_start(model.h, C.byref(d), C.byref(h)))
        self.h = h

    def step(self):
        st = C.c_int()
        check(lib().q3t_session_step(self.h, C.byref(st)))
        return st.value

    def step_forced(self, codes):
        tc = self.model.talker_cfg
        codes = np.ascontiguousarray(codes, np.int64)
        tl = np.zeros(tc.talker.vocab, np.float32)
        pl = np.zeros((tc.n_groups - 1, tc.predictor.vocab), np.float32)
        hid = np.zeros(tc.talker.hidden, np.float32)
        st = C.c_int()
        check(lib().q3t_session_step_forced(self.h, codes.ctypes.data_as(_I64), _fp(tl), _fp(pl),
                                            _fp(hid), C.byref(st)))
        return st.value, tl, pl, hid

    def codes(self):
        T = C.c_int()
        check(lib().q3t_session_codes(self.h, None, C.byref(T)))
        out = np.zeros((self.model.talker_cfg.n_groups, T.value), np.int64)
        check(lib().q3t_session_codes(self.h, out.ctypes.data_as(_I64), C.byref(T)))
        return out

    def finish(self, pcm=False):
        n = C.c_int64()
        check(lib().q3t_session_finish(self.h, None, None, 0, C.byref(n)))
        wave = np.zeros(n.value, np.float32)
        p = np.zeros(n.value, np.int16) if pcm else None
        check(lib().q3t_session_finish(self.h, _fp(wave),
                                       None if p is None else p.ctypes.data_as(C.POINTER(C.c_int16)),
                                       n.value, C.byref(n)))
        return (wave, p) if pcm else wave

    def decode_embeds(self, emb):
        tc = self.model.talker_cfg
        emb = _f32(emb)
        logits = np.zeros(tc.talker.vocab, np.float32)
        hid = np.zeros(tc.talker.hidden, np.float32)
        check(lib().q3t_session_decode_embeds(self.h, _fp(emb), _fp(logits), _fp(hid)))
        return logits, hid

    def load_kv(self, k_bits, v_bits, length, hidden=None):
        k = np.ascontiguousarray(k_bits, np.uint16)
        v = np.ascontiguousarray(v_bits, np.uint16)
        h = None if hidden is None else _f32(hidden)
        check(lib().q3t_session_load_kv(self.h, k.ctypes.data_as(C.POINTER(C.c_uint16)),
                                        v.ctypes.data_as(C.POINTER(C.c_uint16)), length, _fp(h)))

    def last_ms(self):
        ms = C.c_float()
        check(lib().q3t_session_last_ms(self.h, C.byref(ms)))
        return ms.value

    def close(self):
        if getattr(self, "h", None):
            lib().q3t_session_free(self.h)
            self.h = None

    def __del__(self):
        self.close()


class Batch:
    """Ragged continuous batching over one model (q3t_batch_*)."""

    def __init__(self, model, max_active, codec_mode, chunk_frames, left_context, keep_output):
        self.model = model
        d = BatchDesc(max_active, codec_mode, chunk_frames, left_context, keep_output)
        h = C.c_void_p()
        check(lib().q3t_batch_create(model.h, C.byref(d), C.byref(h)))
        self.h = h
        self._keep = {}

    def submit(self, prompt, trailing, pad, max_new_tokens, talker_sampling=None,
               predictor_sampling=None, eos=-1, suppress=None, forced=None, first_logits=None):
        """first_logits (nullable): a float32 [vocab] array that receives the
        logits of the first talker token at admission."""
        keep = []
        d = _session_desc(self.model, prompt, trailing, pad, talker_sampling, predictor_sampling,
                          max_new_tokens, eos, suppress, -1, first_logits, keep)
        fz = None
        if forced is not None:
            fz = np.ascontiguousarray(forced, np.int64)
            keep.append(fz)
        rid = C.c_int64()
        check(lib().q3t_batch_submit(self.h, C.byref(d), None if fz is None else fz.ctypes.data_as(_I64),
                                     C.byref(rid)))
        return rid.value

    def step(self):
        s = StepStats()
        check(lib().q3t_batch_step(self.h, C.byref(s)))
        return {"active": s.active, "admitted": s.admitted, "retired": s.retired,
                "frames": s.frames, "samples": s.samples, "device_ms": s.device_ms,
                "kv_tokens": s.kv_tokens, "h2d_bytes": s.h2d_bytes, "d2h_bytes": s.d2h_bytes,
                "predictor_ms": s.predictor_ms, "talker_ms": s.talker_ms,
                "prefill_tokens": s.prefill_tokens, "first_tokens": s.first_tokens}

    def poll(self, rid):
        st, fr, sm = C.c_int(), C.c_int64(), C.c_int64()
        check(lib().q3t_batch_poll(self.h, rid, C.byref(st), C.byref(fr), C.byref(sm)))
        return st.value, fr.value, sm.value

    def take(self, rid, with_wave=False):
        st, T, ns = self.poll(rid)
        G = self.model.talker_cfg.n_groups
        codes = np.zeros((G, T), np.int64)
        sampled = np.zeros((G, T), np.int32)
        wave = np.zeros(ns, np.float32) if with_wave else None
        check(lib().q3t_batch_take(self.h, rid, codes.ctypes.data_as(_I64),
                                   sampled.ctypes.data_as(C.POINTER(C.c_int32)), T, _fp(wave),
                                   0 if wave is None else ns))
        return codes, sampled, wave

    def stream(self):
        """cudaStream_t of the batch, as an int (torch.cuda.ExternalStream)."""
        p = C.c_void_p()
        check(lib().q3t_batch_stream(self.h, C.byref(p)))
        return p.value or 0

    def logits(self, rid):
        """(talker [vocab], predictor [G-1][cp_vocab]) logits of the request's
        token in the last decode frame."""
        tc = self.model.talker_cfg
        tl = np.zeros(tc.talker.vocab, np.float32)
        pl = np.zeros((tc.n_groups - 1, tc.predictor.vocab), np.float32)
        check(lib().q3t_batch_logits(self.h, rid, _fp(tl), _fp(pl)))
        return tl, pl

    def pending(self):
        q, a = C.c_int(), C.c_int()
        check(lib().q3t_batch_pending(self.h, C.byref(q), C.byref(a)))
        return q.value, a.value

    def close(self):
        if getattr(self, "h", None):
            lib().q3t_batch_free(self.h)
            self.h = None

    def __del__(self):
        self.close()


def kernel_launches():
    return lib().q3t_kernel_launches()

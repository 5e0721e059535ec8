"""Seed-0 synthetic Qwen3-TTS weights and configs (no checkpoint is available).

Tensor names are the checkpoint names the reference loads
(tts_qwen3_tts/src/model/talker/weights.rs:14-93 — module tree of
talker/network/model.rs:15-35 and predictor.rs:11-25 under the `talker.`
root; codec/weights.rs:13-33 with the legacy `._codebook.` spelling).  Layouts
are PyTorch's: Linear [out, in], Conv1d [out, in/groups, k], ConvTranspose1d
[in, out, k].

Every tensor is drawn from its own generator seeded by (seed, crc32(name)),
so a model with fewer layers has the same leading layers as the full one.
Talker / code-predictor tensors are rounded to bf16 (the reference's
load-time dtype cast, loading/load_adapter.rs:18-46); codec tensors stay f32
(the codec is compared against an f32 decode).
"""
from __future__ import annotations

import os
import zlib
from dataclasses import dataclass, field, asdict, replace

import numpy as np


@dataclass
class LMConfig:
    """Decoder-stack hyper-parameters (talker/config.rs:18-61)."""
    hidden: int = 1024
    inter: int = 3072
    n_layers: int = 28
    n_heads: int = 16
    n_kv: int = 8
    head_dim: int = 128
    eps: float = 1e-6
    theta: float = 1e6
    vocab: int = 3072


@dataclass
class TalkerConfig:
    """Talker + code predictor of Qwen3-TTS-12Hz-0.6B (fixture at
    talker/config.rs:343-384)."""
    talker: LMConfig = field(default_factory=LMConfig)
    predictor: LMConfig = field(default_factory=lambda: LMConfig(n_layers=5, vocab=2048))
    n_groups: int = 16

    def small(self, talker_layers=2, predictor_layers=1):
        return TalkerConfig(
            talker=LMConfig(**{**asdict(self.talker), "n_layers": talker_layers}),
            predictor=LMConfig(**{**asdict(self.predictor), "n_layers": predictor_layers}),
            n_groups=self.n_groups)


@dataclass
class CodecConfig:
    """Speech-tokenizer decoder (codec/config.rs:50-76).  The package's
    speech_tokenizer/config.json is not available, so these dims are the
    12 Hz tokenizer's published shape: 16 codebooks of 2048 x 256, latent
    1024, decoder 1536, 8 x 512-wide pre-transformer, upsampling [2, 2],
    rates [8, 5, 4, 3] (1920 samples per frame at 24 kHz)."""
    n_q: int = 16
    n_semantic: int = 1
    codebook_size: int = 2048
    codebook_dim: int = 512
    latent: int = 1024
    decoder_dim: int = 1536
    hidden: int = 512
    inter: int = 1024
    n_layers: int = 8
    n_heads: int = 16
    n_kv: int = 16
    head_dim: int = 64
    eps: float = 1e-5
    theta: float = 1e4
    up_ratios: tuple = (2, 2)
    rates: tuple = (8, 5, 4, 3)
    layer_scale: float = 0.01
    sample_rate: int = 24000

    def out_len(self, T: int) -> int:
        L = T
        for r in self.up_ratios:
            L *= r
        for r in self.rates:
            L = (L - 1) * r if L > 0 else 0
        return L


def bf16_round(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16, returned as f32."""
    a = np.array(a, dtype=np.float32, copy=True, order="C")
    if a.size == 0:
        return a
    u = a.view(np.uint32)
    lsb = (u >> np.uint32(16)) & np.uint32(1)
    u += np.uint32(0x7FFF)
    u += lsb
    u &= np.uint32(0xFFFF0000)
    return a


def bf16_bits(a: np.ndarray) -> np.ndarray:
    """f32 array -> uint16 bf16 bit patterns (round-to-nearest-even)."""
    return (bf16_round(a).view(np.uint32) >> 16).astype(np.uint16)


def _rng(seed: int, name: str) -> np.random.Generator:
    return np.random.default_rng([seed, zlib.crc32(name.encode())])


def _normal(seed, name, shape, std, mean=0.0):
    a = _rng(seed, name).standard_normal(shape, dtype=np.float32)
    a *= np.float32(std)
    if mean:
        a += np.float32(mean)
    return a


def talker_tensor_specs(cfg: TalkerConfig):
    """(name, shape, kind) for every hot-path tensor of the talker bundle."""
    specs = []

    def stack(prefix, c: LMConfig):
        H, I, hd = c.hidden, c.inter, c.head_dim
        for l in range(c.n_layers):
            p = f"{prefix}.layers.{l}"
            specs.extend([
                (f"{p}.input_layernorm.weight", (H,), "gamma"),
                (f"{p}.post_attention_layernorm.weight", (H,), "gamma"),
                (f"{p}.self_attn.q_proj.weight", (c.n_heads * hd, H), "linear"),
                (f"{p}.self_attn.k_proj.weight", (c.n_kv * hd, H), "linear"),
                (f"{p}.self_attn.v_proj.weight", (c.n_kv * hd, H), "linear"),
                (f"{p}.self_attn.o_proj.weight", (H, c.n_heads * hd), "linear"),
                (f"{p}.self_attn.q_norm.weight", (hd,), "gamma"),
                (f"{p}.self_attn.k_norm.weight", (hd,), "gamma"),
                (f"{p}.mlp.gate_proj.weight", (I, H), "linear"),
                (f"{p}.mlp.up_proj.weight", (I, H), "linear"),
                (f"{p}.mlp.down_proj.weight", (H, I), "linear"),
            ])
        specs.append((f"{prefix}.norm.weight", (H,), "gamma"))

    t, p = cfg.talker, cfg.predictor
    stack("talker.model", t)
    specs.append(("talker.model.codec_embedding.weight", (t.vocab, t.hidden), "embed"))
    specs.append(("talker.codec_head.weight", (t.vocab, t.hidden), "linear"))
    stack("talker.code_predictor.model", p)
    for j in range(cfg.n_groups - 1):
        specs.append((f"talker.code_predictor.model.codec_embedding.{j}.weight",
                      (p.vocab, t.hidden), "embed"))
        specs.append((f"talker.code_predictor.lm_head.{j}.weight", (p.vocab, p.hidden), "linear"))
    return specs


def _parallel(fn, items):
    """Tensors are independent, so generate them on a thread pool (numpy's
    generators and ufuncs release the GIL on large arrays)."""
    from concurrent.futures import ThreadPoolExecutor
    with ThreadPoolExecutor(max_workers=min(16, os.cpu_count() or 4)) as ex:
        return dict(ex.map(fn, items))


def make_talker_weights(cfg: TalkerConfig, seed: int = 0) -> dict:
    """Seed-0 talker bundle: Linear ~N(0, 0.02), norm gammas ~1+N(0, 0.1),
    embeddings ~N(0, 0.5); all rounded to bf16."""
    def one(spec):
        name, shape, kind = spec
        if kind == "gamma":
            a = _normal(seed, name, shape, 0.1, 1.0)
        elif kind == "embed":
            a = _normal(seed, name, shape, 0.5)
        else:
            a = _normal(seed, name, shape, 0.02)
        return name, bf16_round(a)
    return _parallel(one, talker_tensor_specs(cfg))


def text_tensor_specs(cfg: TalkerConfig, text_vocab: int = 151936, text_hidden: int = 2048):
    """The prompt text path (talker/config.rs:142-143, 200-209): text embedding
    and the two-layer text projection with biases."""
    H = cfg.talker.hidden
    return [("talker.model.text_embedding.weight", (text_vocab, text_hidden), "embed"),
            ("talker.text_projection.linear_fc1.weight", (text_hidden, text_hidden), "linear"),
            ("talker.text_projection.linear_fc1.bias", (text_hidden,), "bias"),
            ("talker.text_projection.linear_fc2.weight", (H, text_hidden), "linear"),
            ("talker.text_projection.linear_fc2.bias", (H,), "bias")]


def make_text_weights(cfg: TalkerConfig, seed: int = 0, text_vocab: int = 151936, text_hidden: int = 2048) -> dict:
    """Seed-0 text path tensors (embedding ~N(0, 0.5), linears ~N(0, 0.02),
    biases ~N(0, 0.02)), rounded to bf16.  Kept separate from the talker
    bundle: the full text embedding alone is 151936 x 2048."""
    def one(spec):
        name, shape, kind = spec
        a = _normal(seed, name, shape, 0.5 if kind == "embed" else 0.02)
        return name, bf16_round(a)
    return _parallel(one, text_tensor_specs(cfg, text_vocab, text_hidden))


def codec_tensor_specs(c: CodecConfig):
    half, D, LAT, H = c.codebook_dim // 2, c.codebook_dim, c.latent, c.hidden
    s = []
    rvq = [("rvq_first", i) for i in range(c.n_semantic)] + \
          [("rvq_rest", i) for i in range(c.n_q - c.n_semantic)]
    for grp, i in rvq:
        p = f"decoder.quantizer.{grp}.vq.layers.{i}._codebook"
        s.append((f"{p}.embedding_sum", (c.codebook_size, half), ("normal", 1.0)))
        s.append((f"{p}.cluster_usage", (c.codebook_size,), ("usage",)))
    s.append(("decoder.quantizer.rvq_first.output_proj.weight", (D, half, 1), ("fan", half, 1.0)))
    s.append(("decoder.quantizer.rvq_rest.output_proj.weight", (D, half, 1), ("fan", half * 4, 1.0)))
    s.append(("decoder.pre_conv.conv.weight", (LAT, D, 3), ("fan", D * 3, 1.0)))
    s.append(("decoder.pre_conv.conv.bias", (LAT,), ("normal", 0.02)))
    pt = "decoder.pre_transformer"
    s.append((f"{pt}.input_proj.weight", (H, LAT), ("fan", LAT, 1.0)))
    s.append((f"{pt}.input_proj.bias", (H,), ("normal", 0.02)))
    s.append((f"{pt}.output_proj.weight", (LAT, H), ("fan", H, 1.0)))
    s.append((f"{pt}.output_proj.bias", (LAT,), ("normal", 0.02)))
    s.append((f"{pt}.norm.weight", (H,), ("gamma",)))
    qd, kd = c.n_heads * c.head_dim, c.n_kv * c.head_dim
    for l in range(c.n_layers):
        p = f"{pt}.layers.{l}"
        s += [(f"{p}.input_layernorm.weight", (H,), ("gamma",)),
              (f"{p}.post_attention_layernorm.weight", (H,), ("gamma",)),
              (f"{p}.self_attn.q_proj.weight", (qd, H), ("fan", H, 1.0)),
              (f"{p}.self_attn.k_proj.weight", (kd, H), ("fan", H, 1.0)),
              (f"{p}.self_attn.v_proj.weight", (kd, H), ("fan", H, 1.0)),
              (f"{p}.self_attn.o_proj.weight", (H, qd), ("fan", qd, 1.0)),
              (f"{p}.mlp.gate_proj.weight", (c.inter, H), ("fan", H, 1.0)),
              (f"{p}.mlp.up_proj.weight", (c.inter, H), ("fan", H, 1.0)),
              (f"{p}.mlp.down_proj.weight", (H, c.inter), ("fan", c.inter, 1.0)),
              (f"{p}.self_attn_layer_scale.scale", (H,), ("normal", 0.02, 0.1)),
              (f"{p}.mlp_layer_scale.scale", (H,), ("normal", 0.02, 0.1))]
    for u, r in enumerate(c.up_ratios):
        p = f"decoder.upsample.{u}"
        s += [(f"{p}.0.conv.weight", (LAT, LAT, r), ("fan", LAT, 1.0)),
              (f"{p}.0.conv.bias", (LAT,), ("normal", 0.02)),
              (f"{p}.1.dwconv.conv.weight", (LAT, 1, 7), ("fan", 7, 1.0)),
              (f"{p}.1.dwconv.conv.bias", (LAT,), ("normal", 0.02)),
              (f"{p}.1.norm.weight", (LAT,), ("gamma",)),
              (f"{p}.1.norm.bias", (LAT,), ("normal", 0.02)),
              (f"{p}.1.pwconv1.weight", (4 * LAT, LAT), ("fan", LAT, 1.0)),
              (f"{p}.1.pwconv1.bias", (4 * LAT,), ("normal", 0.02)),
              (f"{p}.1.pwconv2.weight", (LAT, 4 * LAT), ("fan", 4 * LAT, 1.0)),
              (f"{p}.1.pwconv2.bias", (LAT,), ("normal", 0.02)),
              (f"{p}.1.gamma", (LAT,), ("normal", 0.02, 0.1))]
    C = c.decoder_dim
    s.append(("decoder.decoder.0.conv.weight", (C, LAT, 7), ("fan", LAT * 7, 1.0)))
    s.append(("decoder.decoder.0.conv.bias", (C,), ("normal", 0.02)))
    for i, r in enumerate(c.rates):
        p = f"decoder.decoder.{i + 1}.block"
        Co = C // 2
        s += [(f"{p}.0.alpha", (C,), ("normal", 0.1)), (f"{p}.0.beta", (C,), ("normal", 0.1)),
              (f"{p}.1.conv.weight", (C, Co, 2 * r), ("fan", C * 2, 1.0)),
              (f"{p}.1.conv.bias", (Co,), ("normal", 0.02))]
        for ru in range(3):
            q = f"{p}.{ru + 2}"
            s += [(f"{q}.act1.alpha", (Co,), ("normal", 0.1)), (f"{q}.act1.beta", (Co,), ("normal", 0.1)),
                  (f"{q}.conv1.conv.weight", (Co, Co, 7), ("fan", Co * 7, 0.5)),
                  (f"{q}.conv1.conv.bias", (Co,), ("normal", 0.02)),
                  (f"{q}.act2.alpha", (Co,), ("normal", 0.1)), (f"{q}.act2.beta", (Co,), ("normal", 0.1)),
                  (f"{q}.conv2.conv.weight", (Co, Co, 1), ("fan", Co, 0.5)),
                  (f"{q}.conv2.conv.bias", (Co,), ("normal", 0.02))]
        C = Co
    n = len(c.rates)
    s += [(f"decoder.decoder.{n + 1}.alpha", (C,), ("normal", 0.1)),
          (f"decoder.decoder.{n + 1}.beta", (C,), ("normal", 0.1)),
          (f"decoder.decoder.{n + 2}.conv.weight", (1, C, 7), ("fan", C * 7, 0.1)),
          (f"decoder.decoder.{n + 2}.conv.bias", (1,), ("normal", 0.01))]
    return s


def make_codec_weights(cfg: CodecConfig, seed: int = 0) -> dict:
    """Seed-0 codec decoder weights (f32): codebooks ~N(0, 1) with cluster
    usage in [0.5, 2), convs/linears ~N(0, gain^2/fan_in), SnakeBeta log-params
    ~N(0, 0.1), layer scales / ConvNeXt gammas ~0.1 so every branch matters."""
    def one(spec):
        name, shape, init = spec
        kind = init[0]
        if kind == "normal":
            mean = init[2] if len(init) > 2 else 0.0
            a = _normal(seed, name, shape, init[1], mean)
        elif kind == "fan":
            a = _normal(seed, name, shape, init[2] / np.sqrt(init[1]))
        elif kind == "gamma":
            a = _normal(seed, name, shape, 0.1, 1.0)
        elif kind == "usage":
            a = _rng(seed, name).uniform(0.5, 2.0, shape).astype(np.float32)
        else:
            raise ValueError(kind)
        return name, np.ascontiguousarray(a, dtype=np.float32)
    return _parallel(one, codec_tensor_specs(cfg))


@dataclass
class CodecEncoderConfig:
    """Speech-tokenizer encoder of the voice-clone path
    (codec/config.rs:79-121, built by config.rs:136-346).  The tokenizer's
    config.json is not available, so these dims are the Mimi-style shape the
    12 Hz tokenizer is published with: 64 filters, ratios [8, 6, 5, 4]
    (960 samples per 25 Hz step, then a stride-2 downsample to 12.5 Hz),
    hidden 512, 8 transformer layers of 8 x 64 heads, MLP 2048, 32 codebooks
    (1 semantic) of 2048 x 256."""
    audio_channels: int = 1
    num_filters: int = 64
    kernel_size: int = 7
    residual_kernel_size: int = 3
    last_kernel_size: int = 3
    compress: int = 2
    upsampling_ratios: tuple = (8, 6, 5, 4)
    hidden: int = 512
    n_layers: int = 8
    n_heads: int = 8
    n_kv: int = 8
    head_dim: int = 64
    inter: int = 2048
    norm_eps: float = 1e-5
    theta: float = 1e4
    layer_scale: float = 0.01
    attention_bias: bool = False
    codebook_size: int = 2048
    vq_dim: int = 256
    n_q: int = 32
    n_semantic: int = 1
    downsample_factor: int = 2  # round(sampling_rate * encode_downsample_rate / (prod(ratios) * input_rate))

    def small(self, **kw):
        """A reduced encoder for fast CPU tests (same structure)."""
        d = dict(num_filters=16, upsampling_ratios=(4, 3), hidden=64, n_layers=2, n_heads=4, n_kv=2,
                 head_dim=16, inter=128, codebook_size=64, vq_dim=32, n_q=4, n_semantic=1)
        d.update(kw)
        return replace(self, **d)

    def frames(self, n: int) -> int:
        """Codec frames the encoder emits for n samples (conv.rs:44-64 lengths)."""
        def conv_len(L, k, stride):
            pt = max(k - stride, 0)
            padded = L + pt
            missing = max(k - padded, 0)
            extra = missing if missing > 0 else (stride - (padded - k) % stride) % stride
            return (padded + extra - k) // stride + 1
        L = conv_len(n, self.kernel_size, 1)
        for r in reversed(self.upsampling_ratios):
            L = conv_len(L, 2 * r, r)
        L = conv_len(L, self.last_kernel_size, 1)
        return conv_len(L, 2 * self.downsample_factor, 2)


def codec_encoder_tensor_specs(c: CodecEncoderConfig):
    """(name, shape, init) of the encoder tensors, named by the reference's
    module paths (encoder.rs:20-110)."""
    s = []
    p = "encoder.encoder.layers"
    s.append((f"{p}.0.conv.weight", (c.num_filters, c.audio_channels, c.kernel_size),
              ("fan", c.audio_channels * c.kernel_size, 1.0)))
    s.append((f"{p}.0.conv.bias", (c.num_filters,), ("normal", 0.02)))
    li, scale = 1, 1
    for r in reversed(c.upsampling_ratios):
        C = scale * c.num_filters
        hid = C // c.compress
        s += [(f"{p}.{li}.conv_in.conv.weight", (hid, C, c.residual_kernel_size),
               ("fan", C * c.residual_kernel_size, 1.0)),
              (f"{p}.{li}.conv_in.conv.bias", (hid,), ("normal", 0.02)),
              (f"{p}.{li}.conv_out.conv.weight", (C, hid, 1), ("fan", hid, 0.5)),
              (f"{p}.{li}.conv_out.conv.bias", (C,), ("normal", 0.02))]
        s += [(f"{p}.{li + 2}.conv.weight", (2 * C, C, 2 * r), ("fan", C * 2 * r, 1.0)),
              (f"{p}.{li + 2}.conv.bias", (2 * C,), ("normal", 0.02))]
        li += 3  # resnet, activation, downsample conv
        scale *= 2
    li += 1  # final activation
    s += [(f"{p}.{li}.conv.weight", (c.hidden, scale * c.num_filters, c.last_kernel_size),
           ("fan", scale * c.num_filters * c.last_kernel_size, 1.0)),
          (f"{p}.{li}.conv.bias", (c.hidden,), ("normal", 0.02))]
    H, qd, kd = c.hidden, c.n_heads * c.head_dim, c.n_kv * c.head_dim
    for l in range(c.n_layers):
        q = f"encoder.encoder_transformer.layers.{l}"
        s += [(f"{q}.input_layernorm.weight", (H,), ("gamma",)), (f"{q}.input_layernorm.bias", (H,), ("normal", 0.02)),
              (f"{q}.post_attention_layernorm.weight", (H,), ("gamma",)),
              (f"{q}.post_attention_layernorm.bias", (H,), ("normal", 0.02)),
              (f"{q}.self_attn.q_proj.weight", (qd, H), ("fan", H, 1.0)),
              (f"{q}.self_attn.k_proj.weight", (kd, H), ("fan", H, 1.0)),
              (f"{q}.self_attn.v_proj.weight", (kd, H), ("fan", H, 1.0)),
              (f"{q}.self_attn.o_proj.weight", (H, qd), ("fan", qd, 1.0)),
              (f"{q}.self_attn_layer_scale.scale", (H,), ("normal", 0.02, c.layer_scale * 10)),
              (f"{q}.mlp_layer_scale.scale", (H,), ("normal", 0.02, c.layer_scale * 10)),
              (f"{q}.mlp.fc1.weight", (c.inter, H), ("fan", H, 1.0)),
              (f"{q}.mlp.fc2.weight", (H, c.inter), ("fan", c.inter, 1.0))]
        if c.attention_bias:
            s += [(f"{q}.self_attn.{n}_proj.bias", (qd if n == "q" else (H if n == "o" else kd),), ("normal", 0.02))
                  for n in ("q", "k", "v", "o")]
    s.append(("encoder.downsample.conv.weight", (H, H, 2 * c.downsample_factor),
              ("fan", H * 2 * c.downsample_factor, 1.0)))
    for grp, n in (("semantic", c.n_semantic), ("acoustic", c.n_q - c.n_semantic)):
        q = f"encoder.quantizer.{grp}_residual_vector_quantizer"
        s.append((f"{q}.input_proj.weight", (c.vq_dim, H, 1), ("fan", H, 1.0)))
        for j in range(n):
            s += [(f"{q}.layers.{j}.codebook.embed_sum", (c.codebook_size, c.vq_dim), ("normal", 1.0)),
                  (f"{q}.layers.{j}.codebook.cluster_usage", (c.codebook_size,), ("usage",))]
    return s


def make_codec_encoder_weights(cfg: CodecEncoderConfig, seed: int = 0) -> dict:
    """Seeded encoder weights (f32), initialised like make_codec_weights
    (convs / linears ~N(0, gain^2 / fan_in), LayerNorm gains ~N(1, 0.1),
    codebooks ~N(0, 1) with usage in [0.5, 2))."""
    def one(spec):
        name, shape, init = spec
        kind = init[0]
        if kind == "normal":
            a = _normal(seed, name, shape, init[1], init[2] if len(init) > 2 else 0.0)
        elif kind == "fan":
            a = _normal(seed, name, shape, init[2] / np.sqrt(init[1]))
        elif kind == "gamma":
            a = _normal(seed, name, shape, 0.1, 1.0)
        elif kind == "usage":
            a = _rng(seed, name).uniform(0.5, 2.0, shape).astype(np.float32)
        else:
            raise ValueError(kind)
        return name, np.ascontiguousarray(a, dtype=np.float32)
    return _parallel(one, codec_encoder_tensor_specs(cfg))


@dataclass
class SpeakerEncoderConfig:
    """ECAPA-TDNN speaker encoder of the voice-clone path: the reference's own
    defaults (model/speaker/config.rs:18-32)."""
    mel_dim: int = 128
    enc_dim: int = 1024
    enc_channels: tuple = (512, 512, 512, 512, 1536)
    enc_kernel_sizes: tuple = (5, 3, 3, 3, 1)
    enc_dilations: tuple = (1, 2, 3, 4, 1)
    enc_attention_channels: int = 128
    enc_res2net_scale: int = 8
    enc_se_channels: int = 128
    sample_rate: int = 24000

    def small(self, **kw):
        """A reduced encoder for fast CPU tests (same structure)."""
        d = dict(mel_dim=32, enc_dim=48, enc_channels=(32, 32, 32, 32, 96), enc_attention_channels=16,
                 enc_res2net_scale=4, enc_se_channels=8)
        d.update(kw)
        return replace(self, **d)

    def frames(self, n: int) -> int:
        """Mel frames for n samples (feature.rs:92-115: pad 384 each side, hop 256)."""
        return (n + 768 - 1024) // 256 + 1


def speaker_tensor_specs(c: SpeakerEncoderConfig):
    """(name, shape, init) of the speaker encoder tensors: 'speaker_encoder.'
    + the reference's module paths (speaker/weights.rs:73, network/*.rs)."""
    p = "speaker_encoder"
    s = []

    def conv(name, co, ci, k):
        s.extend([(f"{name}.weight", (co, ci, k), ("fan", ci * k, 1.0)), (f"{name}.bias", (co,), ("normal", 0.02))])

    ch, ks, dil = c.enc_channels, c.enc_kernel_sizes, c.enc_dilations
    conv(f"{p}.blocks.0.conv", ch[0], c.mel_dim, ks[0])
    for i in range(1, 4):
        b = f"{p}.blocks.{i}"
        C, cs = ch[i], ch[i] // c.enc_res2net_scale
        conv(f"{b}.tdnn1.conv", C, C, 1)
        for j in range(c.enc_res2net_scale - 1):
            conv(f"{b}.res2net_block.blocks.{j}.conv", cs, cs, ks[i])
        conv(f"{b}.tdnn2.conv", C, C, 1)
        conv(f"{b}.se_block.conv1", c.enc_se_channels, C, 1)
        conv(f"{b}.se_block.conv2", C, c.enc_se_channels, 1)
    conv(f"{p}.mfa.conv", ch[4], sum(ch[1:4]), ks[4])
    conv(f"{p}.asp.tdnn.conv", c.enc_attention_channels, 3 * ch[4], 1)
    conv(f"{p}.asp.conv", ch[4], c.enc_attention_channels, 1)
    conv(f"{p}.fc", c.enc_dim, 2 * ch[4], 1)
    return s


def make_speaker_weights(cfg: SpeakerEncoderConfig, seed: int = 0) -> dict:
    """Seeded speaker encoder weights (f32), convs ~N(0, 1/fan_in)."""
    def one(spec):
        name, shape, init = spec
        if init[0] == "normal":
            a = _normal(seed, name, shape, init[1])
        else:
            a = _normal(seed, name, shape, init[2] / np.sqrt(init[1]))
        return name, np.ascontiguousarray(a, dtype=np.float32)
    return _parallel(one, speaker_tensor_specs(cfg))


def synthetic_talker_inputs(cfg: TalkerConfig, S: int, seed: int = 0):
    """Prompt embeddings [S, H], trailing text [1, H] and pad embed [H]:
    stand-ins for the host-side session seed (compiler/session_seed.rs)."""
    H = cfg.talker.hidden
    g = np.random.default_rng([seed, 7])
    prompt = (g.standard_normal((S, H), dtype=np.float32) * 0.5).astype(np.float32)
    trailing = (g.standard_normal((1, H), dtype=np.float32) * 0.5).astype(np.float32)
    pad = (g.standard_normal((H,), dtype=np.float32) * 0.5).astype(np.float32)
    return prompt, trailing, pad


def teacher_codes(n_frames: int, n_groups: int = 16, hi: int = 2048, seed: int = 0):
    """Teacher-forced codes [n_frames, n_groups] uniform in [0, hi)."""
    g = np.random.default_rng([seed, 11])
    return g.integers(0, hi, size=(n_frames, n_groups), dtype=np.int64)

"""ctypes binding of the CPU oracle (liboracle.so) — TEST INFRASTRUCTURE ONLY.

Imported only by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
leg, as the checker.  The product (tts-rs_b200/) never imports this module.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None

F = C.POINTER(C.c_float)
I64 = C.POINTER(C.c_int64)


class LMCfg(C.Structure):
    _fields_ = [("hidden", C.c_int), ("inter", C.c_int), ("n_layers", C.c_int),
                ("n_heads", C.c_int), ("n_kv", C.c_int), ("head_dim", C.c_int),
                ("eps", C.c_float), ("theta", C.c_float)]


class Layer(C.Structure):
    _fields_ = [(n, F) for n in ("in_norm", "post_norm", "wq", "wk", "wv", "wo",
                                 "q_norm", "k_norm", "w_gate", "w_up", "w_down")]


class Stack(C.Structure):
    _fields_ = [("cfg", LMCfg), ("layers", C.POINTER(Layer)), ("final_norm", F)]


class KV(C.Structure):
    _fields_ = [("k", F), ("v", F), ("len", C.c_int), ("cap", C.c_int),
                ("n_kv", C.c_int), ("head_dim", C.c_int)]


class Sampling(C.Structure):
    _fields_ = [("do_sample", C.c_int), ("temperature", C.c_float), ("top_k", C.c_int),
                ("top_p", C.c_float), ("repetition_penalty", C.c_float)]


class Talker(C.Structure):
    _fields_ = [("talker", Stack), ("predictor", Stack), ("codec_head", F),
                ("talker_codec_emb", F), ("cp_codec_emb", C.POINTER(F)),
                ("lm_heads", C.POINTER(F)), ("vocab", C.c_int), ("cp_vocab", C.c_int),
                ("n_groups", C.c_int)]


class ResUnit(C.Structure):
    _fields_ = [(n, F) for n in ("w1", "b1", "w2", "b2", "a1_alpha", "a1_beta",
                                 "a2_alpha", "a2_beta")]


class WaveStage(C.Structure):
    _fields_ = [("snake_alpha", F), ("snake_beta", F), ("wt", F), ("bt", F),
                ("ru", ResUnit * 3)]


class ConvNeXt(C.Structure):
    _fields_ = [(n, F) for n in ("wt", "bt", "dw_w", "dw_b", "ln_w", "ln_b", "pw1_w",
                                 "pw1_b", "pw2_w", "pw2_b", "gamma")]


class CodecLayer(C.Structure):
    _fields_ = [(n, F) for n in ("in_norm", "post_norm", "wq", "wk", "wv", "wo",
                                 "attn_scale", "mlp_scale", "w_gate", "w_up", "w_down")]


class Codec(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("n_q", "n_semantic", "codebook_size", "codebook_dim",
                                       "latent", "decoder_dim", "hidden", "inter", "n_layers",
                                       "n_heads", "n_kv", "head_dim")] + \
               [("eps", C.c_float), ("theta", C.c_float), ("n_up", C.c_int),
                ("up_ratio", C.c_int * 4), ("n_stage", C.c_int), ("rates", C.c_int * 8),
                ("emb_sum", C.POINTER(F)), ("usage", C.POINTER(F)),
                ("first_out_proj", F), ("rest_out_proj", F), ("pre_conv_w", F),
                ("pre_conv_b", F), ("in_proj_w", F), ("in_proj_b", F), ("out_proj_w", F),
                ("out_proj_b", F), ("final_norm", F), ("layers", C.POINTER(CodecLayer)),
                ("up", C.POINTER(ConvNeXt)), ("in_conv_w", F), ("in_conv_b", F),
                ("stages", C.POINTER(WaveStage)), ("out_alpha", F), ("out_beta", F),
                ("out_conv_w", F), ("out_conv_b", F)]


class Conv(C.Structure):
    _fields_ = [("w", F), ("b", F), ("ci", C.c_int), ("co", C.c_int), ("k", C.c_int), ("stride", C.c_int)]


class EncLayer(C.Structure):
    _fields_ = [(n, F) for n in ("ln1_w", "ln1_b", "ln2_w", "ln2_b", "wq", "bq", "wk", "bk", "wv", "bv",
                                 "wo", "bo", "attn_scale", "mlp_scale", "fc1", "fc2")]


class EncRvq(C.Structure):
    _fields_ = [("in_proj", F), ("embed_sum", C.POINTER(F)), ("usage", C.POINTER(F)), ("n_layers", C.c_int)]


class CodecEncoder(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("hidden", "n_layers", "n_heads", "n_kv", "head_dim", "inter",
                                       "codebook_size", "vq_dim")] + \
               [("norm_eps", C.c_float), ("theta", C.c_float), ("n_stages", C.c_int), ("in_conv", Conv),
                ("res_in", Conv * 8), ("res_out", Conv * 8), ("down", Conv * 8), ("out_conv", Conv),
                ("layers", C.POINTER(EncLayer)), ("downsample", Conv), ("semantic", EncRvq),
                ("acoustic", EncRvq)]


class Tdnn(C.Structure):
    _fields_ = [("w", F), ("b", F), ("ci", C.c_int), ("co", C.c_int), ("k", C.c_int), ("dil", C.c_int)]


class SeBlock(C.Structure):
    _fields_ = [("tdnn1", Tdnn), ("tdnn2", Tdnn), ("res", Tdnn * 15), ("scale", C.c_int),
                ("se_w1", F), ("se_b1", F), ("se_w2", F), ("se_b2", F), ("se_ch", C.c_int)]


class Speaker(C.Structure):
    _fields_ = [("mel_dim", C.c_int), ("enc_dim", C.c_int), ("sample_rate", C.c_int), ("channels", C.c_int * 5),
                ("block0", Tdnn), ("se", SeBlock * 3), ("mfa", Tdnn), ("asp_tdnn", Tdnn),
                ("asp_w", F), ("asp_b", F), ("fc_w", F), ("fc_b", F)]


_LIBS = {}
_VARIANT = "liboracle.so"


def use_library(name):
    """Select the oracle build later calls go through: "liboracle.so" (the
    oracle) or "liboracle_wide.so" (the same restatement with double
    accumulation in its dot products, for noise-floor measurements).
    Returns the previous selection."""
    global _VARIANT, _LIB
    prev, _VARIANT = _VARIANT, name
    _LIB = _LIBS.get(name)
    return prev


def lib():
    """Load the selected oracle build, running make if it is missing."""
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, _VARIANT)
        if not os.path.exists(path):
            subprocess.run(["make", "-C", _HERE], check=True, capture_output=True)
        L = C.CDLL(path)
        L.orc_bf16_round.restype = C.c_float
        L.orc_bf16_round.argtypes = [C.c_float]
        L.orc_sample_token.restype = C.c_int64
        L.orc_sample_token.argtypes = [F, C.c_int, C.POINTER(Sampling), I64, C.c_int, C.c_float]
        L.orc_apply_repetition_penalty.argtypes = [F, C.c_int, I64, C.c_int, C.c_float]
        L.orc_repetition_penalty_enabled.argtypes = [C.c_float]
        L.orc_build_suppress_ids.argtypes = [C.c_int, C.c_int64, I64]
        L.orc_kv_forward.argtypes = [C.POINTER(KV), F, F, C.c_int, F, F]
        L.orc_kv_reset_preserve.argtypes = [C.POINTER(KV)]
        L.orc_stack_forward.argtypes = [C.POINTER(Stack), C.POINTER(KV), F, C.c_int, F]
        L.orc_linear.argtypes = [F, F, F, C.c_int, C.c_int, C.c_int, F]
        L.orc_text_project.argtypes = [F, F, F, F, F, C.c_int, C.c_int, I64, C.c_int, F]
        L.orc_gen_start.restype = C.c_void_p
        L.orc_gen_start.argtypes = [C.POINTER(Talker), F, C.c_int, F, C.c_int, F,
                                    C.POINTER(Sampling), C.POINTER(Sampling), C.c_int,
                                    C.c_int64, I64, C.c_int, C.c_int64, F,
                                    C.POINTER(C.c_int)]
        L.orc_gen_step.argtypes = [C.c_void_p, I64, F, F, F, F]
        L.orc_gen_num_frames.argtypes = [C.c_void_p]
        L.orc_gen_codes.argtypes = [C.c_void_p, I64]
        L.orc_gen_free.argtypes = [C.c_void_p]
        L.orc_predict_frame.argtypes = [C.POINTER(Talker), F, C.c_int64, C.POINTER(Sampling),
                                        I64, F, I64, F]
        L.orc_codec_group_embedding.argtypes = [C.POINTER(Talker), I64, F, F]
        L.orc_codec_out_len.restype = C.c_int64
        L.orc_codec_out_len.argtypes = [C.POINTER(Codec), C.c_int]
        L.orc_codec_decode.argtypes = [C.POINTER(Codec), I64, C.c_int, C.c_int, F]
        L.orc_codec_decode_tap.restype = C.c_int64
        L.orc_codec_decode_tap.argtypes = [C.POINTER(Codec), I64, C.c_int, C.c_int, F]
        L.orc_pad_1d.argtypes = [F, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, F]
        L.orc_conv1d_padding.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int,
                                         C.POINTER(C.c_int), C.POINTER(C.c_int)]
        L.orc_to_pcm.argtypes = [F, C.c_int64, C.POINTER(C.c_int16)]
        L.orc_speaker_mel.argtypes = [F, C.c_int, C.c_int, C.c_int, F, C.c_int]
        L.orc_speaker_forward.argtypes = [C.POINTER(Speaker), F, C.c_int, F]
        L.orc_speaker_embed.argtypes = [C.POINTER(Speaker), F, C.c_int, F]
        L.orc_codec_encoder_hidden.argtypes = [C.POINTER(CodecEncoder), F, C.c_int, F, C.c_int]
        L.orc_codec_encode.argtypes = [C.POINTER(CodecEncoder), F, C.c_int, C.c_int, I64, C.c_int]
        L.orc_rvq_encode.argtypes = [C.POINTER(F), C.POINTER(F), C.c_int, C.c_int, C.c_int, F, C.c_int, I64]
        L.orc_sdpa.argtypes = [F, F, F, C.POINTER(C.c_uint8), C.c_int, C.c_int, C.c_int,
                               C.c_int, C.c_float, F]
        L.orc_set_threads.argtypes = [C.c_int]
        L.orc_get_threads.restype = C.c_int
        _LIB = L
        _LIBS[_VARIANT] = L
    return _LIB


def fp(a):
    return None if a is None else a.ctypes.data_as(F)


def ip(a):
    return None if a is None else a.ctypes.data_as(I64)


def bf16_round(a):
    """Round f32 values to the nearest bf16 (ties to even), kept as f32."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    u = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    return u.view(np.float32)


def f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def sampling(do_sample=False, temperature=1.0, top_k=0, top_p=1.0, repetition_penalty=0.0):
    return Sampling(int(do_sample), float(temperature), int(top_k or 0), float(top_p),
                    float(repetition_penalty if repetition_penalty is not None else 0.0))


class OracleTalker:
    """Talker + code predictor bound to the oracle; keeps the numpy weights
    alive for as long as the ctypes structs point at them."""

    def __init__(self, cfg, weights: dict):
        self.cfg = cfg
        self.w = {k: f32(v) for k, v in weights.items()}
        self._keep = []
        self.s = Talker()
        self.s.talker = self._stack("talker.model", cfg.talker)
        self.s.predictor = self._stack("talker.code_predictor.model", cfg.predictor)
        self.s.codec_head = fp(self.w["talker.codec_head.weight"])
        self.s.talker_codec_emb = fp(self.w["talker.model.codec_embedding.weight"])
        G = cfg.n_groups
        emb = (F * (G - 1))(*[fp(self.w[f"talker.code_predictor.model.codec_embedding.{j}.weight"])
                              for j in range(G - 1)])
        heads = (F * (G - 1))(*[fp(self.w[f"talker.code_predictor.lm_head.{j}.weight"])
                                for j in range(G - 1)])
        self._keep += [emb, heads]
        self.s.cp_codec_emb = C.cast(emb, C.POINTER(F))
        self.s.lm_heads = C.cast(heads, C.POINTER(F))
        self.s.vocab = cfg.talker.vocab
        self.s.cp_vocab = cfg.predictor.vocab
        self.s.n_groups = G

    def _stack(self, prefix, c):
        layers = (Layer * c.n_layers)()
        for l in range(c.n_layers):
            p = f"{prefix}.layers.{l}"
            w = self.w
            layers[l] = Layer(fp(w[f"{p}.input_layernorm.weight"]),
                              fp(w[f"{p}.post_attention_layernorm.weight"]),
                              fp(w[f"{p}.self_attn.q_proj.weight"]), fp(w[f"{p}.self_attn.k_proj.weight"]),
                              fp(w[f"{p}.self_attn.v_proj.weight"]), fp(w[f"{p}.self_attn.o_proj.weight"]),
                              fp(w[f"{p}.self_attn.q_norm.weight"]), fp(w[f"{p}.self_attn.k_norm.weight"]),
                              fp(w[f"{p}.mlp.gate_proj.weight"]), fp(w[f"{p}.mlp.up_proj.weight"]),
                              fp(w[f"{p}.mlp.down_proj.weight"]))
        self._keep.append(layers)
        st = Stack(LMCfg(c.hidden, c.inter, c.n_layers, c.n_heads, c.n_kv, c.head_dim,
                         c.eps, c.theta), C.cast(layers, C.POINTER(Layer)),
                   fp(self.w[f"{prefix}.norm.weight"]))
        return st

    # --- dense batch-1 caches ------------------------------------------------
    def make_caches(self, which="talker", cap=4096):
        c = self.cfg.talker if which == "talker" else self.cfg.predictor
        mems, kvs = [], (KV * c.n_layers)()
        for l in range(c.n_layers):
            k = np.zeros((c.n_kv, cap, c.head_dim), np.float32)
            v = np.zeros_like(k)
            mems.append((k, v))
            kvs[l] = KV(fp(k), fp(v), 0, cap, c.n_kv, c.head_dim)
        return kvs, mems

    def stack_forward(self, which, kvs, x):
        x = f32(x)
        S = x.shape[0]
        st = self.s.talker if which == "talker" else self.s.predictor
        H = st.cfg.hidden
        out = np.zeros((S, H), np.float32)
        lib().orc_stack_forward(C.byref(st), kvs, fp(x), S, fp(out))
        return out

    def text_project(self, ids):
        """project_text_ids (session_seed.rs:668-679): [n][hidden] bf16-valued rows."""
        w = self.w
        emb = f32(w["talker.model.text_embedding.weight"])
        Ht = emb.shape[1]
        H = self.cfg.talker.hidden
        ids = np.ascontiguousarray(ids, np.int64)
        out = np.zeros((len(ids), H), np.float32)
        keep = [f32(w[f"talker.text_projection.linear_fc{i}.{k}"]) for i in (1, 2) for k in ("weight", "bias")]
        lib().orc_text_project(fp(emb), fp(keep[0]), fp(keep[1]), fp(keep[2]), fp(keep[3]), Ht, H,
                               ids.ctypes.data_as(I64), len(ids), fp(out))
        return out

    def session_seed(self, text_ids, controls, leading_ids=None):
        """build_non_streaming_seed (session_seed.rs:151-215): (inputs_embeds
        [rows][hidden], tts_pad embedding).  Text rows are project_text_ids
        (:668-679), codec rows the talker codec_embedding (:681-688); every
        sum is rounded to bf16, the talker dtype (the reference adds bf16
        tensors)."""
        text_ids = np.asarray(text_ids, np.int64)
        cp = np.asarray(controls["codec_prefix_ids"], np.int64)
        if len(text_ids) < 8 or len(cp) < 2:
            raise ValueError("need >= 8 text ids and >= 2 codec prefix ids")
        E = f32(self.w["talker.model.codec_embedding.weight"])
        bos, eos, pad = self.text_project([controls["tts_bos_token_id"], controls["tts_eos_token_id"],
                                           controls["tts_pad_token_id"]])
        role = self.text_project(text_ids[:3])
        body = self.text_project(text_ids[3:len(text_ids) - 5])
        n = len(cp)
        prefix = np.concatenate([np.repeat(pad[None], max(n - 2, 0), 0), bos[None]]) + E[cp[:n - 1]]
        segs = [] if leading_ids is None else [self.text_project(np.asarray(leading_ids, np.int64))]
        segs += [role, prefix, body + E[controls["codec_pad_id"]], (eos + E[controls["codec_pad_id"]])[None],
                 (pad + E[controls["codec_bos_id"]])[None]]
        return bf16_round(np.concatenate(segs)), pad

    def ref_codec_sum(self, ref_codes):
        """sum_ref_codec_embeddings (session_seed.rs:602-641): codes
        [groups][T] -> [T][hidden], group 0 through the talker codec
        embedding, group g >= 1 through the predictor's embedding g - 1
        (:643-655), added group by group as bf16 tensors."""
        ref_codes = np.asarray(ref_codes, np.int64)
        G = self.cfg.n_groups
        if ref_codes.ndim != 2 or ref_codes.shape[0] != G or ref_codes.shape[1] == 0:
            raise ValueError(f"reference codes must be [{G}, T > 0]")
        s = f32(self.w["talker.model.codec_embedding.weight"])[ref_codes[0]]
        for g in range(1, G):
            s = bf16_round(s + f32(self.w[f"talker.code_predictor.model.codec_embedding.{g - 1}.weight"])[ref_codes[g]])
        return s

    def session_seed_voice_clone(self, text_ids, controls, speaker, ref_text_ids=None, ref_codes=None):
        """build_voice_clone_seed (session_seed.rs:248-322): (inputs_embeds,
        trailing_text_hidden, tts_pad embedding).  The codec prefix is
        voice_clone_codec_prefix (:538-584): [pad + E(tag) per tag id, pad +
        speaker x-vector (cast to bf16), bos + E(codec_pad)].  Without
        reference text (x-vector only) the seed ends with P(body[0]) +
        E(codec_bos) (:474-493) and the trailing text is P(body[1..]) then
        P(eos) (:495-512); with it, build_voice_clone_icl_seed (:324-396):
        P(reference body + target body + eos) aligned with [E(codec_bos),
        summed reference frames], the longer side's excess becoming the
        trailing text (or pad rows filling the text side, trailing P(pad))."""
        text_ids = np.asarray(text_ids, np.int64)
        cp = np.asarray(controls["codec_prefix_ids"], np.int64)
        H = self.cfg.talker.hidden
        spk = bf16_round(np.asarray(speaker, np.float32).reshape(-1))
        if len(text_ids) < 8 or len(cp) < 2 or spk.shape != (H,):
            raise ValueError("need >= 8 text ids, >= 2 codec prefix ids and a [hidden] speaker embedding")
        E = f32(self.w["talker.model.codec_embedding.weight"])
        bos, eos, pad = self.text_project([controls["tts_bos_token_id"], controls["tts_eos_token_id"],
                                           controls["tts_pad_token_id"]])
        role = self.text_project(text_ids[:3])
        n = len(cp)
        codec_prefix = np.concatenate([E[cp[:n - 2]], spk[None], E[controls["codec_pad_id"]][None]])
        prefix_text = np.concatenate([np.repeat(pad[None], n - 1, 0), bos[None]])
        prefix = bf16_round(prefix_text + codec_prefix)
        body_ids = text_ids[3:len(text_ids) - 5]
        if ref_text_ids is None:
            segs = [role, prefix]
            if len(body_ids):
                segs.append(bf16_round(self.text_project(body_ids[:1]) + E[controls["codec_bos_id"]]))
            rest = body_ids[1:]
            trailing = eos[None] if len(rest) == 0 else np.concatenate([self.text_project(rest), eos[None]])
            return np.concatenate(segs), trailing, pad
        ref_text_ids = np.asarray(ref_text_ids, np.int64)
        if len(ref_text_ids) < 5 or ref_codes is None:
            raise ValueError("the in-context recipe needs >= 5 reference text ids and reference codes")
        all_ids = np.concatenate([ref_text_ids[3:len(ref_text_ids) - 2], body_ids,
                                  [controls["tts_eos_token_id"]]]).astype(np.int64)
        text = self.text_project(all_ids)
        codec = np.concatenate([E[controls["codec_bos_id"]][None], self.ref_codec_sum(ref_codes)])
        tl, cl = len(text), len(codec)
        if tl > cl:
            icl, trailing = bf16_round(text[:cl] + codec), text[cl:]
        else:
            icl = bf16_round(np.concatenate([text, np.repeat(pad[None], cl - tl, 0)]) + codec)
            trailing = pad[None]
        return np.concatenate([role, prefix, icl]), trailing, pad

    def codec_head(self, hidden):
        h = f32(hidden).reshape(-1, self.cfg.talker.hidden)
        out = np.zeros((h.shape[0], self.cfg.talker.vocab), np.float32)
        lib().orc_linear(fp(self.w["talker.codec_head.weight"]), None, fp(h), h.shape[0],
                         self.cfg.talker.hidden, self.cfg.talker.vocab, fp(out))
        return out

    def predict_frame(self, hidden, code0, samp=None, forced=None, u=None):
        G, V = self.cfg.n_groups, self.cfg.predictor.vocab
        codes = np.zeros(G, np.int64)
        logits = np.zeros((G - 1, V), np.float32)
        s = samp or sampling()
        fz = None if forced is None else np.ascontiguousarray(forced, np.int64)
        uu = None if u is None else f32(u)
        lib().orc_predict_frame(C.byref(self.s), fp(f32(hidden)), int(code0), C.byref(s),
                                ip(fz), fp(uu), ip(codes), fp(logits))
        return codes, logits

    def group_embedding(self, codes, extra=None):
        out = np.zeros(self.cfg.talker.hidden, np.float32)
        lib().orc_codec_group_embedding(C.byref(self.s), ip(np.ascontiguousarray(codes, np.int64)),
                                        fp(None if extra is None else f32(extra)), fp(out))
        return out


class OracleGenerator:
    """TalkerGenerator restatement (talker/infer/mod.rs:17-311)."""

    def __init__(self, talker: OracleTalker, prompt, trailing, pad, talker_s=None, cp_s=None,
                 max_new_tokens=64, eos=-1, suppress=None, forced_first=-1):
        self.t = talker
        self._in = [f32(prompt), f32(trailing), f32(pad)]
        self.ts = talker_s or sampling()
        self.cs = cp_s or sampling()
        sup = np.ascontiguousarray(suppress if suppress is not None else [], np.int64)
        self._sup = sup
        self.first_logits = np.zeros(talker.cfg.talker.vocab, np.float32)
        st = C.c_int(0)
        self.h = lib().orc_gen_start(C.byref(talker.s), fp(self._in[0]), self._in[0].shape[0],
                                     fp(self._in[1]), self._in[1].shape[0], fp(self._in[2]),
                                     C.byref(self.ts), C.byref(self.cs), int(max_new_tokens),
                                     int(eos), ip(sup) if len(sup) else None, len(sup),
                                     int(forced_first), fp(self.first_logits), C.byref(st))
        if st.value != 0:
            raise ValueError(f"oracle start failed: {st.value}")

    def step(self, forced=None, u=None):
        G = self.t.cfg.n_groups
        tl = np.zeros(self.t.cfg.talker.vocab, np.float32)
        cl = np.zeros((G - 1, self.t.cfg.predictor.vocab), np.float32)
        hid = np.zeros(self.t.cfg.talker.hidden, np.float32)
        fz = None if forced is None else np.ascontiguousarray(forced, np.int64)
        uu = None if u is None else f32(u)
        r = lib().orc_gen_step(self.h, ip(fz), fp(uu), fp(tl), fp(cl), fp(hid))
        return r, tl, cl, hid

    def codes(self):
        T = lib().orc_gen_num_frames(self.h)
        out = np.zeros((self.t.cfg.n_groups, T), np.int64)
        if T:
            lib().orc_gen_codes(self.h, ip(out))
        return out

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_gen_free(self.h)
            self.h = None


class OracleCodec:
    """Codec decoder restatement (codec/network/decoder.rs:250-278)."""

    def __init__(self, cfg, weights: dict):
        self.cfg = cfg
        w = {k: f32(v) for k, v in weights.items()}
        self.w = w
        self._keep = []
        c = Codec()
        for n in ("n_q", "n_semantic", "codebook_size", "codebook_dim", "latent", "decoder_dim",
                  "hidden", "inter", "n_layers", "n_heads", "n_kv", "head_dim"):
            setattr(c, n, getattr(cfg, n))
        c.eps, c.theta = cfg.eps, cfg.theta
        c.n_up = len(cfg.up_ratios)
        for i, r in enumerate(cfg.up_ratios):
            c.up_ratio[i] = r
        c.n_stage = len(cfg.rates)
        for i, r in enumerate(cfg.rates):
            c.rates[i] = r
        names = [f"decoder.quantizer.rvq_first.vq.layers.{i}._codebook" for i in range(cfg.n_semantic)] + \
                [f"decoder.quantizer.rvq_rest.vq.layers.{i}._codebook" for i in range(cfg.n_q - cfg.n_semantic)]
        es = (F * cfg.n_q)(*[fp(w[n + ".embedding_sum"]) for n in names])
        us = (F * cfg.n_q)(*[fp(w[n + ".cluster_usage"]) for n in names])
        self._keep += [es, us]
        c.emb_sum, c.usage = C.cast(es, C.POINTER(F)), C.cast(us, C.POINTER(F))
        c.first_out_proj = fp(w["decoder.quantizer.rvq_first.output_proj.weight"])
        c.rest_out_proj = fp(w["decoder.quantizer.rvq_rest.output_proj.weight"])
        c.pre_conv_w, c.pre_conv_b = fp(w["decoder.pre_conv.conv.weight"]), fp(w["decoder.pre_conv.conv.bias"])
        pt = "decoder.pre_transformer"
        c.in_proj_w, c.in_proj_b = fp(w[f"{pt}.input_proj.weight"]), fp(w[f"{pt}.input_proj.bias"])
        c.out_proj_w, c.out_proj_b = fp(w[f"{pt}.output_proj.weight"]), fp(w[f"{pt}.output_proj.bias"])
        c.final_norm = fp(w[f"{pt}.norm.weight"])
        layers = (CodecLayer * cfg.n_layers)()
        for l in range(cfg.n_layers):
            p = f"{pt}.layers.{l}"
            layers[l] = CodecLayer(*[fp(w[f"{p}.{n}"]) for n in (
                "input_layernorm.weight", "post_attention_layernorm.weight",
                "self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
                "self_attn.o_proj.weight", "self_attn_layer_scale.scale", "mlp_layer_scale.scale",
                "mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight")])
        ups = (ConvNeXt * len(cfg.up_ratios))()
        for u in range(len(cfg.up_ratios)):
            p = f"decoder.upsample.{u}"
            ups[u] = ConvNeXt(*[fp(w[f"{p}.{n}"]) for n in (
                "0.conv.weight", "0.conv.bias", "1.dwconv.conv.weight", "1.dwconv.conv.bias",
                "1.norm.weight", "1.norm.bias", "1.pwconv1.weight", "1.pwconv1.bias",
                "1.pwconv2.weight", "1.pwconv2.bias", "1.gamma")])
        stages = (WaveStage * len(cfg.rates))()
        for i in range(len(cfg.rates)):
            p = f"decoder.decoder.{i + 1}.block"
            st = WaveStage()
            st.snake_alpha, st.snake_beta = fp(w[f"{p}.0.alpha"]), fp(w[f"{p}.0.beta"])
            st.wt, st.bt = fp(w[f"{p}.1.conv.weight"]), fp(w[f"{p}.1.conv.bias"])
            for ru in range(3):
                q = f"{p}.{ru + 2}"
                st.ru[ru] = ResUnit(fp(w[f"{q}.conv1.conv.weight"]), fp(w[f"{q}.conv1.conv.bias"]),
                                    fp(w[f"{q}.conv2.conv.weight"]), fp(w[f"{q}.conv2.conv.bias"]),
                                    fp(w[f"{q}.act1.alpha"]), fp(w[f"{q}.act1.beta"]),
                                    fp(w[f"{q}.act2.alpha"]), fp(w[f"{q}.act2.beta"]))
            stages[i] = st
        self._keep += [layers, ups, stages]
        c.layers = C.cast(layers, C.POINTER(CodecLayer))
        c.up = C.cast(ups, C.POINTER(ConvNeXt))
        c.stages = C.cast(stages, C.POINTER(WaveStage))
        c.in_conv_w, c.in_conv_b = fp(w["decoder.decoder.0.conv.weight"]), fp(w["decoder.decoder.0.conv.bias"])
        n = len(cfg.rates)
        c.out_alpha, c.out_beta = fp(w[f"decoder.decoder.{n + 1}.alpha"]), fp(w[f"decoder.decoder.{n + 1}.beta"])
        c.out_conv_w = fp(w[f"decoder.decoder.{n + 2}.conv.weight"])
        c.out_conv_b = fp(w[f"decoder.decoder.{n + 2}.conv.bias"])
        self.s = c

    def out_len(self, T):
        return lib().orc_codec_out_len(C.byref(self.s), T)

    def decode(self, codes):
        codes = np.ascontiguousarray(codes, np.int64)
        B, _, T = codes.shape
        out = np.zeros((B, self.out_len(T)), np.float32)
        r = lib().orc_codec_decode(C.byref(self.s), ip(codes), B, T, fp(out))
        if r != 0:
            raise ValueError("oracle codec: invalid codes")
        return out

    def tap(self, codes, tap):
        codes = np.ascontiguousarray(codes, np.int64)
        T = codes.shape[-1]
        n = lib().orc_codec_decode_tap(C.byref(self.s), ip(codes), T, tap, None)
        out = np.zeros(n, np.float32)
        lib().orc_codec_decode_tap(C.byref(self.s), ip(codes), T, tap, fp(out))
        return out


class OracleCodecEncoder:
    """Speech-tokenizer encoder of the voice-clone path
    (Qwen3TtsAudioCodecEncoder::encode_reference_prefix, codec/network/
    encoder.rs:121-136): 24 kHz samples -> codes [n_valid][frames].  Weights
    are named by the reference's module paths (synthetic.codec_encoder_tensor_specs)."""

    def __init__(self, cfg, weights: dict):
        self.cfg = cfg
        w = {k: f32(v) for k, v in weights.items()}
        self.w = w
        self._keep = []
        e = CodecEncoder()
        for n in ("hidden", "n_layers", "n_heads", "n_kv", "head_dim", "inter", "codebook_size", "vq_dim"):
            setattr(e, n, getattr(cfg, n))
        e.norm_eps, e.theta = cfg.norm_eps, cfg.theta
        e.n_stages = len(cfg.upsampling_ratios)
        if e.n_stages > 8:
            raise ValueError("at most 8 encoder stages")
        p = "encoder.encoder.layers"

        def conv(name, ci, co, k, stride, bias=True):
            wt = w[f"{name}.weight"]
            assert wt.shape == (co, ci, k), (name, wt.shape)
            return Conv(fp(wt), fp(w[f"{name}.bias"]) if bias else None, ci, co, k, stride)

        e.in_conv = conv(f"{p}.0.conv", cfg.audio_channels, cfg.num_filters, cfg.kernel_size, 1)
        li, scale = 1, 1
        for s_, r in enumerate(reversed(cfg.upsampling_ratios)):
            Cc = scale * cfg.num_filters
            e.res_in[s_] = conv(f"{p}.{li}.conv_in.conv", Cc, Cc // cfg.compress, cfg.residual_kernel_size, 1)
            e.res_out[s_] = conv(f"{p}.{li}.conv_out.conv", Cc // cfg.compress, Cc, 1, 1)
            e.down[s_] = conv(f"{p}.{li + 2}.conv", Cc, 2 * Cc, 2 * r, r)
            li += 3
            scale *= 2
        e.out_conv = conv(f"{p}.{li + 1}.conv", scale * cfg.num_filters, cfg.hidden, cfg.last_kernel_size, 1)
        layers = (EncLayer * cfg.n_layers)()
        for l in range(cfg.n_layers):
            q = f"encoder.encoder_transformer.layers.{l}"
            g = lambda n: fp(w[f"{q}.{n}"]) if f"{q}.{n}" in w else None
            layers[l] = EncLayer(g("input_layernorm.weight"), g("input_layernorm.bias"),
                                 g("post_attention_layernorm.weight"), g("post_attention_layernorm.bias"),
                                 g("self_attn.q_proj.weight"), g("self_attn.q_proj.bias"),
                                 g("self_attn.k_proj.weight"), g("self_attn.k_proj.bias"),
                                 g("self_attn.v_proj.weight"), g("self_attn.v_proj.bias"),
                                 g("self_attn.o_proj.weight"), g("self_attn.o_proj.bias"),
                                 g("self_attn_layer_scale.scale"), g("mlp_layer_scale.scale"),
                                 g("mlp.fc1.weight"), g("mlp.fc2.weight"))
        self._keep.append(layers)
        e.layers = C.cast(layers, C.POINTER(EncLayer))
        e.downsample = conv("encoder.downsample.conv", cfg.hidden, cfg.hidden, 2 * cfg.downsample_factor, 2,
                            bias=False)
        for grp, n in (("semantic", cfg.n_semantic), ("acoustic", cfg.n_q - cfg.n_semantic)):
            q = f"encoder.quantizer.{grp}_residual_vector_quantizer"
            es = (F * max(n, 1))(*[fp(w[f"{q}.layers.{j}.codebook.embed_sum"]) for j in range(n)])
            us = (F * max(n, 1))(*[fp(w[f"{q}.layers.{j}.codebook.cluster_usage"]) for j in range(n)])
            self._keep += [es, us]
            setattr(e, grp, EncRvq(fp(w[f"{q}.input_proj.weight"]), C.cast(es, C.POINTER(F)),
                                   C.cast(us, C.POINTER(F)), n))
        self.e = e

    def encode(self, wave, n_valid=None):
        """wave [n] f32 -> codes [n_valid][frames] (n_valid defaults to all codebooks)."""
        wave = np.ascontiguousarray(wave, np.float32)
        n_valid = self.cfg.n_q if n_valid is None else n_valid
        T = self.cfg.frames(len(wave))
        codes = np.zeros((n_valid, T), np.int64)
        got = lib().orc_codec_encode(C.byref(self.e), fp(wave), len(wave), n_valid,
                                     codes.ctypes.data_as(I64), T)
        if got < 0:
            raise ValueError("bad encoder input")
        assert got == T, (got, T)
        return codes


def _encoder_hidden(self, wave):
    """The hidden [hidden][frames] the quantizers read (after the downsample)."""
    wave = np.ascontiguousarray(wave, np.float32)
    T = self.cfg.frames(len(wave))
    out = np.zeros((self.cfg.hidden, T), np.float32)
    if lib().orc_codec_encoder_hidden(C.byref(self.e), fp(wave), len(wave), fp(out), T) != T:
        raise ValueError("bad encoder input")
    return out


OracleCodecEncoder.hidden = _encoder_hidden


def rvq_encode(embed_sum, usage, x):
    """One residual vector quantizer's encode (encoder.rs:319-368) of x
    [vq][T]: (codes [n_layers][T], final residual [vq][T])."""
    x = np.array(x, np.float32, order="C", copy=True)
    es = [f32(a) for a in embed_sum]
    us = [f32(a) for a in usage]
    n, (cb, vq), T = len(es), es[0].shape, x.shape[1]
    pe = (F * n)(*[fp(a) for a in es])
    pu = (F * n)(*[fp(a) for a in us])
    codes = np.zeros((n, T), np.int64)
    lib().orc_rvq_encode(C.cast(pe, C.POINTER(F)), C.cast(pu, C.POINTER(F)), n, cb, vq, fp(x), T,
                         codes.ctypes.data_as(I64))
    return codes, x


def decode_reference_audio(data):
    """decode_reference_audio (execution/reference_audio.rs:17-50, 76-121)
    on a WAV image, restated with hound's reading rules: (mono f32 samples,
    sample rate).  Integer PCM 16 / 24 / 32-bit is value / 2^(bits-1)
    clamped to [-1, 1], 32-bit float as stored; each whole frame is the f32
    sum of its channels (from -0.0, in channel order) over the channel
    count.  Raises ValueError where the reference returns an error."""
    import struct
    b = bytes(data)
    if len(b) < 12 or b[:4] != b"RIFF" or b[8:12] != b"WAVE":
        raise ValueError("not a RIFF/WAVE image")
    off, fmt, payload = 12, None, None
    while off + 8 <= len(b) and payload is None:
        cid, n = b[off:off + 4], struct.unpack_from("<I", b, off + 4)[0]
        if off + 8 + n > len(b):
            raise ValueError("chunk runs past the image")
        if cid == b"fmt ":
            tag, ch, rate, _, align, bits = struct.unpack_from("<HHIIHH", b, off + 8)
            if tag == 0xFFFE:
                tag = struct.unpack_from("<H", b, off + 8 + 24)[0]
            fmt = (tag, ch, rate, align, bits)
        elif cid == b"data":
            if fmt is None:
                raise ValueError("data before fmt")
            payload = b[off + 8:off + 8 + n]
        off += 8 + n + (n & 1)
    if fmt is None or payload is None:
        raise ValueError("missing chunk")
    tag, ch, rate, align, bits = fmt
    if ch == 0:
        raise ValueError("zero channels")
    if not ((tag == 3 and bits == 32) or (tag == 1 and bits in (16, 24, 32))):
        raise ValueError("unsupported wav format")
    bps = bits // 8
    if align != ch * bps:
        raise ValueError("block align")
    total = len(payload) // bps
    if total == 0:
        raise ValueError("contains no audio samples")
    raw = np.frombuffer(payload[:total * bps], np.uint8).reshape(total, bps)
    if tag == 3:
        x = raw.copy().view("<f4").reshape(-1)
    else:
        v = np.zeros(total, np.int64)
        for k in range(bps):
            v |= raw[:, k].astype(np.int64) << (8 * k)
        v = np.where(v >= 1 << (bits - 1), v - (1 << bits), v)
        x = np.clip(v.astype(np.float32) / np.float32(2.0 ** (bits - 1)), np.float32(-1), np.float32(1))
    frames = total // ch
    if frames == 0:
        raise ValueError("contains no complete audio frames")
    x = x[:frames * ch].reshape(frames, ch).astype(np.float32)
    acc = np.full(frames, -0.0, np.float32)
    for c in range(ch):
        acc = (acc + x[:, c]).astype(np.float32)
    return (acc / np.float32(ch)).astype(np.float32), rate


def resample_linear(samples, source_rate, target_rate):
    """resample_linear (reference_audio.rs:123-156) in f32: out[i] =
    s[l] (1 - m) + s[r] m with l = i src / dst, r = min(l + 1, n - 1),
    m = (i src mod dst) / dst; (n dst + src / 2) / src outputs (at least
    one), none for an empty input or a zero rate, a copy for equal rates or
    a single sample."""
    s = np.ascontiguousarray(samples, np.float32).reshape(-1)
    n = len(s)
    if n == 0 or source_rate == 0 or target_rate == 0:
        return np.zeros(0, np.float32)
    if source_rate == target_rate or n == 1:
        return s.copy()
    m = max((n * target_rate + source_rate // 2) // source_rate, 1)
    pos = np.arange(m, dtype=np.uint64) * np.uint64(source_rate)
    left = (pos // np.uint64(target_rate)).astype(np.int64)
    right = np.minimum(left + 1, n - 1)
    mix = (pos % np.uint64(target_rate)).astype(np.float32) / np.float32(target_rate)
    return (s[left] * (np.float32(1) - mix) + s[right] * mix).astype(np.float32)


def speaker_mel(samples, n_mels=128, sample_rate=24000):
    """Log-mel features of the speaker encoder (speaker/infer/feature.rs):
    [n_mels][frames]."""
    x = np.ascontiguousarray(samples, np.float32)
    frames = (len(x) + 768 - 1024) // 256 + 1
    out = np.zeros((n_mels, max(frames, 1)), np.float32)
    got = lib().orc_speaker_mel(fp(x), len(x), sample_rate, n_mels, fp(out), max(frames, 0))
    if got < 0:
        raise ValueError("speaker mel needs at least 256 samples")
    return out[:, :got]


class OracleSpeaker:
    """ECAPA-TDNN speaker encoder of the voice-clone path
    (LoadedQwen3TtsSpeakerEncoder::encode_embedding, speaker/infer/mod.rs:11-20;
    network in speaker/network/*.rs)."""

    def __init__(self, cfg, weights: dict):
        self.cfg = cfg
        w = {k: f32(v) for k, v in weights.items()}
        self.w = w
        p = "speaker_encoder"
        sp = Speaker()
        sp.mel_dim, sp.enc_dim, sp.sample_rate = cfg.mel_dim, cfg.enc_dim, cfg.sample_rate
        for i, c in enumerate(cfg.enc_channels):
            sp.channels[i] = c
        if cfg.enc_res2net_scale > 16:
            raise ValueError("Res2Net scale above 16")

        def tdnn(name, k=1, dil=1):
            wt = w[f"{name}.weight"]
            return Tdnn(fp(wt), fp(w[f"{name}.bias"]), wt.shape[1], wt.shape[0], k, dil)

        ks, dl = cfg.enc_kernel_sizes, cfg.enc_dilations
        sp.block0 = tdnn(f"{p}.blocks.0.conv", ks[0], dl[0])
        for i in range(1, 4):
            b = f"{p}.blocks.{i}"
            se = SeBlock()
            se.tdnn1, se.tdnn2 = tdnn(f"{b}.tdnn1.conv"), tdnn(f"{b}.tdnn2.conv")
            for j in range(cfg.enc_res2net_scale - 1):
                se.res[j] = tdnn(f"{b}.res2net_block.blocks.{j}.conv", ks[i], dl[i])
            se.scale, se.se_ch = cfg.enc_res2net_scale, cfg.enc_se_channels
            se.se_w1, se.se_b1 = fp(w[f"{b}.se_block.conv1.weight"]), fp(w[f"{b}.se_block.conv1.bias"])
            se.se_w2, se.se_b2 = fp(w[f"{b}.se_block.conv2.weight"]), fp(w[f"{b}.se_block.conv2.bias"])
            sp.se[i - 1] = se
        sp.mfa = tdnn(f"{p}.mfa.conv", ks[4], dl[4])
        sp.asp_tdnn = tdnn(f"{p}.asp.tdnn.conv")
        sp.asp_w, sp.asp_b = fp(w[f"{p}.asp.conv.weight"]), fp(w[f"{p}.asp.conv.bias"])
        sp.fc_w, sp.fc_b = fp(w[f"{p}.fc.weight"]), fp(w[f"{p}.fc.bias"])
        self.s = sp

    def forward(self, mel):
        mel = np.ascontiguousarray(mel, np.float32)
        emb = np.zeros(self.cfg.enc_dim, np.float32)
        if lib().orc_speaker_forward(C.byref(self.s), fp(mel), mel.shape[1], fp(emb)) < 0:
            raise ValueError("speaker encoder: too few frames for the reflect padding")
        return emb

    def embed(self, samples):
        x = np.ascontiguousarray(samples, np.float32)
        emb = np.zeros(self.cfg.enc_dim, np.float32)
        if lib().orc_speaker_embed(C.byref(self.s), fp(x), len(x), fp(emb)) < 0:
            raise ValueError("speaker encoder: bad input")
        return emb

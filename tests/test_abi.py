"""The C-ABI library loads without a GPU, exports every symbol that
include/q3t.h declares, and its struct layouts (q3t_abi_struct /
q3t_abi_field) agree with the ctypes mirror and with the Rust binding that
INTEGRATION.md gives a maintainer (no compute calls)."""
import ctypes
import os
import re

import pytest

import q3t

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_text():
    src = open(os.path.join(ROOT, "include", "q3t.h")).read()
    return re.sub(r"/\*.*?\*/", "", src, flags=re.S)


def header_symbols():
    return sorted(set(re.findall(r"\b(q3t_[a-z0-9_]+)\s*\(", header_text())))


def header_structs():
    """C names of the public struct typedefs with a body (opaque handles excluded)."""
    return sorted(set(re.findall(r"typedef struct\s*\{.*?\}\s*(q3t_[a-z0-9_]+)\s*;", header_text(), flags=re.S)))


def rust_block():
    doc = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    blocks = re.findall(r"```rust\n(.*?)```", doc, flags=re.S)
    src = next(b for b in blocks if "extern \"C\"" in b)
    return re.sub(r"//[^\n]*", "", src)


def rust_structs(src):
    """{name: [(field, type), ...]} of the #[repr(C)] structs in the binding."""
    out = {}
    for name, body in re.findall(r"#\[repr\(C\)\][^\n]*\s*pub struct (\w+)\s*\{(.*?)\}", src, flags=re.S):
        fields = re.findall(r"pub (\w+)\s*:\s*([^,]+?)\s*(?:,|$)", body.strip())
        out[name] = [(f, t.strip()) for f, t in fields]
    return out


_PRIM = {"c_int": 4, "f32": 4, "i64": 8, "u64": 8, "usize": 8, "u8": 1, "u16": 2, "i16": 2, "i32": 4,
         "c_char": 1}


def rust_layout(ty, structs, cache):
    """(size, align) of a Rust type under #[repr(C)] (the C rules)."""
    ty = ty.strip()
    if ty.startswith("*"):
        return 8, 8
    if ty in _PRIM:
        return _PRIM[ty], _PRIM[ty]
    m = re.fullmatch(r"\[(.+);\s*(\d+)\]", ty)
    if m:
        s, a = rust_layout(m.group(1), structs, cache)
        return s * int(m.group(2)), a
    if ty in cache:
        return cache[ty][0], cache[ty][1]
    if ty not in structs:
        raise KeyError(f"unknown Rust type {ty}")
    off, align, fields = 0, 1, []
    for f, t in structs[ty]:
        s, a = rust_layout(t, structs, cache)
        off = (off + a - 1) // a * a
        fields.append((f, off, s))
        off += s
        align = max(align, a)
    size = (off + align - 1) // align * align
    cache[ty] = (size, align, fields)
    return size, align


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(q3t.LIB_PATH)
    syms = header_symbols()
    assert len(syms) >= 20
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing


def test_python_mirror_binds_every_declared_symbol():
    assert sorted(q3t.EXPORTS) == header_symbols()


def test_version_and_error_without_gpu():
    L = q3t.lib()
    assert b"sm_100a" in L.q3t_version()
    assert isinstance(L.q3t_last_error(), bytes)
    assert L.q3t_kernel_launches() >= 0


def test_layout_table_covers_every_public_struct():
    assert sorted(q3t.STRUCTS) == header_structs()
    for name in header_structs():
        size, align, fields = q3t.abi_layout(name)
        assert size > 0 and align in (4, 8) and fields
    with pytest.raises(q3t.Q3TError) as e:
        q3t.abi_layout("q3t_no_such_struct")
    assert e.value.status == q3t.INVALID_INPUT


@pytest.mark.parametrize("name", sorted(q3t.STRUCTS))
def test_ctypes_mirror_matches_library_layout(name):
    size, align, fields = q3t.abi_layout(name)
    cls = q3t.STRUCTS[name]
    assert ctypes.sizeof(cls) == size, (name, ctypes.sizeof(cls), size)
    assert ctypes.alignment(cls) == align
    mirror = [(f, getattr(cls, f).offset, getattr(cls, f).size) for f, *_ in cls._fields_]
    assert mirror == fields


def test_rust_binding_matches_library_layout():
    src = rust_block()
    structs = rust_structs(src)
    assert sorted(structs) == header_structs()
    cache = {}
    for name in structs:
        size, align, fields = q3t.abi_layout(name)
        rsize, ralign = rust_layout(name, structs, cache)
        assert cache[name][2] == fields, (name, cache[name][2], fields)
        assert (rsize, ralign) == (size, align), name


def test_rust_binding_declares_every_entry_point():
    declared = set(re.findall(r"pub fn (q3t_\w+)\s*\(", rust_block()))
    missing = sorted(set(header_symbols()) - declared)
    assert not missing, missing


def test_layout_check_catches_a_missing_field():
    """The Rust check above fails for a binding that drops a field (the
    mistake an earlier copy of the binding made with q3t_step_stats)."""
    structs = rust_structs(rust_block())
    structs["q3t_step_stats"] = [f for f in structs["q3t_step_stats"] if f[0] != "talker_ms"]
    cache = {}
    rust_layout("q3t_step_stats", structs, cache)
    assert cache["q3t_step_stats"][2] != q3t.abi_layout("q3t_step_stats")[2]


def test_encoder_loads_reject_bad_input_without_a_gpu():
    """The voice-clone encoders validate their config and arguments on the
    host before any CUDA call, so these fail the same way with no GPU."""
    import numpy as np
    import synthetic as S
    with pytest.raises(q3t.Q3TError) as e:  # 32 channels do not split into 5 Res2Net groups
        q3t.SpeakerEncoder(S.SpeakerEncoderConfig().small(enc_res2net_scale=5), {})
    assert e.value.status == q3t.INVALID_INPUT
    with pytest.raises(q3t.Q3TError) as e:  # an SE bottleneck wider than the gate kernel holds
        q3t.SpeakerEncoder(S.SpeakerEncoderConfig().small(enc_se_channels=2048), {})
    assert e.value.status == q3t.INVALID_INPUT
    with pytest.raises(q3t.Q3TError) as e:  # query heads not a multiple of the kv heads
        q3t.CodecEncoder(S.CodecEncoderConfig().small(n_heads=3, n_kv=2), {})
    assert e.value.status == q3t.INVALID_INPUT
    L = q3t.lib()
    x = np.zeros(4096, np.float32)
    out = np.zeros(4096, np.float32)
    fp = lambda a: a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    assert L.q3t_speaker_embed(None, fp(x), len(x), fp(out)) == q3t.INVALID_INPUT
    assert L.q3t_speaker_mel(None, fp(x), len(x), fp(out), 16, None) == q3t.INVALID_INPUT
    assert L.q3t_codec_encode(None, fp(x), len(x), 1, None, 16, None) == q3t.INVALID_INPUT

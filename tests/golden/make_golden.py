"""Extracts the reference's own known-answer tests for the hot path into
tests/golden/reference_kats.json.

Run in a container where the reference checkout exists:
    python tests/golden/make_golden.py <path of the tts-rs checkout>

Each KAT is parsed out of the Rust test it comes from (the file:line is
recorded next to it), so the oracle is pinned to the reference's numbers,
not to values typed in by hand.  The reference itself cannot be compiled
here (Rust/Burn), so these literal test vectors are the pin.
"""
import json
import os
import re
import sys


def _floats(s):
    return [float(x) for x in re.findall(r"-?\d+\.\d+", s)]


def _line_of(text, needle):
    return text[: text.index(needle)].count("\n") + 1


def main(ref):
    q = os.path.join(ref, "tts_qwen3_tts", "src", "model")
    out = {}

    # sampling.rs: sample_token_skips_masked_logits / top-k=1 test
    path = os.path.join(q, "talker", "infer", "sampling.rs")
    src = open(path).read()
    m = re.search(r"fn sample_token_skips_masked_logits\(\).*?from_floats\(\[([^\]]*)\].*?"
                  r"SamplingConfig::default\(\), &\[(\d+)\]\).*?assert_eq!\(values, vec!\[(\d+)\]\)",
                  src, re.S)
    out["sample_suppress"] = {"logits": _floats(m.group(1)), "suppress": [int(m.group(2))],
                              "expected": int(m.group(3)),
                              "source": f"tts_qwen3_tts/src/model/talker/infer/sampling.rs:{_line_of(src, 'fn sample_token_skips_masked_logits')}"}
    m = re.search(r"fn sampling_path_accepts_all_runtime_float_dtypes\(\).*?do_sample: (\w+),\s*"
                  r"temperature: ([\d.]+),\s*top_k: Some\((\d+)\),\s*top_p: ([\d.]+),.*?"
                  r"from_floats\(\[([^\]]*)\].*?assert_eq!\(values, vec!\[(\d+)\]\)", src, re.S)
    out["sample_topk1"] = {"do_sample": m.group(1) == "true", "temperature": float(m.group(2)),
                           "top_k": int(m.group(3)), "top_p": float(m.group(4)),
                           "logits": _floats(m.group(5)), "expected": int(m.group(6)),
                           "source": f"tts_qwen3_tts/src/model/talker/infer/sampling.rs:{_line_of(src, 'fn sampling_path_accepts_all_runtime_float_dtypes')}"}
    m = re.search(r"fn repetition_penalty_enabled_only_accepts_meaningful_positive_values\(\) \{(.*?)\n    \}",
                  src, re.S)
    cases = []
    for neg, arg in re.findall(r"assert!\((!?)repetition_penalty_enabled\(([^)]*\)?)\)\);", m.group(1)):
        arg = arg.strip()
        val = None if arg == "None" else arg[len("Some("):-1]
        val = {"f32::NAN": "nan"}.get(val, val)
        cases.append({"penalty": val, "enabled": neg != "!"})
    out["repetition_penalty_enabled"] = {"cases": cases,
                                         "source": f"tts_qwen3_tts/src/model/talker/infer/sampling.rs:{_line_of(src, 'fn repetition_penalty_enabled_only')}"}

    # kv.rs: reset_preserve_allocation tests
    path = os.path.join(q, "talker", "network", "kv.rs")
    src = open(path).read()
    m = re.search(r"fn reset_preserve_allocation_clears_len_without_dropping_cache_tensors\(\).*?"
                  r"KeyValueCache::<RuntimeBackend>::new\((\d+), (\d+), (\d+), (\d+)\);.*?"
                  r"ones\(\[(\d+), (\d+), (\d+), (\d+)\].*?assert_eq!\(cache.len\(\), (\d+)\);.*?"
                  r"assert_eq!\(cache.len\(\), (\d+)\);", src, re.S)
    out["kv_reset_len"] = {"cache": [int(m.group(i)) for i in range(1, 5)],
                           "input": [int(m.group(i)) for i in range(5, 9)],
                           "len_after_forward": int(m.group(9)), "len_after_reset": int(m.group(10)),
                           "source": f"tts_qwen3_tts/src/model/talker/network/kv.rs:{_line_of(src, 'fn reset_preserve_allocation_clears_len')}"}
    m = re.search(r"fn reset_preserve_allocation_exposes_only_new_forward_values\(\).*?"
                  r"new\((\d+), (\d+), (\d+), (\d+)\);.*?from_floats\(\[([^\]]*)\].*?from_floats\(\[([^\]]*)\]"
                  r".*?from_floats\(\[([^\]]*)\].*?from_floats\(\[([^\]]*)\].*?"
                  r"assert_eq!\(cache.len\(\), (\d+)\);\s*assert_eq!\(key_values, vec!\[([^\]]*)\]\);\s*"
                  r"assert_eq!\(value_values, vec!\[([^\]]*)\]\);", src, re.S)
    out["kv_reset_values"] = {"cache": [int(m.group(i)) for i in range(1, 5)],
                              "first_key": _floats(m.group(5)), "first_value": _floats(m.group(6)),
                              "next_key": _floats(m.group(7)), "next_value": _floats(m.group(8)),
                              "len": int(m.group(9)), "key_out": _floats(m.group(10)),
                              "value_out": _floats(m.group(11)),
                              "source": f"tts_qwen3_tts/src/model/talker/network/kv.rs:{_line_of(src, 'fn reset_preserve_allocation_exposes_only')}"}

    # conv.rs: pad_1d tests
    path = os.path.join(q, "codec", "network", "conv.rs")
    src = open(path).read()
    pads = []
    for name in ("constant_padding_preserves_runtime_dtype", "edge_padding_preserves_runtime_dtype"):
        m = re.search(rf"fn {name}\(\).*?from_data\(\[([^\]]*)\].*?pad_1d\(hidden, (\d+), (\d+), "
                      rf"PadMode::(\w+)(?:\(([\d.]+)\))?\);.*?assert_eq!\(samples, vec!\[([^\]]*)\]\);",
                      src, re.S)
        pads.append({"input": _floats(m.group(1).replace("f32", "")), "left": int(m.group(2)),
                     "right": int(m.group(3)), "mode": m.group(4).lower(),
                     "expected": _floats(m.group(6)),
                     "source": f"tts_qwen3_tts/src/model/codec/network/conv.rs:{_line_of(src, 'fn ' + name)}"})
    out["pad_1d"] = pads

    # talker/config.rs: the 0.6B config fixture
    path = os.path.join(q, "talker", "config.rs")
    src = open(path).read()
    m = re.search(r'const TALKER_CONFIG_JSON: &str = r#"(.*?)"#;', src, re.S)
    cfg = json.loads(m.group(1))["talker_config"]
    out["talker_config"] = {"config": cfg,
                            "source": f"tts_qwen3_tts/src/model/talker/config.rs:{_line_of(src, 'const TALKER_CONFIG_JSON')}"}

    # attention.rs: the SDPA test inputs (shape-only in the reference)
    path = os.path.join(q, "nn", "attention.rs")
    src = open(path).read()
    fl = re.findall(r"from_floats\(\s*\[([^\]]*)\]", src, re.S)
    mk = re.search(r"from_ints\(\[\[(\d+), (\d+)\], \[(\d+), (\d+)\]\]", src)
    out["sdpa_shape"] = {"query": _floats(fl[0]), "key": _floats(fl[1]), "value": _floats(fl[2]),
                         "mask": [int(mk.group(i)) for i in range(1, 5)], "shape": [1, 2, 2, 2],
                         "source": f"tts_qwen3_tts/src/model/nn/attention.rs:{_line_of(src, 'fn attention_restores_requested_dtype')}"}

    # execution/reference_audio.rs: the voice-clone clip reader's tests
    path = os.path.join(ref, "tts_qwen3_tts", "src", "execution", "reference_audio.rs")
    src = open(path).read()
    at = lambda name: f"tts_qwen3_tts/src/execution/reference_audio.rs:{_line_of(src, 'fn ' + name)}"
    m = re.search(r"fn linear_resample_changes_length_for_new_sample_rate\(\).*?vec!\[([^\]]*)\];\s*"
                  r"let resampled = resample_linear\(&source, (\d+), (\d+)\);\s*"
                  r"assert_eq!\(resampled.len\(\), (\d+)\);", src, re.S)
    out["resample_length"] = {"input": _floats(m.group(1)), "source_rate": int(m.group(2)),
                              "target_rate": int(m.group(3)), "expected_len": int(m.group(4)),
                              "source": at("linear_resample_changes_length_for_new_sample_rate")}
    m = re.search(r"fn linear_resample_returns_empty_for_invalid_rates\(\) \{(.*?)\n    \}", src, re.S)
    out["resample_invalid_rates"] = {
        "cases": [{"input": _floats(a), "source_rate": int(b.replace("_", "")), "target_rate": int(c.replace("_", ""))}
                  for a, b, c in re.findall(r"resample_linear\(&\[([^\]]*)\], ([\d_]+), ([\d_]+)\)", m.group(1))],
        "source": at("linear_resample_returns_empty_for_invalid_rates")}
    m = re.search(r"fn decoded_reference_audio_can_prepare_multiple_sample_rates\(\).*?write_wav_i16\(\s*&path,\s*"
                  r"([\d_]+),\s*(\d+),\s*&\[([^\]]*)\],\s*\);.*?prepare_reference_audio\(&decoded, ([\d_]+)\).*?"
                  r"prepare_reference_audio\(&decoded, ([\d_]+)\).*?native.samples.len\(\), (\d+)\);.*?"
                  r"resampled.samples.len\(\), (\d+)\);", src, re.S)
    out["wav_stereo_prepare"] = {"rate": int(m.group(1).replace("_", "")), "channels": int(m.group(2)),
                                 "pcm": [int(x.replace("_", "")) for x in re.findall(r"-?[\d_]+", m.group(3))],
                                 "native_rate": int(m.group(4).replace("_", "")),
                                 "target_rate": int(m.group(5).replace("_", "")),
                                 "native_len": int(m.group(6)), "resampled_len": int(m.group(7)),
                                 "source": at("decoded_reference_audio_can_prepare_multiple_sample_rates")}
    m = re.search(r"fn decoded_reference_audio_mixdowns_stereo_and_resamples\(\).*?"
                  r"sample.abs\(\) < ([\d.]+)\)", src, re.S)
    out["wav_stereo_prepare"]["max_abs"] = float(m.group(1))
    m = re.search(r"fn decode_reference_audio_rejects_empty_payload\(\).*?contains\(\"([^\"]*)\"\)", src, re.S)
    out["wav_empty_payload"] = {"message": m.group(1), "source": at("decode_reference_audio_rejects_empty_payload")}

    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_kats.json")
    with open(dst, "w") as f:
        json.dump(out, f, indent=1)
    print("wrote", dst)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <path of the tts-rs checkout>")
    main(sys.argv[1])

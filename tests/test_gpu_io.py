"""Model loading from .safetensors checkpoints (q3t_safetensors_open ->
q3t_model_load) gives exactly the model loaded from host tensors: talker
linears stored as BF16, norms as F32, the codec's quantizer statistics under
the newer `.codebook.` spelling (the legacy `._codebook.` one is what the
host-tensor path uses), so the loader's checkpoint-name aliasing is covered.
Outputs must be bit-identical."""
import numpy as np
import pytest

import q3t
import synthetic as S
from st_file import write_safetensors

pytestmark = pytest.mark.gpu


def test_model_from_safetensors_is_bit_identical(tmp_path):
    cfg = S.TalkerConfig().small(talker_layers=2, predictor_layers=1)
    tw = S.make_talker_weights(cfg, seed=0)
    cc = S.CodecConfig()
    cw = S.make_codec_weights(cc, seed=0)
    tfile, cfile = tmp_path / "model.safetensors", tmp_path / "speech_tokenizer.safetensors"
    write_safetensors(tfile, {n: (a, "F32" if a.ndim == 1 else "BF16") for n, a in tw.items()})
    write_safetensors(cfile, {n.replace("._codebook.", ".codebook."): (a, "F32") for n, a in cw.items()})
    sets = [q3t.TensorSet(tfile), q3t.TensorSet(cfile)]
    m_file = q3t.Model(cfg, None, cc, None, kv_pages=64, max_active=1, tensor_sets=sets)
    m_dict = q3t.Model(cfg, tw, cc, cw, kv_pages=64, max_active=1)
    prompt, trailing, pad = S.synthetic_talker_inputs(cfg, 8, seed=1)
    codes = S.teacher_codes(3, seed=2)
    outs = []
    for m in (m_file, m_dict):
        s = m.session(prompt, trailing, pad, max_new_tokens=3, forced_first=int(codes[0, 0]), first_logits=True)
        o = [s.first_logits.copy()]
        for f in range(2):
            _, tl, pl, hid = s.step_forced(codes[f])
            o += [tl, pl, hid]
        o.append(m.codec_decode(np.random.default_rng(4).integers(0, 2048, (1, 16, 5))))
        s.close()
        outs.append(o)
    for a, b in zip(*outs):
        assert np.array_equal(a, b)
    m_file.close()
    m_dict.close()
    for s in sets:
        s.close()

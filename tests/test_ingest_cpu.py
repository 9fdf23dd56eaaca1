"""Host side of the checkpoint ingest, on CPU: the safetensors reader returns
what was written (bf16 as its bits, f32 as is), rejects other dtypes like the
reference's read_tensor (src/core/loader.rs:25-46), and the oracle holding a
checkpoint's quantised weights (the reference loader restated) decodes."""
import numpy as np
import pytest

from test_gpu_ingest import CFG, bf16_bits, bf16_to_f32, make_checkpoint, reference_tensors, write_safetensors


def test_bf16_rounding_and_exact_widening():
    x = np.array([1.0, -2.5, 3.14159265, 1e-3, 65504.0, -0.0], np.float32)
    h = bf16_bits(x)
    back = bf16_to_f32(h)
    assert np.array_equal(bf16_to_f32(bf16_bits(back)), back)         # representable values survive
    assert np.all(np.abs(back - x) <= np.abs(x) * 2.0 ** -8)           # half an ulp of an 8-bit mantissa
    assert back[0] == 1.0 and back[1] == -2.5


def test_read_safetensors_round_trip(llmrs, tmp_path):
    stored, seen = make_checkpoint(CFG, 1, "BF16")
    p = str(tmp_path / "m.safetensors")
    write_safetensors(p, stored)
    got = llmrs.read_safetensors(p)
    assert set(got) == set(stored)
    for name, (a, dt) in stored.items():
        g, gdt = got[name]
        assert gdt == dt and g.shape == a.shape and np.array_equal(g, a)
    bad = dict(stored)
    bad["model.norm.weight"] = (stored["model.norm.weight"][0], "F16")
    write_safetensors(p, bad)
    with pytest.raises(ValueError):
        llmrs.read_safetensors(p)


def test_oracle_holds_a_checkpoint(orc):
    _, seen = make_checkpoint(CFG, 2, "F32")
    om = orc.Model(CFG)
    om.init_synthetic(0)
    for layer, which, codes, scales in reference_tensors(orc, CFG, seen):
        om.set_tensor(layer, which, codes, scales)
    codes, scales = om.tensor(0, orc.W_Q)
    q, s = orc.quantize_q4(seen["model.layers.0.self_attn.q_proj.weight"].ravel())
    assert np.array_equal(codes, q) and np.array_equal(scales, s)
    logits = om.forward([1, 2, 3], 0)
    assert np.all(np.isfinite(logits))
    om.close()

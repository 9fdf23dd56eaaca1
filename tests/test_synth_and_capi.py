"""Host-only checks: the shared synthetic generator, the golden fixtures, and the
C-ABI library (loads, exports every declared symbol, host-only helpers)."""
import os
import re

import numpy as np

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "llmrs_cuda.h")


def test_f16_conversion_matches_numpy(orc, rng):
    vals = np.concatenate([
        rng.normal(0, 1, 2000).astype(np.float32) * np.float32(0.01),
        np.float32([0.0, -0.0, 6.0e-8, 3.0e-8, 2.9802322e-08, 5.96e-8, 1e-5, 6.1e-5, 65504.0, 65519.0, 65520.0,
                    1e9, -1e9]),
        (np.arange(1, 2000, dtype=np.float32) * np.float32(2.0 ** -24)),
    ])
    for v in vals:
        h = orc.f32_to_f16_bits(v)
        assert h == int(np.float16(v).view(np.uint16)), v
        if np.isfinite(np.float16(v)):
            assert orc.f16_bits_to_f32(h) == float(np.float16(v))


def test_synthetic_recipe(orc):
    z = orc.synth_normal(1, 0, 5, 200000)
    assert abs(z.mean()) < 0.01 and abs(z.std() - 1.0) < 0.01
    assert np.abs(z).max() <= 6.0
    qs, sc = orc.synth_q4(1, 3, 11, 64, 2048)
    nib = np.concatenate([qs & 15, qs >> 4])
    assert nib.min() == 0 and nib.max() == 15 and abs(nib.mean() - 7.5) < 0.05
    # scales are fp16 values of |N(0,0.02)|/8, widened exactly to f32
    assert np.array_equal(sc.astype(np.float16).astype(np.float32), sc)
    assert abs(sc.mean() - 0.0025 * np.sqrt(2 / np.pi)) < 1e-4
    qw, _ = orc.synth_q8(1, 3, 11, 16, 1024)
    assert qw.min() == -127 and qw.max() == 127
    toks = [orc.synth_token(1, i, 128256) for i in range(100)]
    assert min(toks) >= 0 and max(toks) < 128256 and len(set(toks)) > 90


def test_golden_fixtures(orc):
    """tests/golden/*.npz were produced by tests/golden/make_golden.py from the
    oracle; they pin the oracle against accidental change."""
    path = os.path.join(ROOT, "tests", "golden", "golden_small.npz")
    g = np.load(path)
    q, s = orc.quantize_row_q8_0(g["q8_x"])
    assert np.array_equal(q, g["q8_q"]) and np.array_equal(s, g["q8_s"])
    qs, sc = orc.quantize_q4(g["q4_w"])
    assert np.array_equal(qs, g["q4_qs"]) and np.array_equal(sc, g["q4_sc"])
    y = orc.matmul_transposed_q4(g["mv_a"], g["mv_qs"], g["mv_sw"], int(g["mv_n"]))[0]
    assert np.array_equal(y, g["mv_y"])
    m = orc.Model({k: (float(v) if k in ("rms_eps", "rope_theta") else int(v))
                   for k, v in zip(g["tiny_cfg_keys"], g["tiny_cfg_vals"])})
    m.init_synthetic(int(g["tiny_seed"]))
    logits = m.forward(g["tiny_ids"], 0)
    assert np.array_equal(logits, g["tiny_logits"])


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(llmrs_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol(llmrs):
    import ctypes
    lib = ctypes.CDLL(llmrs.LIB_PATH)
    decl = declared_symbols()
    assert len(decl) >= 40
    for name in decl:
        assert hasattr(lib, name), name
    assert sorted(llmrs.EXPORTS) == sorted(decl)


def test_host_only_entry_points(llmrs, orc):
    assert llmrs.version().startswith("llmrs-b200")
    assert llmrs.lib().llmrs_backend_name().decode() == "Cuda"
    # RoPE table used by the decode step == the reference's formula with the
    # host libm (rope of a (1,..,1 | 0,..,0) row yields (cos | sin))
    D, npos = 128, 300
    c, s = llmrs.rope_table(D, npos)
    x = np.zeros((npos, D), np.float32)
    x[:, :D // 2] = 1.0
    r = orc.rope_inplace(x, D, 0).reshape(npos, D)
    assert np.array_equal(r[:, :D // 2], c)
    assert np.array_equal(r[:, D // 2:], s)


def test_errors_without_gpu_are_reported(llmrs):
    # on a machine without a GPU the context call fails with a status, not a crash
    import ctypes
    n = llmrs.device_count()
    if n == 0:
        h = ctypes.c_void_p()
        rc = llmrs.lib().llmrs_ctx_create(0, ctypes.byref(h))
        assert rc != llmrs.OK
        assert llmrs.lib().llmrs_last_error()

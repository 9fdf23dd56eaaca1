"""Regenerate tests/golden/golden_small.npz from the CPU oracle.

The reference (Rust) cannot be built in this image, so these fixtures are
oracle outputs: they pin the oracle (and, through the GPU parity tests, the
CUDA path) against unnoticed change.  Run from the repository root:
    python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from oracle import oracle as O  # noqa: E402


def main():
    rng = np.random.default_rng(20261201)
    out = {}
    x = rng.normal(0, 1, 1024).astype(np.float32)
    x[:32] = 0.0
    x[32:64] = np.linspace(-2.5, 2.5, 32, dtype=np.float32)
    out["q8_x"] = x
    out["q8_q"], out["q8_s"] = O.quantize_row_q8_0(x)
    w = rng.uniform(-1, 1, 4096).astype(np.float32)
    w[:32] = 0.0
    out["q4_w"] = w
    out["q4_qs"], out["q4_sc"] = O.quantize_q4(w)
    n, k = 256, 2048
    qs, sw = O.synth_q4(1234, 0, 11, n, k)
    a = rng.normal(0, 1, k).astype(np.float32)
    out["mv_a"], out["mv_qs"], out["mv_sw"], out["mv_n"] = a, qs, sw, np.int64(n)
    out["mv_y"] = O.matmul_transposed_q4(a, qs, sw, n)[0]
    cfg = dict(n_layers=2, hidden=256, n_heads=8, n_kv_heads=2, head_dim=32, ffn=512, vocab=1000, max_seq=64,
               rms_eps=1e-5, rope_theta=500000.0, weight_format=0, tied_embeddings=1)
    out["tiny_cfg_keys"] = np.array(list(cfg.keys()))
    out["tiny_cfg_vals"] = np.array([float(v) for v in cfg.values()])
    out["tiny_seed"] = np.int64(77)
    ids = np.array([5, 17, 900, 3], np.int32)
    out["tiny_ids"] = ids
    m = O.Model(cfg)
    m.init_synthetic(77)
    out["tiny_logits"] = m.forward(ids, 0)
    path = os.path.join(ROOT, "tests", "golden", "golden_small.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()

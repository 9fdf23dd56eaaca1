"""Prefill (M>1 rows) on the tcgen05 path against the CPU oracle.

Models whose linears have K a multiple of 256 prefill every prompt of >= 8
tokens as M = n contractions (per-row Q8_0 quantise, int8 tensor-core block
dots, in-order f32 block sums) followed by causal attention over the cache.
The contractions are bit-exact with the reference (and the batch-1 GEMV); the
RMSNorm and attention reductions are ordered differently, so values agree to
rounding.

Q4_0 models (4-bit codes times |N(0, 0.02)|/8 scales) are well conditioned:
their logits meet the decode tolerances (max-abs 2e-2, relative L2 1e-3) over
long prompts.  The Q8_0 synthetic models are not: codes are uniform in
-127..127, so every linear amplifies a perturbation ~10x, and a rounding-level
difference that moves one activation across a Q8_0 rounding boundary flips a
code and shifts the next layer by ~1e-2 relative.  The batch-1 decode path
shows the same isolated flips (measured: 64-token prompt, layer-1 K rows 44
and 48 off by 3e-2 against the oracle, every other row within 1e-5).  Long
Q8_0 prompts are therefore checked row by row: greedy tokens identical, cache
rows within 1e-4 relative of the oracle (all of them in the first layer of the
hidden-512 model, >= 90% where flips can reach), logits within 5e-2 relative
L2.
"""
import numpy as np
import pytest

from conftest import CFG_1B, CFG_8B, with_
from test_gpu_model import LOGIT_REL_L2, abs_tol, compare_run

pytestmark = pytest.mark.gpu

CFG_Q8 = dict(n_layers=2, hidden=512, n_heads=8, n_kv_heads=2, head_dim=64, ffn=1024, vocab=1000, max_seq=640,
              rms_eps=1e-5, rope_theta=500000.0, weight_format=1, tied_embeddings=0)
CFG_Q4 = with_(CFG_Q8, weight_format=0)
Q8_LOGIT_REL = 5e-2
Q8_ROW_FRACTION = 0.9


def check(r):
    assert r["mismatches"] == 0, r
    assert r["abs_ok"] and r["rel"] < LOGIT_REL_L2, r


def row_agreement(r, n, rtol=1e-4):
    """Per layer: fraction of cache positions whose K and V rows agree with the oracle."""
    gm, om, out = r["model"], r["oracle"], []
    for layer in range(om.cfg["n_layers"] if hasattr(om, "cfg") else gm.cfg["n_layers"]):
        gk, gv = gm.kv_read(layer, n)
        ok = om.kcache(layer)[:, :n]
        ov = np.transpose(om.vcache(layer)[:, :, :n], (0, 2, 1))
        dk = np.abs(gk - ok).max(axis=(0, 2)) <= rtol * (1 + np.abs(ok).max())
        dv = np.abs(gv - ov).max(axis=(0, 2)) <= rtol * (1 + np.abs(ov).max())
        out.append(float(np.mean(dk & dv)))
    return out


def check_q8(r, n, min_rows):
    """min_rows[l]: the fraction of layer l's cache rows that must agree."""
    assert r["mismatches"] == 0, r
    assert r["rel"] < Q8_LOGIT_REL, r
    frac = row_agreement(r, n)
    assert all(f >= m for f, m in zip(frac, min_rows)), frac


def test_q4_prefill_long_prompt(llmrs, ctx, orc):
    # 300 rows (two full 128-row tiles and a ragged one), Q4_0: decode tolerances
    prompt = [orc.synth_token(31, i, CFG_Q4["vocab"]) for i in range(300)]
    check(compare_run(llmrs, ctx, orc, CFG_Q4, 31, prompt, 4))


def test_q4_prefill_after_cached_positions_f32_scales(llmrs, ctx, orc):
    prompt = [orc.synth_token(32, i, CFG_Q4["vocab"]) for i in range(150)]
    check(compare_run(llmrs, ctx, orc, CFG_Q4, 32, prompt, 3, kv_prefill=40, scale_dtype=1))


def test_q4_prefill_chunks_over_512_rows(llmrs, ctx, orc):
    # 600 rows: a 512-row chunk, then an 88-row chunk that attends to it
    prompt = [orc.synth_token(33, i, CFG_Q4["vocab"]) for i in range(600)]
    check(compare_run(llmrs, ctx, orc, with_(CFG_Q4, n_layers=1), 33, prompt, 2))


def test_config1_1b_long_prompt(llmrs, ctx, orc):
    # Llama-3.2-1B shape (tied Q4 LM head, 16 layers), 256-token prompt
    cfg = with_(CFG_1B, max_seq=320)
    prompt = [orc.synth_token(34, i, cfg["vocab"]) for i in range(256)]
    check(compare_run(llmrs, ctx, orc, cfg, 34, prompt, 2))


def test_q8_prefill_ragged_prompt(llmrs, ctx, orc):
    prompt = [orc.synth_token(21, i, CFG_Q8["vocab"]) for i in range(300)]
    check_q8(compare_run(llmrs, ctx, orc, CFG_Q8, 21, prompt, 4), 300, (1.0, Q8_ROW_FRACTION))


def test_q8_prefill_after_cached_positions(llmrs, ctx, orc):
    prompt = [orc.synth_token(22, i, CFG_Q8["vocab"]) for i in range(150)]
    r = compare_run(llmrs, ctx, orc, CFG_Q8, 22, prompt, 3, kv_prefill=40, scale_dtype=1)
    check_q8(r, 190, (1.0, Q8_ROW_FRACTION))


def test_q8_prefill_first_layer_cache_equals_decode_path(llmrs, ctx, orc):
    # layer 0's K/V rows come from the first contraction and RoPE alone, so the
    # tensor-core prefill and the batch-1 path (chunks of < 8 rows) must
    # write identical bits
    prompt = [orc.synth_token(24, i, CFG_Q8["vocab"]) for i in range(64)]
    a = llmrs.Model(ctx, dict(CFG_Q8, scale_dtype=0))
    b = llmrs.Model(ctx, dict(CFG_Q8, scale_dtype=0))
    a.init_synthetic(24)
    b.init_synthetic(24)
    ta, la = a.prefill(prompt, 0)
    for i in range(0, 64, 4):
        tb, lb = b.prefill(prompt[i:i + 4], i)
    ka, va = a.kv_read(0, 64)
    kb, vb = b.kv_read(0, 64)
    assert np.array_equal(ka.view(np.uint32), kb.view(np.uint32))
    assert np.array_equal(va.view(np.uint32), vb.view(np.uint32))
    assert ta == tb


def test_config4_8b_q8_prefill(llmrs, ctx, orc):
    # config 4 shapes (8B, Q8_0 weights, f16 scales), 2 layers, 160-token prompt.
    # With 4096 activations per row, ~5% of the rows already see a flipped
    # code in layer 0's QKV input (the RMSNorm sum order), and attention
    # spreads each flip to later rows of the next layer, so only layer 0 is
    # checked row by row; tokens and the logits bound cover the rest.
    cfg = with_(CFG_8B, n_layers=2, weight_format=1, max_seq=512)
    prompt = [orc.synth_token(4, i, cfg["vocab"]) for i in range(160)]
    check_q8(compare_run(llmrs, ctx, orc, cfg, 4, prompt, 2), 160, (Q8_ROW_FRACTION, 0.0))


def test_prefill_without_room_for_the_bf16_copy(llmrs, ctx, monkeypatch):
    """When the bf16 copy of the weights does not fit (forced here with
    LLMRS_PREFILL_BF16_MAX_MB=1, read when a model first prefills), the
    tensor-core prefill runs the int8 GEMM straight from the Q4_0 storage:
    no error, and the same exact contractions give the same logits."""
    cfg = with_(CFG_8B, n_layers=2, max_seq=128)
    ids = [(17 * i + 5) % cfg["vocab"] for i in range(40)]
    monkeypatch.setenv("LLMRS_PREFILL_BF16_MAX_MB", "1")
    a = llmrs.Model(ctx, cfg)
    a.init_synthetic(9)
    ta, la = a.prefill(ids, 0)
    ta2, la2 = a.prefill(ids, 0)  # a later prefill reuses the decision, no retry
    monkeypatch.delenv("LLMRS_PREFILL_BF16_MAX_MB")
    b = llmrs.Model(ctx, cfg)
    b.init_synthetic(9)
    tb, lb = b.prefill(ids, 0)
    a.close()
    b.close()
    assert ta == ta2 == tb
    assert np.array_equal(la, la2) and np.array_equal(la, lb)

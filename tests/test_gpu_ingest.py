"""Checkpoint ingest on the GPU (llmrs_model_load_weight, load_safetensors)
against the reference's loader (src/core/loader.rs:25-198).

A small Llama checkpoint is written as a real safetensors file (bf16 or f32
tensors with the reference's names).  The loader's work -- bf16 -> f32,
quantize_q4 of every linear (src/core/tensor.rs:102-167), gate/up fused,
K/V at n_kv_heads rows (the reference's replicated rows quantise identically),
the LM head from lm_head.weight or, absent, from the embedding -- is restated
on the CPU: the oracle quantises the same f32 weights and holds them.  The GPU
model that ingested the file must (1) give bit-identical logits to a GPU model
filled with llmrs_model_set_weight from the oracle-quantised tensors (so the
device quantiser produced exactly the reference's codes and scales) and (2)
agree with the oracle: greedy tokens identical, logits max-abs 2e-2.  This
small Gaussian checkpoint has logits of order 0.5, and one activation code
that rounds the other way moves every output of a K = 512 linear by ~1e-3
relative, so its relative L2 is bounded at 1e-2 (measured 3.6e-3)."""
import json
import struct

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CFG = dict(n_layers=2, hidden=512, n_heads=8, n_kv_heads=2, head_dim=64, ffn=1024, vocab=1000, max_seq=64,
           rms_eps=1e-5, rope_theta=500000.0, weight_format=0, tied_embeddings=0, scale_dtype=1)


def bf16_bits(x):
    """f32 -> bf16 bits, rounded to nearest even (finite inputs)"""
    b = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)


def bf16_to_f32(h):
    return (np.asarray(h).astype(np.uint32) << 16).view(np.float32)


def write_safetensors(path, tensors):
    header, blobs, off = {}, [], 0
    for name, (a, dt) in tensors.items():
        b = np.ascontiguousarray(a).tobytes()
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def make_checkpoint(cfg, seed, dtype="BF16", with_lm_head=True):
    """{name: (stored array, dtype)} and {name: f32 values the loader sees}"""
    rng = np.random.default_rng(seed)
    H, D, F, V = cfg["hidden"], cfg["head_dim"], cfg["ffn"], cfg["vocab"]
    qd, kd = cfg["n_heads"] * D, cfg["n_kv_heads"] * D
    f32 = {"model.embed_tokens.weight": rng.normal(0, 1, (V, H)), "model.norm.weight": rng.normal(1, 0.02, H)}
    for i in range(cfg["n_layers"]):
        p = "model.layers.%d." % i
        f32[p + "self_attn.q_proj.weight"] = rng.normal(0, 0.02, (qd, H))
        f32[p + "self_attn.k_proj.weight"] = rng.normal(0, 0.02, (kd, H))
        f32[p + "self_attn.v_proj.weight"] = rng.normal(0, 0.02, (kd, H))
        f32[p + "self_attn.o_proj.weight"] = rng.normal(0, 0.02, (H, qd))
        f32[p + "mlp.gate_proj.weight"] = rng.normal(0, 0.02, (F, H))
        f32[p + "mlp.up_proj.weight"] = rng.normal(0, 0.02, (F, H))
        f32[p + "mlp.down_proj.weight"] = rng.normal(0, 0.02, (H, F))
        f32[p + "input_layernorm.weight"] = rng.normal(1, 0.02, H)
        f32[p + "post_attention_layernorm.weight"] = rng.normal(1, 0.02, H)
    if with_lm_head:
        f32["lm_head.weight"] = rng.normal(0, 0.02, (V, H))
    stored, seen = {}, {}
    for name, v in f32.items():
        v = v.astype(np.float32)
        if dtype == "BF16":
            stored[name] = (bf16_bits(v), "BF16")
            seen[name] = bf16_to_f32(stored[name][0])
        else:
            stored[name] = (v, "F32")
            seen[name] = v
    return stored, seen


def reference_tensors(orc, cfg, seen):
    """(layer, which, codes, scales) of the reference loader's model (scales None: f32 tensor)"""
    out = [(-1, orc.W_EMBED, seen["model.embed_tokens.weight"], None),
           (-1, orc.W_FINAL_NORM, seen["model.norm.weight"], None)]
    q8 = cfg["weight_format"] == 1

    def quant(w):
        if q8:  # Q8_0 models: the Q8_0 block quantiser per row
            qs, sc = zip(*(orc.quantize_row_q8_0(r) for r in w))
            return np.concatenate(qs), np.concatenate(sc)
        return orc.quantize_q4(w.ravel())

    for i in range(cfg["n_layers"]):
        p = "model.layers.%d." % i
        for which, name in ((orc.W_Q, "self_attn.q_proj"), (orc.W_K, "self_attn.k_proj"),
                            (orc.W_V, "self_attn.v_proj"), (orc.W_O, "self_attn.o_proj"),
                            (orc.W_DOWN, "mlp.down_proj")):
            out.append((i, which) + tuple(quant(seen[p + name + ".weight"])))
        fused = np.concatenate([seen[p + "mlp.gate_proj.weight"], seen[p + "mlp.up_proj.weight"]])
        out.append((i, orc.W_GATE_UP) + tuple(quant(fused)))  # src/core/loader.rs:128-147
        out.append((i, orc.W_ATTN_NORM, seen[p + "input_layernorm.weight"], None))
        out.append((i, orc.W_MLP_NORM, seen[p + "post_attention_layernorm.weight"], None))
    head = seen.get("lm_head.weight", seen["model.embed_tokens.weight"])  # loader.rs:186-190
    out.append((-1, orc.W_LM_HEAD) + tuple(orc.quantize_q4(head.ravel()) if not q8 or "lm_head.weight" not in seen
                                           else quant(head)))
    return out


def rel_l2(a, b):
    return float(np.linalg.norm(a.astype(np.float64) - b) / np.linalg.norm(b.astype(np.float64)))


def run(model, prompt, steps):
    t, lg = model.prefill(prompt, 0)
    out = [(t, lg)]
    pos = len(prompt)
    for _ in range(steps):
        t, lg = model.decode_step(t, pos)
        out.append((t, lg))
        pos += 1
    return out


@pytest.mark.parametrize("dtype,tied,fmt", [("BF16", 0, 0), ("F32", 1, 0), ("BF16", 0, 1)])
def test_safetensors_ingest_matches_reference_loader(llmrs, ctx, orc, tmp_path, dtype, tied, fmt):
    cfg = dict(CFG, tied_embeddings=tied, weight_format=fmt)
    stored, seen = make_checkpoint(cfg, 7 + tied + 2 * fmt, dtype, with_lm_head=not tied)
    path = str(tmp_path / "model.safetensors")
    write_safetensors(path, stored)
    ga = llmrs.Model(ctx, cfg)
    llmrs.load_safetensors(ga, path)
    ref = reference_tensors(orc, cfg, seen)
    gb = llmrs.Model(ctx, cfg)
    for layer, which, codes, scales in ref:
        gb.set_weight(layer, which, codes, scales)
    prompt = [11, 500, 7, 999, 3, 42, 8, 100, 64]  # >= 8 tokens: the tensor-core prefill
    a, b = run(ga, prompt, 4), run(gb, prompt, 4)
    for (ta, la), (tb, lb) in zip(a, b):
        assert ta == tb and np.array_equal(la, lb)  # the device quantised exactly as the reference
    if fmt == 0:  # the oracle restates the reference's Q4_0 model
        om = orc.Model(cfg)
        om.init_synthetic(0)
        for layer, which, codes, scales in ref:
            om.set_tensor(layer, which, codes, scales)
        ol = om.forward(prompt, 0)
        pos, tok = len(prompt), orc.argmax(ol)
        for i, (t, lg) in enumerate(a):
            if i:
                ol = om.forward([tok], pos)
                pos += 1
            assert t == orc.argmax(ol) or orc.top2_margin(ol) < 1e-3, (i, t, orc.argmax(ol))
            tol = 2e-2 * max(1.0, float(np.abs(ol).max()) / 100.0)
            assert float(np.abs(lg - ol).max()) < tol and rel_l2(lg, ol) < 1e-2, i
            tok = orc.argmax(ol)
        om.close()
    ga.close()
    gb.close()


def test_ingest_errors(llmrs, ctx, tmp_path):
    stored, _ = make_checkpoint(CFG, 3, "BF16")
    name = "model.layers.0.self_attn.q_proj.weight"
    bad = dict(stored)
    bad[name] = (stored[name][0], "F16")  # the reference's read_tensor rejects other dtypes
    p = str(tmp_path / "bad.safetensors")
    write_safetensors(p, bad)
    m = llmrs.Model(ctx, CFG)
    with pytest.raises(ValueError):
        llmrs.load_safetensors(m, p)
    missing = {k: v for k, v in stored.items() if k != name}
    p2 = str(tmp_path / "missing.safetensors")
    write_safetensors(p2, missing)
    with pytest.raises(KeyError):
        llmrs.load_safetensors(m, p2)
    # quantize_q4 scales are not f16-exact: an f16-scale model refuses them
    m16 = llmrs.Model(ctx, dict(CFG, scale_dtype=0))
    with pytest.raises(llmrs.LlmrsError) as e:
        m16.load_weight(0, llmrs.W_Q, stored[name][0])
    assert e.value.code == llmrs.EINVAL
    m.close()
    m16.close()

"""GPU parity of the fused decode attention (llmrs_attention_decode) against the
reference's per-head loop (src/core/layer.rs:175-333, seq == 1) restated with
the CPU oracle's Backend operations.  RoPE and the KV append are bit-exact (the
cos/sin table comes from the same host libm); the split softmax / P.V sums are
reordered on the GPU, so the output is compared at 2e-5 relative."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def oracle_attention(orc, q, k_new, v_new, kc, vc, n_heads, n_kv, D, pos):
    """src/core/layer.rs:212-299 per query head, native GQA (kv head = h // n_rep)."""
    n_rep = n_heads // n_kv
    kc = kc.copy()
    vc = vc.copy()
    for g in range(n_kv):
        kc[g, pos] = orc.rope_inplace(k_new[g], D, pos)
        vc[g, pos] = v_new[g]
    out = np.zeros((n_heads, D), np.float32)
    inv = np.float32(1.0) / np.sqrt(np.float32(D))
    for h in range(n_heads):
        g = h // n_rep
        qh = orc.rope_inplace(q[h], D, pos)
        scores = orc.matmul_slice(qh[None, :], kc[g, :pos + 1], pos + 1, D)
        probs = orc.softmax(orc.scale(scores, inv))
        out[h] = orc.matmul_f32(probs, vc[g, :pos + 1])[0]
    return out, kc, vc


@pytest.mark.parametrize("n_heads,n_kv,D,pos", [(32, 8, 128, 300), (32, 8, 64, 77), (64, 8, 128, 1000), (32, 8, 128, 0)])
def test_attention_decode_matches_reference(llmrs, ctx, be, orc, rng, n_heads, n_kv, D, pos):
    S = 1100
    q = rng.normal(0, 1, (n_heads, D)).astype(np.float32)
    k_new = rng.normal(0, 1, (n_kv, D)).astype(np.float32)
    v_new = rng.normal(0, 1, (n_kv, D)).astype(np.float32)
    kc = rng.normal(0, 1, (n_kv, S, D)).astype(np.float32)
    vc = rng.normal(0, 1, (n_kv, S, D)).astype(np.float32)
    cos, sin = llmrs.rope_table(D, S)
    qkv = np.concatenate([q.ravel(), k_new.ravel(), v_new.ravel()])
    d_qkv = llmrs.DeviceTensor.from_numpy(ctx, qkv)
    d_kc = llmrs.DeviceTensor.from_numpy(ctx, kc)
    d_vc = llmrs.DeviceTensor.from_numpy(ctx, vc)
    d_cos = llmrs.DeviceTensor.from_numpy(ctx, cos)
    d_sin = llmrs.DeviceTensor.from_numpy(ctx, sin)
    out = be.attention_decode(d_qkv, d_kc, d_vc, d_cos, d_sin, n_heads, n_kv, D, pos).numpy()
    ref, kc2, vc2 = oracle_attention(orc, q, k_new, v_new, kc, vc, n_heads, n_kv, D, pos)
    # KV append: bit-exact RoPE of the new key, exact copy of the new value
    assert np.array_equal(d_kc.numpy()[:, pos], kc2[:, pos])
    assert np.array_equal(d_vc.numpy()[:, pos], vc2[:, pos])
    assert np.abs(out.reshape(n_heads, D) - ref).max() <= 2e-5 * max(1.0, np.abs(ref).max())


def oracle_attention_prefill(orc, qkv, kc, vc, n_heads, n_kv, D, start):
    """src/core/layer.rs:212-333 for seq_len = n rows: RoPE, KV append, causal
    mask (-inf past start + i), softmax, P.V through CpuBackend::matmul."""
    n = qkv.shape[0]
    n_rep = n_heads // n_kv
    q = qkv[:, :n_heads * D].reshape(n, n_heads, D)
    k = qkv[:, n_heads * D:(n_heads + n_kv) * D].reshape(n, n_kv, D)
    v = qkv[:, (n_heads + n_kv) * D:].reshape(n, n_kv, D)
    kc, vc = kc.copy(), vc.copy()
    for g in range(n_kv):
        kc[g, start:start + n] = orc.rope_inplace(np.ascontiguousarray(k[:, g]), D, start)
        vc[g, start:start + n] = v[:, g]
    total = start + n
    inv = np.float32(1.0) / np.sqrt(np.float32(D))
    out = np.zeros((n, n_heads, D), np.float32)
    for h in range(n_heads):
        g = h // n_rep
        qh = orc.rope_inplace(np.ascontiguousarray(q[:, h]), D, start)
        scores = orc.scale(orc.matmul_slice(qh, kc[g, :total], total, D), inv)
        for i in range(n):
            scores[i, start + i + 1:] = -np.inf
        probs = orc.softmax(scores)
        out[:, h] = orc.matmul_f32(probs, vc[g, :total])
    return out.reshape(n, n_heads * D), kc, vc


@pytest.mark.parametrize("n_heads,n_kv,D,n,start", [(32, 8, 128, 300, 0), (32, 8, 128, 40, 1000), (8, 2, 64, 77, 5),
                                                    (64, 8, 128, 33, 200)])
def test_attention_prefill_matches_reference(llmrs, ctx, be, orc, rng, n_heads, n_kv, D, n, start):
    S = 1100
    qkv = rng.normal(0, 1, (n, (n_heads + 2 * n_kv) * D)).astype(np.float32)
    kc = rng.normal(0, 1, (n_kv, S, D)).astype(np.float32)
    vc = rng.normal(0, 1, (n_kv, S, D)).astype(np.float32)
    cos, sin = llmrs.rope_table(D, S)
    d_qkv = llmrs.DeviceTensor.from_numpy(ctx, qkv)
    d_kc = llmrs.DeviceTensor.from_numpy(ctx, kc)
    d_vc = llmrs.DeviceTensor.from_numpy(ctx, vc)
    d_cos = llmrs.DeviceTensor.from_numpy(ctx, cos)
    d_sin = llmrs.DeviceTensor.from_numpy(ctx, sin)
    out = be.attention_prefill(d_qkv, d_kc, d_vc, d_cos, d_sin, n_heads, n_kv, D, start).numpy()
    ref, kc2, vc2 = oracle_attention_prefill(orc, qkv, kc, vc, n_heads, n_kv, D, start)
    # KV append of every row: bit-exact RoPE, exact copy
    assert np.array_equal(d_kc.numpy()[:, start:start + n], kc2[:, start:start + n])
    assert np.array_equal(d_vc.numpy()[:, start:start + n], vc2[:, start:start + n])
    assert np.abs(out - ref).max() <= 2e-5 * max(1.0, np.abs(ref).max())


def test_attention_decode_rejects_bad_position(llmrs, ctx, be):
    D, S = 64, 16
    t = llmrs.DeviceTensor.from_numpy(ctx, np.zeros(4 * S * D, np.float32))
    with pytest.raises(llmrs.LlmrsError) as e:
        llmrs.check(llmrs.lib().llmrs_attention_decode(ctx.h, t.ptr, t.ptr, t.ptr, t.ptr, t.ptr, t.ptr, 4, 1, D, S, S))
    assert e.value.code == llmrs.EINVAL

"""CPU oracle checks: the reference's own known-answer / property tests
(src/test/cpu.rs, src/test/opencl.rs, src/core/layer.rs tests) plus independent
numpy restatements of the block arithmetic, so the C oracle is not trusted on
its own word."""
import numpy as np
import pytest

from conftest import CFG_TINY, with_


def naive_matmul(a, b):  # src/test/cpu.rs:45-66 (f32 sequential)
    m, k = a.shape
    n = b.shape[1]
    c = np.zeros((m, n), np.float32)
    for p in range(k):
        c = (c + np.outer(a[:, p], b[p, :]).astype(np.float32)).astype(np.float32)
    return c


def test_rms_norm_known_answer(orc):
    # src/test/cpu.rs:197-212
    d = orc.rms_norm([1.0, 2.0, 3.0, 4.0], [1.0, 1.0, 1.0, 1.0], 1e-5)[0]
    assert abs(d[0] - 0.3651) < 1e-3
    assert abs(d[3] - 1.4605) < 1e-3


def test_softmax_properties(orc):
    # src/test/cpu.rs:214-227
    d = orc.softmax([1.0, 2.0, 3.0])[0]
    assert abs(d.sum() - 1.0) < 1e-5
    assert d[2] > d[1] > d[0]


def test_rope_magnitude(orc):
    # src/test/cpu.rs:229-245
    d = orc.rope_inplace([1.0, 0.0, 0.0, 1.0], 4, 1)
    assert abs(np.hypot(d[0], d[2]) - 1.0) < 1e-5
    assert abs(np.hypot(d[1], d[3]) - 1.0) < 1e-5
    assert d[0] != 1.0


def test_matmul_variants(orc, rng):
    # src/test/cpu.rs:103-160 (tolerance 1e-4)
    a = rng.uniform(-1, 1, (1, 128)).astype(np.float32)
    b = rng.uniform(-1, 1, (128, 256)).astype(np.float32)
    assert np.abs(orc.matmul_f32(a, b) - naive_matmul(a, b)).max() < 1e-4
    a = rng.uniform(-1, 1, (16, 64)).astype(np.float32)
    b = rng.uniform(-1, 1, (64, 32)).astype(np.float32)
    assert np.abs(orc.matmul_f32(a, b) - naive_matmul(a, b)).max() < 1e-4
    a = rng.uniform(-1, 1, (4, 128)).astype(np.float32)
    w = rng.uniform(-1, 1, (64, 128)).astype(np.float32)
    assert np.abs(orc.matmul_transposed_f32(a, w) - naive_matmul(a, w.T.copy())).max() < 1e-4
    q = rng.uniform(-1, 1, (1, 64)).astype(np.float32)
    kc = rng.uniform(-1, 1, (10, 64)).astype(np.float32)
    assert np.abs(orc.matmul_slice(q, kc, 10, 64) - naive_matmul(q, kc.T.copy())).max() < 1e-4


def test_elementwise(orc, rng):
    # src/test/cpu.rs:162-195
    a = rng.uniform(-1, 1, 100).astype(np.float32)
    b = rng.uniform(-1, 1, 100).astype(np.float32)
    assert np.abs(orc.add_assign(a, b) - (a + b)).max() < 1e-5
    g = rng.uniform(-1, 1, 25).astype(np.float32)
    u = rng.uniform(-1, 1, 25).astype(np.float32)
    ref = g / (1.0 + np.exp(-g)) * u
    assert np.abs(orc.silu_mul(g, u) - ref).max() < 1e-5


def np_quantize_q8(x):
    """numpy restatement of quantize_row_q8_0 (src/backend/cpu.rs:724-743)."""
    x = np.asarray(x, np.float32).reshape(-1, 32)
    amax = np.abs(x).max(axis=1)
    scale = (amax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = (np.float32(1.0) / scale).astype(np.float32)
    y = (x * inv[:, None]).astype(np.float32)
    r = np.sign(y) * np.floor(np.abs(y).astype(np.float64) + 0.5)  # round half away from zero
    q = np.clip(r, -127, 127)
    q[amax == 0] = 0
    scale[amax == 0] = 0
    return q.astype(np.int8).ravel(), scale


def test_q8_quantiser_independent(orc, rng):
    x = rng.normal(0, 1, 4096).astype(np.float32)
    x[:32] = 0.0  # zero block -> scale 0, codes 0
    x[32:64] = np.linspace(-2.5, 2.5, 32)  # exact ties after scaling
    q, s = orc.quantize_row_q8_0(x)
    q2, s2 = np_quantize_q8(x)
    assert np.array_equal(q, q2)
    assert np.array_equal(s.view(np.uint32), s2.view(np.uint32))


def np_q4q8_matvec(a, qs, sw, n, k):
    """numpy restatement of kernel_avx2's block arithmetic (src/backend/cpu.rs:903-938)."""
    q, sa = np_quantize_q8(a)
    nb = k // 32
    nib = np.zeros((n, k), np.int32)
    b = qs.reshape(n, k // 2)
    nib[:, 0::2] = b & 0x0F
    nib[:, 1::2] = b >> 4
    isum = ((nib - 8).reshape(n, nb, 32) * q.astype(np.int32).reshape(1, nb, 32)).sum(axis=2)
    sw = sw.reshape(n, nb)
    acc = np.zeros(n, np.float32)
    for blk in range(nb):
        scale = (sw[:, blk] * sa[blk]).astype(np.float32)
        acc = (acc + (isum[:, blk].astype(np.float32) * scale).astype(np.float32)).astype(np.float32)
    return acc


def test_q4_matvec_independent(orc, rng):
    n, k = 96, 1024
    qs, sw = orc.synth_q4(7, 0, 11, n, k)
    a = rng.normal(0, 1, k).astype(np.float32)
    got = orc.matmul_transposed_q4(a, qs, sw, n)[0]
    ref = np_q4q8_matvec(a, qs, sw, n, k)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_q4_dequant_identity(orc, rng):
    # src/test/opencl.rs:182-258: quantize_q4 then (q-8)*scale reproduces the
    # weights to within one quantisation step
    w = rng.uniform(-1, 1, (64, 128)).astype(np.float32)
    qs, sc = orc.quantize_q4(w)
    deq = orc.dequantize_q4(qs, sc, w.size).reshape(w.shape)
    step = np.repeat(sc, 32).reshape(w.shape)
    assert np.all(np.abs(deq - w) <= step * 1.0 + 1e-7)
    # zero block -> 0x88 bytes, scale 0 (src/core/tensor.rs:120-122)
    qz, sz = orc.quantize_q4(np.zeros(64, np.float32))
    assert np.all(qz == 0x88) and np.all(sz == 0)
    # Q4xQ8 matvec against the dequantised weights: only the Q8 activation
    # rounding separates them
    a = rng.uniform(-1, 1, (1, 128)).astype(np.float32)
    got = orc.matmul_transposed_q4(a, qs, sc, 64)[0]
    ref = deq.astype(np.float64) @ a[0].astype(np.float64)
    assert np.abs(got - ref).max() < 0.05


def test_q4_matmul_m_rows(orc, rng):
    # m>1 path (src/backend/cpu.rs:90-110): each row is quantised and processed alone
    n, k = 64, 256
    qs, sw = orc.synth_q4(3, 1, 12, n, k)
    a = rng.normal(0, 1, (4, k)).astype(np.float32)
    full = orc.matmul_transposed_q4(a, qs, sw, n)
    for i in range(4):
        assert np.array_equal(full[i], orc.matmul_transposed_q4(a[i:i + 1], qs, sw, n)[0])


def test_gqa_expansion_equivalence(orc):
    # src/core/loader.rs:62-98 replicates K/V rows per query head; native GQA
    # must give bit-identical logits
    a = orc.Model(CFG_TINY, expand_gqa=False)
    b = orc.Model(CFG_TINY, expand_gqa=True)
    for m in (a, b):
        m.init_synthetic(5)
    la = a.forward([3, 1, 4, 1, 5], 0)
    lb = b.forward([3, 1, 4, 1, 5], 0)
    assert np.array_equal(la, lb)
    assert np.array_equal(a.forward([9], 5), b.forward([9], 5))


def test_prefill_equals_sequential_decode(orc):
    # a causal chunk equals the same tokens fed one at a time
    ids = [11, 22, 33, 44, 55, 66]
    a = orc.Model(CFG_TINY)
    a.init_synthetic(9)
    la = a.forward(ids, 0)
    b = orc.Model(CFG_TINY)
    b.init_synthetic(9)
    for i, t in enumerate(ids):
        lb = b.forward([t], i)
    assert np.array_equal(la, lb)
    for layer in range(CFG_TINY["n_layers"]):
        assert np.array_equal(a.kcache(layer)[:, :6], b.kcache(layer)[:, :6])


def test_attention_causality_and_kv_update(orc):
    # src/core/layer.rs:430-489: position 0 is unaffected by position 1, and the
    # cache fills position by position
    m1 = orc.Model(CFG_TINY)
    m1.init_synthetic(2)
    m1.forward([7, 8], 0)
    m2 = orc.Model(CFG_TINY)
    m2.init_synthetic(2)
    m2.forward([7, 99], 0)
    assert np.array_equal(m1.kcache(0)[:, 0], m2.kcache(0)[:, 0])
    assert not np.array_equal(m1.kcache(0)[:, 1], m2.kcache(0)[:, 1])
    m3 = orc.Model(CFG_TINY)
    m3.init_synthetic(2)
    assert np.all(m3.kcache(0)[:, 0] == 0)
    m3.forward([7], 0)
    assert np.any(m3.kcache(0)[:, 0] != 0) and np.all(m3.kcache(0)[:, 1] == 0)
    m3.forward([8], 1)
    assert np.any(m3.kcache(0)[:, 1] != 0)


def test_forward_error_paths(orc):
    m = orc.Model(CFG_TINY)
    m.init_synthetic(1)
    with pytest.raises(ValueError):
        m.forward([1], CFG_TINY["max_seq"])  # beyond the KV capacity
    with pytest.raises(ValueError):
        m.forward([CFG_TINY["vocab"]], 0)  # token out of range


def test_q8_weight_matvec_independent(orc, rng):
    n, k = 48, 512
    qw, sw = orc.synth_q8(4, 0, 11, n, k)
    a = rng.normal(0, 1, k).astype(np.float32)
    got = orc.matmul_transposed_q8w(a, qw, sw, n)[0]
    q, sa = np_quantize_q8(a)
    nb = k // 32
    isum = (qw.astype(np.int32).reshape(n, nb, 32) * q.astype(np.int32).reshape(1, nb, 32)).sum(axis=2)
    acc = np.zeros(n, np.float32)
    swr = sw.reshape(n, nb)
    for b in range(nb):
        acc = (acc + (isum[:, b].astype(np.float32) * (swr[:, b] * sa[b]).astype(np.float32))).astype(np.float32)
    assert np.array_equal(got.view(np.uint32), acc.view(np.uint32))


def test_tiny_model_q8_and_untied(orc):
    cfg = with_(CFG_TINY, weight_format=1, tied_embeddings=0)
    m = orc.Model(cfg)
    m.init_synthetic(3)
    logits = m.forward([1, 2, 3], 0)
    assert np.all(np.isfinite(logits))

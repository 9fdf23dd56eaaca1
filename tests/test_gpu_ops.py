"""GPU parity of the Backend-trait operations (through the C ABI) against the
CPU oracle.  Integer/byte work and the reference-ordered contractions are
checked bit-exactly; ops whose reduction order or libm differ use the stated
tolerances."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SWEEP = [(2048, 2048), (8192, 2048), (2048, 8192), (14336, 4096), (4096, 14336), (128256, 4096)]


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def dev(llmrs, ctx, a, dtype=None):
    return llmrs.DeviceTensor.from_numpy(ctx, np.asarray(a), dtype)


def test_backend_identity(be):
    assert be.device() == "Cuda"
    assert be.name() == "Cuda"


def test_quantize_row_q8_0_bit_exact(llmrs, ctx, be, orc, rng):
    x = rng.normal(0, 1, (3, 4096)).astype(np.float32)
    x[0, :32] = 0.0
    x[1, 32:64] = np.linspace(-2.5, 2.5, 32)
    x[2, 64:96] = rng.normal(0, 1e-30, 32)
    q, s = be.quantize_row_q8_0(dev(llmrs, ctx, x))
    for i in range(3):
        q2, s2 = orc.quantize_row_q8_0(x[i])
        assert np.array_equal(q.numpy()[i], q2)
        assert np.array_equal(bits(s.numpy()[i]), bits(s2))


def test_quantize_q4_bit_exact(llmrs, ctx, be, orc, rng):
    w = rng.uniform(-1, 1, 64 * 128 + 17).astype(np.float32)  # ragged tail block
    w[:32] = 0.0
    qs, sc = be.quantize_q4(dev(llmrs, ctx, w))
    qs2, sc2 = orc.quantize_q4(w)
    assert np.array_equal(qs.numpy(), qs2)
    assert np.array_equal(bits(sc.numpy()), bits(sc2))


def test_golden_vectors_on_gpu(llmrs, ctx, be):
    import os
    from conftest import ROOT
    g = np.load(os.path.join(ROOT, "tests", "golden", "golden_small.npz"))
    q, s = be.quantize_row_q8_0(dev(llmrs, ctx, g["q8_x"][None, :]))
    assert np.array_equal(q.numpy()[0], g["q8_q"]) and np.array_equal(bits(s.numpy()[0]), bits(g["q8_s"]))
    qs, sc = be.quantize_q4(dev(llmrs, ctx, g["q4_w"]))
    assert np.array_equal(qs.numpy(), g["q4_qs"]) and np.array_equal(bits(sc.numpy()), bits(g["q4_sc"]))
    n, k = int(g["mv_n"]), g["mv_a"].size
    for st in (llmrs.F16, llmrs.F32):
        W = llmrs.QuantWeight(ctx, g["mv_qs"], g["mv_sw"], n, k, llmrs.WFMT_Q4_0, st)
        y = be.matmul_transposed(dev(llmrs, ctx, g["mv_a"][None, :]), W).numpy()[0]
        assert np.array_equal(bits(y), bits(g["mv_y"]))


@pytest.mark.parametrize("n,k", SWEEP)
@pytest.mark.parametrize("st", [0, 1])
def test_q4_gemv_sweep_bit_exact(llmrs, ctx, be, orc, rng, n, k, st):
    # config 2 shapes: Q8_0 activation bit-exact, outputs bit-exact with the
    # reference's sequential block accumulation
    qs, sw = orc.synth_q4(2026, 0, 11, n, k)
    a = rng.normal(0, 1, (1, k)).astype(np.float32)
    W = llmrs.QuantWeight(ctx, qs, sw, n, k, llmrs.WFMT_Q4_0, st)
    y = be.matmul_transposed(dev(llmrs, ctx, a), W).numpy()[0]
    ref = orc.matmul_transposed_q4(a, qs, sw, n)[0]
    assert np.array_equal(bits(y), bits(ref)), np.abs(y - ref).max()


@pytest.mark.parametrize("m,k,n", [(1, 128, 64), (4, 256, 128), (4, 128, 64), (3, 1792, 4096), (1, 96, 10)])
def test_q4_small_and_ragged_shapes(llmrs, ctx, be, orc, rng, m, k, n):
    # reference test shapes (src/test/opencl.rs:237-276, 473-510) and a TP-shard K
    w = rng.uniform(-1, 1, (n, k)).astype(np.float32)
    qs, sc = orc.quantize_q4(w)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    W = llmrs.QuantWeight(ctx, qs, sc, n, k, llmrs.WFMT_Q4_0, llmrs.F32)
    y = be.matmul_transposed(dev(llmrs, ctx, a), W).numpy()
    ref = orc.matmul_transposed_q4(a, qs, sc, n)
    assert np.array_equal(bits(y), bits(ref))
    # and against the dequantised weights (only Q8 activation rounding differs)
    deq = orc.dequantize_q4(qs, sc, w.size).reshape(n, k).astype(np.float64)
    assert np.abs(y - a.astype(np.float64) @ deq.T).max() < 0.1 * np.sqrt(k / 128)


@pytest.mark.parametrize("n,k", [(4096, 4096), (1024, 14336), (256, 512)])
def test_q8_weight_gemv_bit_exact(llmrs, ctx, be, orc, rng, n, k):
    qw, sw = orc.synth_q8(99, 1, 14, n, k)
    a = rng.normal(0, 1, (1, k)).astype(np.float32)
    W = llmrs.QuantWeight(ctx, qw, sw, n, k, llmrs.WFMT_Q8_0, llmrs.F16)
    y = be.matmul_transposed(dev(llmrs, ctx, a), W).numpy()[0]
    ref = orc.matmul_transposed_q8w(a, qw, sw, n)[0]
    assert np.array_equal(bits(y), bits(ref))


@pytest.mark.parametrize("m,n,k", [(8, 256, 512), (200, 1000, 4096), (512, 512, 4096), (160, 1024, 14336),
                                   (129, 6144, 4096)])
@pytest.mark.parametrize("st", [0, 1])
def test_q8_prefill_gemm_bit_exact(llmrs, ctx, be, orc, rng, m, n, k, st):
    # M>1 rows on the tcgen05 path (m >= 8, k % 256 == 0): per-row Q8_0
    # quantise, per-block int8 MMA, in-order f32 block sums -- bit-exact with
    # the reference's m>1 loop (src/backend/cpu.rs:90-110), ragged m and n
    qw, sw = orc.synth_q8(7, 2, 14, n, k)
    a = rng.normal(0, 1, (m, k)).astype(np.float32)
    a[m // 2, :] = 0.0  # an all-zero row: zero scales, zero outputs
    W = llmrs.QuantWeight(ctx, qw, sw, n, k, llmrs.WFMT_Q8_0, st)
    y = be.matmul_transposed(dev(llmrs, ctx, a), W).numpy()
    ref = orc.matmul_transposed_q8w(a, qw, sw, n)
    assert y.shape == ref.shape
    bad = np.argwhere(bits(y) != bits(ref))
    assert bad.size == 0, (len(bad), bad[:5], np.abs(y - ref).max())


@pytest.mark.parametrize("m,n,k", [(8, 256, 512), (300, 1000, 4096), (160, 4096, 14336), (129, 2048, 2048)])
@pytest.mark.parametrize("st", [0, 1])
def test_q4_prefill_gemm_bit_exact(llmrs, ctx, be, orc, rng, m, n, k, st):
    # Q4_0 weights on the tcgen05 path: nibbles unpacked in shared memory to
    # unsigned codes, the -8 offset folded into the per-block bias
    qs, sw = orc.synth_q4(5, 1, 11, n, k)
    a = rng.normal(0, 1, (m, k)).astype(np.float32)
    a[m // 3, :] = 0.0
    W = llmrs.QuantWeight(ctx, qs, sw, n, k, llmrs.WFMT_Q4_0, st)
    y = be.matmul_transposed(dev(llmrs, ctx, a), W).numpy()
    ref = orc.matmul_transposed_q4(a, qs, sw, n)
    bad = np.argwhere(bits(y) != bits(ref))
    assert bad.size == 0, (len(bad), bad[:5], np.abs(y - ref).max())


def test_gemv_rejects_bad_k(llmrs, ctx, be, rng):
    a = dev(llmrs, ctx, rng.normal(0, 1, (1, 100)).astype(np.float32))
    W = llmrs.QuantWeight(ctx, np.zeros(50 * 8, np.uint8), np.zeros(8, np.float32), 8, 100)
    with pytest.raises(llmrs.LlmrsError) as e:
        be.matmul_transposed(a, W)
    assert e.value.code == llmrs.EINVAL


def test_rms_norm_known_answer(llmrs, ctx, be):
    # src/test/opencl.rs:329-346
    y = be.rms_norm(dev(llmrs, ctx, np.float32([[1, 2, 3, 4]])), dev(llmrs, ctx, np.ones(4, np.float32)), 1e-5)
    d = y.numpy()[0]
    assert abs(d[0] - 0.3651) < 1e-3 and abs(d[3] - 1.4605) < 1e-3


def test_rms_norm_vs_oracle(llmrs, ctx, be, orc, rng):
    x = rng.normal(0, 3, (5, 4096)).astype(np.float32)
    w = rng.normal(1, 0.02, 4096).astype(np.float32)
    y = be.rms_norm(dev(llmrs, ctx, x), dev(llmrs, ctx, w), 1e-5).numpy()
    ref = orc.rms_norm(x, w, 1e-5)
    assert np.abs(y - ref).max() <= 2e-6 * np.abs(ref).max()


def test_softmax(llmrs, ctx, be, orc, rng):
    d = be.softmax(dev(llmrs, ctx, np.float32([[1, 2, 3]]))).numpy()[0]
    assert abs(d.sum() - 1) < 1e-5 and d[2] > d[1] > d[0]
    x = rng.normal(0, 4, (7, 1000)).astype(np.float32)
    x[3, 500:] = -np.inf  # masked tail, as the causal mask writes
    y = be.softmax(dev(llmrs, ctx, x)).numpy()
    ref = orc.softmax(x)
    assert np.abs(y - ref).max() < 1e-6


def test_rope_inplace(llmrs, ctx, be, orc, rng):
    x = dev(llmrs, ctx, np.float32([[1, 0, 0, 1]]))
    be.rope_inplace(x, 1)
    d = x.numpy()[0]
    assert abs(np.hypot(d[0], d[2]) - 1) < 1e-4 and abs(np.hypot(d[1], d[3]) - 1) < 1e-4 and d[0] != 1.0
    h = rng.normal(0, 1, (50, 128)).astype(np.float32)
    t = dev(llmrs, ctx, h)
    be.rope_inplace(t, 7)
    ref = orc.rope_inplace(h, 128, 7).reshape(50, 128)
    # device powf/sinf/cosf vs the host libm: a few ulp of the angle
    assert np.abs(t.numpy() - ref).max() < 2e-5 * (1 + np.abs(h).max()) * 8


def test_matmuls_bit_exact(llmrs, ctx, be, orc, rng):
    # sequential f32 dot / SAXPY order of src/backend/cpu.rs:113-269
    a = rng.uniform(-1, 1, (16, 64)).astype(np.float32)
    b = rng.uniform(-1, 1, (64, 32)).astype(np.float32)
    a[0, 5] = 0.0
    assert np.array_equal(bits(be.matmul(dev(llmrs, ctx, a), dev(llmrs, ctx, b)).numpy()),
                          bits(orc.matmul_f32(a, b)))
    w = rng.uniform(-1, 1, (64, 64)).astype(np.float32)
    assert np.array_equal(bits(be.matmul_transposed(dev(llmrs, ctx, a), dev(llmrs, ctx, w)).numpy()),
                          bits(orc.matmul_transposed_f32(a, w)))
    q = rng.uniform(-1, 1, (1, 64)).astype(np.float32)
    kc = rng.uniform(-1, 1, (10, 64)).astype(np.float32)
    assert np.array_equal(bits(be.matmul_slice(dev(llmrs, ctx, q), dev(llmrs, ctx, kc), 10, 64).numpy()),
                          bits(orc.matmul_slice(q, kc, 10, 64)))


def test_elementwise(llmrs, ctx, be, orc, rng):
    a = rng.uniform(-1, 1, 1024).astype(np.float32)
    b = rng.uniform(-1, 1, 1024).astype(np.float32)
    ta = dev(llmrs, ctx, a)
    be.add_assign(ta, dev(llmrs, ctx, b))
    assert np.array_equal(bits(ta.numpy()), bits(orc.add_assign(a, b)))
    g = rng.uniform(-4, 4, 1000).astype(np.float32)
    u = rng.uniform(-1, 1, 1000).astype(np.float32)
    tg = dev(llmrs, ctx, g)
    be.silu_mul(tg, dev(llmrs, ctx, u))
    assert np.abs(tg.numpy() - orc.silu_mul(g, u)).max() < 1e-6
    assert np.array_equal(bits(be.scale(ta, 0.125).numpy()), bits(orc.scale(ta.numpy(), 0.125)))
    assert np.array_equal(be.copy_from(ta).numpy(), ta.numpy())


def test_memory_sync_loop(llmrs, ctx, be):
    # src/test/opencl.rs:412-437
    a = dev(llmrs, ctx, np.zeros((1, 1024), np.float32))
    one = dev(llmrs, ctx, np.ones((1, 1024), np.float32))
    for i in range(1, 101):
        be.add_assign(a, one)
        assert a.numpy()[0, 0] == float(i)

"""The allocation-free decode attention (llmrs_attention_decode_noalloc) must give
the same results as llmrs_attention_decode, for callers that cannot allocate
device memory (their memory belongs to another allocator, or they must not
allocate after start-up).  Two calls in a row check that the fixed scratch array
is reused correctly; the file is collected last on purpose."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 2e-5  # the attention tolerance the other GPU tests use


def _setup(llmrs, ctx, rng, n_heads, n_kv, D, S):
    q = rng.normal(0, 1, (2, n_heads * D + 2 * n_kv * D)).astype(np.float32)
    kc = rng.normal(0, 1, (n_kv, S, D)).astype(np.float32)
    vc = rng.normal(0, 1, (n_kv, S, D)).astype(np.float32)
    cos, sin = llmrs.rope_table(D, S)
    T = llmrs.DeviceTensor.from_numpy
    return q, [T(ctx, kc), T(ctx, vc)], [T(ctx, kc), T(ctx, vc)], T(ctx, cos), T(ctx, sin)


@pytest.mark.parametrize("n_heads,n_kv,D,pos", [(32, 8, 128, 400), (32, 8, 64, 50)])
def test_noalloc_matches_allocating_entry_point(llmrs, ctx, be, rng, n_heads, n_kv, D, pos):
    import torch

    S = 512
    qkv, cache_a, cache_b, cos, sin = _setup(llmrs, ctx, rng, n_heads, n_kv, D, S)
    stream = torch.cuda.Stream()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    for step in range(2):  # two calls in a row, positions pos and pos + 1
        d_qkv = llmrs.DeviceTensor.from_numpy(ctx, qkv[step])
        want = be.attention_decode(d_qkv, cache_a[0], cache_a[1], cos, sin, n_heads, n_kv, D, pos + step).numpy()
        got = llmrs.DeviceTensor(ctx, (n_heads * D,))
        ctx.sync()  # inputs were uploaded on the context's stream
        rc = llmrs.lib().llmrs_attention_decode_noalloc(
            ctypes.c_void_p(stream.cuda_stream), d_qkv.ptr, cache_b[0].ptr, cache_b[1].ptr, cos.ptr, sin.ptr,
            got.ptr, n_heads, n_kv, D, S, pos + step, ctypes.c_void_p(err.data_ptr()))
        llmrs.check(rc)
        stream.synchronize()
        out = got.numpy()
        assert np.abs(out - want).max() <= TOL * max(1.0, np.abs(want).max())
        assert np.array_equal(cache_b[0].numpy()[:, pos + step], cache_a[0].numpy()[:, pos + step])
        assert np.array_equal(cache_b[1].numpy()[:, pos + step], cache_a[1].numpy()[:, pos + step])
    assert int(err.item()) == 0


def test_noalloc_rejects_sizes_beyond_its_scratch(llmrs, ctx):
    t = llmrs.DeviceTensor.from_numpy(ctx, np.zeros(1024, np.float32))
    # 1024 heads x 18 splits x 130 floats is far more than the fixed 2 MiB
    rc = llmrs.lib().llmrs_attention_decode_noalloc(None, t.ptr, t.ptr, t.ptr, t.ptr, t.ptr, t.ptr,
                                                     1024, 8, 128, 16, 0, None)
    assert rc == llmrs.EINVAL
    assert b"scratch" in llmrs.lib().llmrs_last_error()
    rc = llmrs.lib().llmrs_attention_decode_noalloc(None, t.ptr, t.ptr, t.ptr, t.ptr, t.ptr, t.ptr,
                                                     1024, 256, 64, 16, 0, None)
    assert rc == llmrs.EINVAL

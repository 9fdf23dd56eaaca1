"""llm.rs B200 backend: ctypes view of libllmrs_cuda.so (include/llmrs_cuda.h).

`CudaBackend` mirrors the reference's `trait Backend` (src/backend.rs:15-40)
method by method on device tensors, so tests read like src/test/cpu.rs; `Model`
drives the fused, device-resident decode step (src/core/model.rs:17-49).
Every call goes through the C ABI; a nonzero status raises `LlmrsError`, the
way the reference's panics would fire.  There is no CPU fallback: importing
this package on a machine without the built library raises ImportError.

The directory name contains a dot, so load it by path, e.g.::

    spec = importlib.util.spec_from_file_location(
        "llmrs_b200", "llm.rs_b200/__init__.py",
        submodule_search_locations=["llm.rs_b200"])
"""
import ctypes
import os
import weakref

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libllmrs_cuda.so")

OK, EINVAL, ENOMEM, ECUDA, ETIMEDOUT, ENOTSUP, ENCCL, EDEVICE = range(8)
F16, F32, BF16 = 0, 1, 2
WFMT_Q4_0, WFMT_Q8_0 = 0, 1
(W_Q, W_K, W_V, W_O, W_GATE_UP, W_DOWN, W_ATTN_NORM, W_MLP_NORM, W_EMBED, W_FINAL_NORM,
 W_LM_HEAD, W_GATE, W_UP) = range(13)

# every symbol include/llmrs_cuda.h declares (checked by tests/test_synth_and_capi.py)
EXPORTS = [
    "llmrs_last_error", "llmrs_version", "llmrs_device_count", "llmrs_ctx_create", "llmrs_ctx_destroy",
    "llmrs_ctx_set_stream", "llmrs_malloc", "llmrs_free", "llmrs_h2d", "llmrs_d2h", "llmrs_d2d",
    "llmrs_memset", "llmrs_sync", "llmrs_backend_name", "llmrs_ctx_device",
    "llmrs_matmul_transposed_q4", "llmrs_matmul_transposed_q8", "llmrs_matmul_transposed_f32",
    "llmrs_matmul", "llmrs_matmul_slice", "llmrs_add_assign", "llmrs_silu_mul", "llmrs_rope_inplace",
    "llmrs_rms_norm", "llmrs_softmax", "llmrs_scale", "llmrs_copy_from", "llmrs_quantize_row_q8_0",
    "llmrs_quantize_q4", "llmrs_rms_norm_quantize_q8_0", "llmrs_model_create", "llmrs_model_destroy", "llmrs_model_init_synthetic",
    "llmrs_model_set_weight", "llmrs_model_load_weight", "llmrs_kv_fill", "llmrs_kv_fill_synthetic", "llmrs_kv_read",
    "llmrs_decode_step", "llmrs_generate", "llmrs_prefill", "llmrs_model_logits", "llmrs_rope_table",
    "llmrs_model_decode_kernel_count", "llmrs_model_time_decode", "llmrs_model_time_prefill",
    "llmrs_model_profile_decode", "llmrs_time_gemv",
    "llmrs_attention_decode", "llmrs_attention_decode_noalloc", "llmrs_attention_prefill",
    "llmrs_sample", "llmrs_model_sample", "llmrs_model_trace_decode",
    "llmrs_model_tp_region", "llmrs_model_tp_connect", "llmrs_ipc_get_handle", "llmrs_ipc_open_handle",
    "llmrs_ipc_close_handle", "llmrs_model_set_peer_timeout", "llmrs_model_tp_epoch", "llmrs_model_tp_resync",
]
IPC_HANDLE_BYTES = 64


class LlmrsError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__("llmrs error %d: %s" % (code, msg))
        self.code = code


class Config(ctypes.Structure):
    _fields_ = [
        ("n_layers", ctypes.c_int), ("hidden", ctypes.c_int), ("n_heads", ctypes.c_int),
        ("n_kv_heads", ctypes.c_int), ("head_dim", ctypes.c_int), ("ffn", ctypes.c_int),
        ("vocab", ctypes.c_int), ("max_seq", ctypes.c_int), ("rms_eps", ctypes.c_float),
        ("rope_theta", ctypes.c_float), ("weight_format", ctypes.c_int),
        ("tied_embeddings", ctypes.c_int), ("scale_dtype", ctypes.c_int),
        ("tp_rank", ctypes.c_int), ("tp_size", ctypes.c_int),
    ]


_lib = None


def lib():
    """The loaded library (raises ImportError when it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError("libllmrs_cuda.so is missing: run `python llm.rs_b200/build.py` "
                          "(or __graft_entry__.build())")
    L = ctypes.CDLL(LIB_PATH)
    vp, sz, ci, cf = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_float
    pp = ctypes.POINTER(ctypes.c_void_p)
    ip = ctypes.POINTER(ctypes.c_int)
    fp = ctypes.POINTER(ctypes.c_float)
    sig = {
        "llmrs_last_error": (ctypes.c_char_p, []),
        "llmrs_version": (ctypes.c_char_p, []),
        "llmrs_backend_name": (ctypes.c_char_p, []),
        "llmrs_device_count": (ci, [ip]),
        "llmrs_ctx_create": (ci, [ci, pp]),
        "llmrs_ctx_destroy": (ci, [vp]),
        "llmrs_ctx_set_stream": (ci, [vp, vp]),
        "llmrs_ctx_device": (ci, [vp, ip]),
        "llmrs_malloc": (ci, [vp, sz, pp]),
        "llmrs_free": (ci, [vp, vp]),
        "llmrs_h2d": (ci, [vp, vp, vp, sz]),
        "llmrs_d2h": (ci, [vp, vp, vp, sz]),
        "llmrs_d2d": (ci, [vp, vp, vp, sz]),
        "llmrs_memset": (ci, [vp, vp, ci, sz]),
        "llmrs_sync": (ci, [vp]),
        "llmrs_matmul_transposed_q4": (ci, [vp, vp, vp, vp, ci, vp, ci, ci, ci]),
        "llmrs_matmul_transposed_q8": (ci, [vp, vp, vp, vp, ci, vp, ci, ci, ci]),
        "llmrs_matmul_transposed_f32": (ci, [vp, vp, vp, vp, ci, ci, ci]),
        "llmrs_matmul": (ci, [vp, vp, vp, vp, ci, ci, ci]),
        "llmrs_matmul_slice": (ci, [vp, vp, vp, vp, ci, ci, ci]),
        "llmrs_add_assign": (ci, [vp, vp, vp, sz]),
        "llmrs_silu_mul": (ci, [vp, vp, vp, sz]),
        "llmrs_rope_inplace": (ci, [vp, vp, ci, ci, ci, cf]),
        "llmrs_rms_norm": (ci, [vp, vp, vp, vp, ci, ci, cf]),
        "llmrs_softmax": (ci, [vp, vp, vp, ci, ci]),
        "llmrs_scale": (ci, [vp, vp, vp, sz, cf]),
        "llmrs_copy_from": (ci, [vp, vp, vp, sz]),
        "llmrs_quantize_row_q8_0": (ci, [vp, vp, vp, vp, ci, ci]),
        "llmrs_quantize_q4": (ci, [vp, vp, sz, vp, vp]),
        "llmrs_rms_norm_quantize_q8_0": (ci, [vp, vp, vp, vp, vp, ci, cf]),
        "llmrs_model_create": (ci, [vp, ctypes.POINTER(Config), pp]),
        "llmrs_model_destroy": (ci, [vp]),
        "llmrs_model_init_synthetic": (ci, [vp, ctypes.c_uint64]),
        "llmrs_model_set_weight": (ci, [vp, ci, ci, vp, vp]),
        "llmrs_model_load_weight": (ci, [vp, ci, ci, vp, ci]),
        "llmrs_kv_fill": (ci, [vp, ci, vp, vp, ci]),
        "llmrs_kv_fill_synthetic": (ci, [vp, ctypes.c_uint64, ci]),
        "llmrs_kv_read": (ci, [vp, ci, vp, vp, ci]),
        "llmrs_decode_step": (ci, [vp, ci, ci, vp, ip]),
        "llmrs_generate": (ci, [vp, ci, ci, ci, vp]),
        "llmrs_prefill": (ci, [vp, vp, ci, ci, vp, ip]),
        "llmrs_model_logits": (ci, [vp, vp]),
        "llmrs_rope_table": (ci, [ci, ci, cf, vp, vp]),
        "llmrs_model_decode_kernel_count": (ci, [vp, ip]),
        "llmrs_model_time_decode": (ci, [vp, ci, ci, ci, fp]),
        "llmrs_time_gemv": (ci, [vp, ci, ci, vp, vp, ci, vp, vp, ci, ci, ci, fp]),
        "llmrs_model_time_prefill": (ci, [vp, vp, ci, ci, ci, fp]),
        "llmrs_model_profile_decode": (ci, [vp, ci, ci, vp, vp, ip]),
        "llmrs_attention_decode": (ci, [vp, vp, vp, vp, vp, vp, vp, ci, ci, ci, ci, ci]),
        "llmrs_attention_prefill": (ci, [vp, vp, vp, vp, vp, vp, vp, ci, ci, ci, ci, ci, ci]),
        "llmrs_sample": (ci, [vp, vp, ci, vp, ci, cf, cf, cf, cf, ip]),
        "llmrs_model_sample": (ci, [vp, vp, ci, cf, cf, cf, cf, ip]),
        "llmrs_attention_decode_noalloc": (ci, [vp, vp, vp, vp, vp, vp, vp, ci, ci, ci, ci, ci, vp]),
        "llmrs_model_trace_decode": (ci, [vp, ci, ci, vp, vp, ip]),
        "llmrs_model_tp_region": (ci, [vp, pp, ctypes.POINTER(sz)]),
        "llmrs_model_tp_connect": (ci, [vp, pp]),
        "llmrs_ipc_get_handle": (ci, [vp, vp]),
        "llmrs_ipc_open_handle": (ci, [ci, vp, pp]),
        "llmrs_ipc_close_handle": (ci, [ci, vp]),
        "llmrs_model_set_peer_timeout": (ci, [vp, ci]),
        "llmrs_model_tp_epoch": (ci, [vp, ctypes.POINTER(ctypes.c_uint64)]),
        "llmrs_model_tp_resync": (ci, [vp, ctypes.c_uint64]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def check(rc):
    if rc != OK:
        raise LlmrsError(rc, lib().llmrs_last_error().decode(errors="replace"))


def version():
    return lib().llmrs_version().decode()


def device_count():
    n = ctypes.c_int(0)
    rc = lib().llmrs_device_count(ctypes.byref(n))
    return n.value if rc == OK else 0


def rope_table(head_dim, n_pos, theta=500000.0):
    c = np.zeros((n_pos, head_dim // 2), np.float32)
    s = np.zeros((n_pos, head_dim // 2), np.float32)
    check(lib().llmrs_rope_table(head_dim, n_pos, theta, c.ctypes.data, s.ctypes.data))
    return c, s


def _ptr(a):
    return ctypes.c_void_p(a.ctypes.data)


class Context:
    """A CUDA device + stream (llmrs_ctx)."""

    def __init__(self, device=0):
        h = ctypes.c_void_p()
        check(lib().llmrs_ctx_create(device, ctypes.byref(h)))
        self.h = h
        self.device = device
        self._children = weakref.WeakSet()  # models / tensors that must go first

    def _adopt(self, obj):
        self._children.add(obj)

    def close(self):
        if self.h:
            for child in list(self._children):
                child._release()
            lib().llmrs_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def sync(self):
        check(lib().llmrs_sync(self.h))


class DeviceTensor:
    """Device buffer with a numpy dtype and shape (the reference's Tensor on Device::Cuda)."""

    def __init__(self, ctx, shape, dtype=np.float32):
        self.ctx = ctx
        self.shape = tuple(int(s) for s in np.atleast_1d(shape)) if not isinstance(shape, tuple) else shape
        self.dtype = np.dtype(dtype)
        self.nbytes = int(np.prod(self.shape)) * self.dtype.itemsize
        p = ctypes.c_void_p()
        check(lib().llmrs_malloc(ctx.h, max(self.nbytes, 16), ctypes.byref(p)))
        self.ptr = p
        ctx._adopt(self)

    @classmethod
    def from_numpy(cls, ctx, a, dtype=None):
        a = np.ascontiguousarray(a, dtype=dtype if dtype is not None else a.dtype)
        t = cls(ctx, a.shape, a.dtype)
        if t.nbytes:
            check(lib().llmrs_h2d(ctx.h, t.ptr, _ptr(a), t.nbytes))
        return t

    def numpy(self):
        out = np.empty(self.shape, self.dtype)
        if self.nbytes:
            check(lib().llmrs_d2h(self.ctx.h, _ptr(out), self.ptr, self.nbytes))
        return out

    def free(self):
        if self.ptr and self.ctx.h:
            lib().llmrs_free(self.ctx.h, self.ptr)
        self.ptr = None

    _release = free

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass

    @property
    def size(self):
        return int(np.prod(self.shape))


class QuantWeight:
    """Quantised weight [n, k] on the device in the reference's planar layout."""

    def __init__(self, ctx, codes, scales, n, k, fmt=WFMT_Q4_0, scale_dtype=F32):
        self.n, self.k, self.fmt, self.scale_dtype = n, k, fmt, scale_dtype
        self.codes = DeviceTensor.from_numpy(ctx, codes)
        if scale_dtype == F16:
            scales = np.asarray(scales, np.float32).astype(np.float16)
        else:
            scales = np.asarray(scales, np.float32)
        self.scales = DeviceTensor.from_numpy(ctx, scales)


class CudaBackend:
    """Mirror of `trait Backend` (src/backend.rs:15-40) over the C ABI.

    Ops that return a new Tensor in the reference return a new DeviceTensor;
    in-place ops (add_assign, silu_mul, rope_inplace) mutate their argument.
    """

    def __init__(self, ctx):
        self.ctx = ctx

    def device(self):
        return "Cuda"

    def name(self):
        return lib().llmrs_backend_name().decode()

    def _out(self, shape):
        return DeviceTensor(self.ctx, shape)

    def matmul(self, a, b):
        m, k = a.shape
        k2, n = b.shape
        assert k == k2, "MatMul Dimension mismatch"
        c = self._out((m, n))
        check(lib().llmrs_matmul(self.ctx.h, a.ptr, b.ptr, c.ptr, m, k, n))
        return c

    def matmul_transposed(self, a, b):
        m, k = a.shape
        if isinstance(b, QuantWeight):
            assert b.k == k, "MatMul Transposed dimensions mismatch"
            c = self._out((m, b.n))
            fn = lib().llmrs_matmul_transposed_q4 if b.fmt == WFMT_Q4_0 else lib().llmrs_matmul_transposed_q8
            check(fn(self.ctx.h, a.ptr, b.codes.ptr, b.scales.ptr, b.scale_dtype, c.ptr, m, k, b.n))
            return c
        n, k2 = b.shape
        assert k == k2, "MatMul Transposed dimensions mismatch"
        c = self._out((m, n))
        check(lib().llmrs_matmul_transposed_f32(self.ctx.h, a.ptr, b.ptr, c.ptr, m, k, n))
        return c

    def matmul_slice(self, a, other, rows, cols):
        m, k = a.shape
        assert k == cols, "MatMul Slice mismatch"
        c = self._out((m, rows))
        check(lib().llmrs_matmul_slice(self.ctx.h, a.ptr, other.ptr, c.ptr, m, rows, cols))
        return c

    def add_assign(self, a, b):
        assert a.shape == b.shape, "Shape mismatch"
        check(lib().llmrs_add_assign(self.ctx.h, a.ptr, b.ptr, a.size))

    def silu_mul(self, gate, up):
        assert gate.shape == up.shape, "Shape mismatch"
        check(lib().llmrs_silu_mul(self.ctx.h, gate.ptr, up.ptr, gate.size))

    def rope_inplace(self, x, start_pos, theta=500000.0):
        head_dim = x.shape[-1]
        rows = x.size // head_dim
        check(lib().llmrs_rope_inplace(self.ctx.h, x.ptr, rows, head_dim, start_pos, theta))

    def rms_norm(self, x, w, eps):
        cols = x.shape[-1]
        rows = x.size // cols
        y = self._out(x.shape)
        check(lib().llmrs_rms_norm(self.ctx.h, x.ptr, w.ptr, y.ptr, rows, cols, eps))
        return y

    def softmax(self, x):
        cols = x.shape[-1]
        rows = x.size // cols
        y = self._out(x.shape)
        check(lib().llmrs_softmax(self.ctx.h, x.ptr, y.ptr, rows, cols))
        return y

    def scale(self, x, value):
        y = self._out(x.shape)
        check(lib().llmrs_scale(self.ctx.h, x.ptr, y.ptr, x.size, value))
        return y

    def copy_from(self, t):
        y = self._out(t.shape)
        check(lib().llmrs_copy_from(self.ctx.h, t.ptr, y.ptr, t.size))
        return y

    def attention_decode(self, qkv, kcache, vcache, rope_cos, rope_sin, n_heads, n_kv_heads, head_dim, pos):
        """Fused decode attention (one token at `pos`); appends k/v to the caches."""
        out = self._out((n_heads * head_dim,))
        max_seq = kcache.shape[1]
        check(lib().llmrs_attention_decode(self.ctx.h, qkv.ptr, kcache.ptr, vcache.ptr, rope_cos.ptr, rope_sin.ptr,
                                           out.ptr, n_heads, n_kv_heads, head_dim, max_seq, pos))
        return out

    def attention_prefill(self, qkv, kcache, vcache, rope_cos, rope_sin, n_heads, n_kv_heads, head_dim, start_pos):
        """Causal attention of qkv's rows at start_pos..; RoPEs q in place, appends k/v."""
        n_rows = qkv.shape[0]
        out = self._out((n_rows, n_heads * head_dim))
        max_seq = kcache.shape[1]
        check(lib().llmrs_attention_prefill(self.ctx.h, qkv.ptr, kcache.ptr, vcache.ptr, rope_cos.ptr, rope_sin.ptr,
                                            out.ptr, n_rows, n_heads, n_kv_heads, head_dim, max_seq, start_pos))
        return out

    def sample(self, logits, recent, repeat_penalty, temperature, top_p, u):
        """Next-token sampling of src/main.rs:192-305 over device logits (u: the uniform draw)."""
        r = np.ascontiguousarray(recent, np.int32)
        tok = ctypes.c_int(-1)
        check(lib().llmrs_sample(self.ctx.h, logits.ptr, int(logits.nbytes // 4), _ptr(r) if r.size else None,
                                 int(r.size), float(repeat_penalty), float(temperature), float(top_p), float(u),
                                 ctypes.byref(tok)))
        return tok.value

    # CpuBackend::quantize_row_q8_0 and Tensor::quantize_q4 (bit-exact)
    def quantize_row_q8_0(self, x):
        k = x.shape[-1]
        rows = x.size // k
        q = DeviceTensor(self.ctx, x.shape, np.int8)
        s = DeviceTensor(self.ctx, tuple(x.shape[:-1]) + (k // 32,), np.float32)
        check(lib().llmrs_quantize_row_q8_0(self.ctx.h, x.ptr, q.ptr, s.ptr, rows, k))
        return q, s

    def rms_norm_quantize_q8_0(self, x, w, eps):
        """RMSNorm + Q8_0 of one row as the decode GEMV prologue computes it: (codes, scales)."""
        k = x.size
        q = DeviceTensor(self.ctx, (k,), np.int8)
        s = DeviceTensor(self.ctx, (k // 32,), np.float32)
        check(lib().llmrs_rms_norm_quantize_q8_0(self.ctx.h, x.ptr, w.ptr, q.ptr, s.ptr, k, eps))
        return q.numpy(), s.numpy()

    def quantize_q4(self, w):
        n = w.size
        qs = DeviceTensor(self.ctx, ((n + 1) // 2,), np.uint8)
        sc = DeviceTensor(self.ctx, ((n + 31) // 32,), np.float32)
        check(lib().llmrs_quantize_q4(self.ctx.h, w.ptr, n, qs.ptr, sc.ptr))
        return qs, sc


class Model:
    """Device-resident Llama model (llmrs_model)."""

    def __init__(self, ctx, cfg):
        self.ctx = ctx
        self.cfg = dict(cfg)
        self.cfg.setdefault("scale_dtype", F16)
        self.cfg.setdefault("tp_rank", 0)
        self.cfg.setdefault("tp_size", 1)
        self.tp = max(1, int(self.cfg["tp_size"]))
        self.vocab_local = self.cfg["vocab"] // self.tp
        self._peer_maps = []
        c = Config(**{f: self.cfg[f] for f, _ in Config._fields_})
        h = ctypes.c_void_p()
        check(lib().llmrs_model_create(ctx.h, ctypes.byref(c), ctypes.byref(h)))
        self.h = h
        ctx._adopt(self)

    def close(self):
        if self.h and self.ctx.h:
            for ptr in self._peer_maps:
                lib().llmrs_ipc_close_handle(self.ctx.device, ptr)
            self._peer_maps = []
            lib().llmrs_model_destroy(self.h)
        self.h = None

    _release = close

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def init_synthetic(self, seed):
        check(lib().llmrs_model_init_synthetic(self.h, seed))

    def set_weight(self, layer, which, codes, scales=None):
        codes = np.ascontiguousarray(codes)
        sc = None if scales is None else np.ascontiguousarray(scales, np.float32)
        check(lib().llmrs_model_set_weight(self.h, layer, which, _ptr(codes),
                                           None if sc is None else _ptr(sc)))

    def load_weight(self, layer, which, data):
        """One checkpoint tensor, whole and unsharded (llmrs_model_load_weight):
        float32, or bfloat16 bits as uint16, in the safetensors layout."""
        a = np.ascontiguousarray(data)
        if a.dtype == np.float32:
            dt = F32
        elif a.dtype == np.uint16:
            dt = BF16
        else:
            raise TypeError("load_weight takes float32 or bfloat16 bits (uint16), not %s" % a.dtype)
        check(lib().llmrs_model_load_weight(self.h, int(layer), int(which), _ptr(a), dt))

    def kv_fill(self, layer, k, v):
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        check(lib().llmrs_kv_fill(self.h, layer, _ptr(k), _ptr(v), k.shape[1]))

    def kv_fill_synthetic(self, seed, n_pos):
        check(lib().llmrs_kv_fill_synthetic(self.h, seed, n_pos))

    def kv_read(self, layer, n_pos):
        c = self.cfg
        k = np.zeros((c["n_kv_heads"] // self.tp, n_pos, c["head_dim"]), np.float32)
        v = np.zeros_like(k)
        check(lib().llmrs_kv_read(self.h, layer, _ptr(k), _ptr(v), n_pos))
        return k, v

    def decode_step(self, token, pos, want_logits=True):
        logits = np.zeros(self.vocab_local, np.float32) if want_logits else None
        am = ctypes.c_int(-1)
        check(lib().llmrs_decode_step(self.h, int(token), int(pos),
                                      None if logits is None else _ptr(logits), ctypes.byref(am)))
        return am.value, logits

    def generate(self, token, pos, n_steps):
        out = np.zeros(n_steps, np.int32)
        check(lib().llmrs_generate(self.h, int(token), int(pos), int(n_steps), _ptr(out)))
        return out

    def prefill(self, ids, start_pos, want_logits=True):
        ids = np.ascontiguousarray(ids, np.int32)
        logits = np.zeros(self.vocab_local, np.float32) if want_logits else None
        am = ctypes.c_int(-1)
        check(lib().llmrs_prefill(self.h, _ptr(ids), ids.size, int(start_pos),
                                  None if logits is None else _ptr(logits), ctypes.byref(am)))
        return am.value, logits

    def sample(self, recent, repeat_penalty, temperature, top_p, u):
        """Sample the next token from the last step's logits (one GPU)."""
        r = np.ascontiguousarray(recent, np.int32)
        tok = ctypes.c_int(-1)
        check(lib().llmrs_model_sample(self.h, _ptr(r) if r.size else None, int(r.size), float(repeat_penalty),
                                       float(temperature), float(top_p), float(u), ctypes.byref(tok)))
        return tok.value

    def logits(self):
        out = np.zeros(self.vocab_local, np.float32)
        check(lib().llmrs_model_logits(self.h, _ptr(out)))
        return out

    # ---- tensor parallel: one process per GPU
    def tp_handle(self):
        """IPC handle (bytes) of this rank's communication region."""
        ptr, n = ctypes.c_void_p(), ctypes.c_size_t()
        check(lib().llmrs_model_tp_region(self.h, ctypes.byref(ptr), ctypes.byref(n)))
        hbuf = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
        check(lib().llmrs_ipc_get_handle(ptr, hbuf))
        return hbuf.raw, ptr.value

    def tp_connect(self, handles):
        """handles[q] = rank q's tp_handle()[0]; maps the peers' regions (over
        NVLink) and links the model to them."""
        rank = self.cfg["tp_rank"]
        own = self.tp_handle()[1]
        regions = (ctypes.c_void_p * self.tp)()
        for q, hb in enumerate(handles):
            if q == rank:
                regions[q] = own
                continue
            ptr = ctypes.c_void_p()
            check(lib().llmrs_ipc_open_handle(self.ctx.device, ctypes.create_string_buffer(hb, IPC_HANDLE_BYTES),
                                              ctypes.byref(ptr)))
            self._peer_maps.append(ptr.value)
            regions[q] = ptr.value
        check(lib().llmrs_model_tp_connect(self.h, regions))

    def set_peer_timeout(self, ms):
        """Longest wait (ms) of a decode-step kernel for another rank."""
        check(lib().llmrs_model_set_peer_timeout(self.h, int(ms)))

    def tp_epoch(self):
        """Decode steps this rank has completed."""
        e = ctypes.c_uint64(0)
        check(lib().llmrs_model_tp_epoch(self.h, ctypes.byref(e)))
        return e.value

    def tp_resync(self, epoch):
        """Set this rank's step count (and arrival counters) to `epoch`; see resync_tensor_parallel."""
        check(lib().llmrs_model_tp_resync(self.h, int(epoch)))

    def decode_kernel_count(self):
        n = ctypes.c_int(0)
        check(lib().llmrs_model_decode_kernel_count(self.h, ctypes.byref(n)))
        return n.value

    KERNEL_KINDS = ("qkv_gemv", "attention", "o_gemv", "gate_up_gemv", "down_gemv", "lm_head_gemv")

    def profile_decode(self, token, pos):
        """Per-kernel durations (ms) of one decode step, kernel by kernel."""
        cap = self.decode_kernel_count() + 8
        ms = np.zeros(cap, np.float32)
        kinds = np.zeros(cap, np.int32)
        n = ctypes.c_int(cap)
        check(lib().llmrs_model_profile_decode(self.h, int(token), int(pos), _ptr(ms), _ptr(kinds),
                                               ctypes.byref(n)))
        return [(self.KERNEL_KINDS[k], float(t)) for k, t in zip(kinds[:n.value], ms[:n.value])]

    def trace_decode(self, token, pos):
        """Device timeline of one graph-launched decode step: list of
        (kind, start_ns, go_ns, ready_ns, end_ns) relative to the first kernel's
        start (ready: last CTA done with its activation prologue)."""
        cap = self.decode_kernel_count()
        marks = np.zeros(4 * cap, np.uint64)
        kinds = np.zeros(cap, np.int32)
        n = ctypes.c_int(cap)
        check(lib().llmrs_model_trace_decode(self.h, int(token), int(pos), _ptr(marks), _ptr(kinds), ctypes.byref(n)))
        marks = marks[:4 * n.value].reshape(-1, 4).astype(np.int64)
        t0 = int(marks[0, 0])
        return [(self.KERNEL_KINDS[k], int(a - t0), int(b - t0), int(r - t0), int(c - t0))
                for k, (a, b, r, c) in zip(kinds, marks)]

    def time_decode(self, token, pos, iters):
        ms = ctypes.c_float(0)
        check(lib().llmrs_model_time_decode(self.h, int(token), int(pos), int(iters), ctypes.byref(ms)))
        return ms.value

    def time_prefill(self, ids, start_pos, iters):
        """Device ms of one tensor-core prefill of `ids` (mean of `iters`)."""
        ids = np.ascontiguousarray(ids, np.int32)
        ms = ctypes.c_float(0)
        check(lib().llmrs_model_time_prefill(self.h, _ptr(ids), ids.size, int(start_pos), int(iters),
                                             ctypes.byref(ms)))
        return ms.value


def read_safetensors(path):
    """{name: (array, dtype name)} of a safetensors file, memory-mapped: an
    8-byte little-endian header length, a JSON header {name: {dtype, shape,
    data_offsets}}, then the data.  BF16 tensors come back as their uint16 bits."""
    import json
    import struct
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
    raw = np.memmap(path, np.uint8, mode="r", offset=8 + n)
    kinds = {"F32": np.float32, "BF16": np.uint16}
    out = {}
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        if meta["dtype"] not in kinds:  # the reference's read_tensor bails the same way
            raise ValueError("Unsupported dtype: %s (%s)" % (meta["dtype"], name))
        b, e = meta["data_offsets"]
        out[name] = (raw[b:e].view(kinds[meta["dtype"]]).reshape(meta["shape"]), meta["dtype"])
    return out


def load_safetensors(model, path):
    """Load a Llama checkpoint into `model` with the reference's tensor names
    and layout decisions (src/core/loader.rs:100-198): q/k/v/o, gate/up/down,
    the two norms per layer, the embedding, the final norm and lm_head.weight
    (absent: the LM head is quantize_q4 of the embedding, loader.rs:186-190).
    Every tensor goes whole to llmrs_model_load_weight, which quantises it on
    the device and keeps this rank's shard."""
    t = read_safetensors(path)

    def put(layer, which, name):
        if name not in t:
            raise KeyError("Tensor not found: %s" % name)
        model.load_weight(layer, which, t[name][0])

    put(-1, W_EMBED, "model.embed_tokens.weight")
    for i in range(model.cfg["n_layers"]):
        p = "model.layers.%d." % i
        for which, name in ((W_Q, "self_attn.q_proj"), (W_K, "self_attn.k_proj"), (W_V, "self_attn.v_proj"),
                            (W_O, "self_attn.o_proj"), (W_GATE, "mlp.gate_proj"), (W_UP, "mlp.up_proj"),
                            (W_DOWN, "mlp.down_proj"), (W_ATTN_NORM, "input_layernorm"),
                            (W_MLP_NORM, "post_attention_layernorm")):
            put(i, which, p + name + ".weight")
    put(-1, W_FINAL_NORM, "model.norm.weight")
    if "lm_head.weight" in t:
        put(-1, W_LM_HEAD, "lm_head.weight")
    elif not model.cfg["tied_embeddings"]:
        put(-1, W_LM_HEAD, "model.embed_tokens.weight")  # the reference's fallback: quantize_q4(embedding)


def time_gemv(ctx, codes, scales, x, y, n, k, reps, fmt=WFMT_Q4_0, scale_dtype=F16):
    """Device microseconds per launch of the batch-1 GEMV (llmrs_time_gemv):
    `codes` / `scales` are device addresses (ints) of weight copies [n][k] that
    are multiplied with x[k] into y[n] back to back in one CUDA graph."""
    assert len(codes) == len(scales) and codes
    c = (ctypes.c_void_p * len(codes))(*[int(p) for p in codes])
    s = (ctypes.c_void_p * len(scales))(*[int(p) for p in scales])
    us = ctypes.c_float(0)
    check(lib().llmrs_time_gemv(ctx.h, int(fmt), int(scale_dtype), ctypes.cast(c, ctypes.c_void_p),
                                ctypes.cast(s, ctypes.c_void_p), len(codes), ctypes.c_void_p(int(x)),
                                ctypes.c_void_p(int(y)), int(n), int(k), int(reps), ctypes.byref(us)))
    return us.value


def resync_tensor_parallel(model, group=None):
    """After a decode step that failed on some rank (LLMRS_ETIMEDOUT): every
    rank calls this, with no step running.  The ranks agree on the largest
    completed-step count and set it (llmrs_model_tp_resync) between two
    barriers, so the next step's exchanges match again.  Returns that count."""
    import torch.distributed as dist

    dist.barrier(group)
    epochs = [None] * dist.get_world_size(group)
    dist.all_gather_object(epochs, int(model.tp_epoch()), group=group)
    agreed = max(epochs)
    model.tp_resync(agreed)
    dist.barrier(group)
    return agreed


def connect_tensor_parallel(model, group=None):
    """Exchange the ranks' IPC handles over torch.distributed (any backend;
    host plumbing only) and connect `model`; every rank calls this once."""
    import torch.distributed as dist

    handle, _ = model.tp_handle()
    handles = [None] * dist.get_world_size(group)
    dist.all_gather_object(handles, handle, group=group)
    model.tp_connect(handles)
    dist.barrier(group)


def tp_sample(model, recent, repeat_penalty, temperature, top_p, u, group=None):
    """Next-token sampling (src/main.rs:192-305) for a tensor-parallel model.

    Each rank holds the last step's logits for its vocabulary rows
    [rank*V/T, (rank+1)*V/T).  The shards are gathered over the host channel
    (torch.distributed, any backend), and every rank runs the device sampler
    (llmrs_sample) over the full vocabulary on its own GPU with the same draw
    `u`, so all ranks pick the same token.  Every rank calls this in the same
    order with the same arguments."""
    import torch
    import torch.distributed as dist

    shard = torch.from_numpy(model.logits())
    parts = [torch.empty_like(shard) for _ in range(dist.get_world_size(group))]
    dist.all_gather(parts, shard, group=group)
    full = DeviceTensor.from_numpy(model.ctx, torch.cat(parts).numpy())
    try:
        return CudaBackend(model.ctx).sample(full, recent, repeat_penalty, temperature, top_p, u)
    finally:
        full.free()

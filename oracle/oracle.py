"""ctypes view of the CPU oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py.  The shipped CUDA library never loads it.

The oracle restates hedone21/llm.rs's x86_64 CPU path (src/backend/cpu.rs,
src/core/{tensor,layer,model,loader}.rs); see oracle.h for the file:line map and
for which parts the reference's own tests pin ("parity unpinned" otherwise).
"""
import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

F32P = ctypes.POINTER(ctypes.c_float)
U8P = ctypes.POINTER(ctypes.c_uint8)
I8P = ctypes.POINTER(ctypes.c_int8)
I32P = ctypes.POINTER(ctypes.c_int32)


class OrcConfig(ctypes.Structure):
    _fields_ = [
        ("n_layers", ctypes.c_int), ("hidden", ctypes.c_int), ("n_heads", ctypes.c_int),
        ("n_kv_heads", ctypes.c_int), ("head_dim", ctypes.c_int), ("ffn", ctypes.c_int),
        ("vocab", ctypes.c_int), ("max_seq", ctypes.c_int), ("rms_eps", ctypes.c_float),
        ("rope_theta", ctypes.c_float), ("weight_format", ctypes.c_int),
        ("tied_embeddings", ctypes.c_int),
    ]


W_Q, W_K, W_V, W_O, W_GATE_UP, W_DOWN, W_ATTN_NORM, W_MLP_NORM, W_EMBED, W_FINAL_NORM, W_LM_HEAD = range(11)


def build():
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        vp = ctypes.c_void_p
        sz = ctypes.c_size_t
        ci = ctypes.c_int
        cf = ctypes.c_float
        u64 = ctypes.c_uint64
        u32 = ctypes.c_uint32
        sig = {
            "orc_set_threads": (None, [ci]),
            "orc_get_threads": (ci, []),
            "orc_quantize_row_q8_0": (None, [F32P, ci, I8P, F32P]),
            "orc_quantize_q4": (None, [F32P, sz, U8P, F32P]),
            "orc_dequantize_q4": (None, [U8P, F32P, sz, F32P]),
            "orc_matmul_transposed_q4": (None, [F32P, ci, ci, U8P, F32P, ci, F32P]),
            "orc_matmul_transposed_q8w": (None, [F32P, ci, ci, I8P, F32P, ci, F32P]),
            "orc_matmul_transposed_f32": (None, [F32P, ci, ci, F32P, ci, F32P]),
            "orc_matmul_f32": (None, [F32P, ci, ci, F32P, ci, F32P]),
            "orc_matmul_slice": (None, [F32P, ci, ci, F32P, ci, F32P]),
            "orc_add_assign": (None, [F32P, F32P, sz]),
            "orc_silu_mul": (None, [F32P, F32P, sz]),
            "orc_rope_inplace": (None, [F32P, ci, ci, ci, cf]),
            "orc_rms_norm": (None, [F32P, F32P, F32P, ci, ci, cf]),
            "orc_softmax": (None, [F32P, F32P, ci, ci]),
            "orc_scale": (None, [F32P, F32P, sz, cf]),
            "orc_model_create": (vp, [ctypes.POINTER(OrcConfig), ci]),
            "orc_model_destroy": (None, [vp]),
            "orc_model_init_synthetic": (None, [vp, u64]),
            "orc_model_kv_fill_synthetic": (None, [vp, u64, ci]),
            "orc_model_forward": (ci, [vp, I32P, ci, ci, F32P]),
            "orc_model_forward_embeds": (ci, [vp, F32P, ci, ci, F32P]),
            "orc_model_tensor": (ci, [vp, ci, ci, ctypes.POINTER(vp), ctypes.POINTER(vp),
                                      ctypes.POINTER(sz), ctypes.POINTER(sz)]),
            "orc_model_set_trace": (None, [vp, F32P]),
            "orc_model_kcache": (F32P, [vp, ci]),
            "orc_model_vcache": (F32P, [vp, ci]),
            "orc_model_cache_heads": (sz, [vp]),
            "orc_argmax": (ci, [F32P, ci]),
            "orc_sample": (ci, [F32P, ci, I32P, ci, cf, cf, cf, cf, F32P]),
            "orc_top2_margin": (cf, [F32P, ci]),
            "orc_synth_q4": (None, [u64, u32, u32, sz, sz, U8P, F32P]),
            "orc_synth_q8": (None, [u64, u32, u32, sz, sz, I8P, F32P]),
            "orc_synth_normal": (None, [u64, u32, u32, sz, cf, cf, F32P]),
            "orc_f32_to_f16": (ctypes.c_uint16, [cf]),
            "orc_f16_to_f32": (cf, [ctypes.c_uint16]),
            "orc_synth_token": (u32, [u64, u64, u32]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a, t):
    return a.ctypes.data_as(t)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def set_threads(n):
    lib().orc_set_threads(int(n))


def get_threads():
    return lib().orc_get_threads()


# ---- Backend-trait restatement ---------------------------------------------
def quantize_row_q8_0(x):
    x = _f32(x)
    k = x.shape[-1]
    q = np.zeros(k, np.int8)
    s = np.zeros(k // 32, np.float32)
    lib().orc_quantize_row_q8_0(_p(x, F32P), k, _p(q, I8P), _p(s, F32P))
    return q, s


def quantize_q4(w):
    w = _f32(w).ravel()
    n = w.size
    qs = np.zeros((n + 1) // 2, np.uint8)
    sc = np.zeros((n + 31) // 32, np.float32)
    lib().orc_quantize_q4(_p(w, F32P), n, _p(qs, U8P), _p(sc, F32P))
    return qs, sc


def dequantize_q4(qs, sc, n):
    out = np.zeros(n, np.float32)
    qs = np.ascontiguousarray(qs, np.uint8)
    sc = _f32(sc)
    lib().orc_dequantize_q4(_p(qs, U8P), _p(sc, F32P), n, _p(out, F32P))
    return out


def matmul_transposed_q4(a, qs, sw, n):
    a = _f32(np.atleast_2d(a))
    m, k = a.shape
    qs = np.ascontiguousarray(qs, np.uint8)
    sw = _f32(sw)
    c = np.zeros((m, n), np.float32)
    lib().orc_matmul_transposed_q4(_p(a, F32P), m, k, _p(qs, U8P), _p(sw, F32P), n, _p(c, F32P))
    return c


def matmul_transposed_q8w(a, qw, sw, n):
    a = _f32(np.atleast_2d(a))
    m, k = a.shape
    qw = np.ascontiguousarray(qw, np.int8)
    sw = _f32(sw)
    c = np.zeros((m, n), np.float32)
    lib().orc_matmul_transposed_q8w(_p(a, F32P), m, k, _p(qw, I8P), _p(sw, F32P), n, _p(c, F32P))
    return c


def matmul_transposed_f32(a, b):
    a = _f32(np.atleast_2d(a))
    b = _f32(b)
    m, k = a.shape
    n = b.shape[0]
    c = np.zeros((m, n), np.float32)
    lib().orc_matmul_transposed_f32(_p(a, F32P), m, k, _p(b, F32P), n, _p(c, F32P))
    return c


def matmul_f32(a, b):
    a = _f32(np.atleast_2d(a))
    b = _f32(b)
    m, k = a.shape
    n = b.shape[1]
    c = np.zeros((m, n), np.float32)
    lib().orc_matmul_f32(_p(a, F32P), m, k, _p(b, F32P), n, _p(c, F32P))
    return c


def matmul_slice(a, other, rows, cols):
    a = _f32(np.atleast_2d(a))
    other = _f32(other)
    m, k = a.shape
    assert k == cols
    c = np.zeros((m, rows), np.float32)
    lib().orc_matmul_slice(_p(a, F32P), m, k, _p(other, F32P), rows, _p(c, F32P))
    return c


def add_assign(a, b):
    a = _f32(a).copy()
    b = _f32(b)
    lib().orc_add_assign(_p(a, F32P), _p(b, F32P), a.size)
    return a


def silu_mul(g, u):
    g = _f32(g).copy()
    u = _f32(u)
    lib().orc_silu_mul(_p(g, F32P), _p(u, F32P), g.size)
    return g


def rope_inplace(x, head_dim, start_pos, theta=500000.0):
    x = _f32(x).copy()
    rows = x.size // head_dim
    lib().orc_rope_inplace(_p(x, F32P), rows, head_dim, start_pos, theta)
    return x


def rms_norm(x, w, eps):
    x = _f32(np.atleast_2d(x))
    w = _f32(w)
    rows, cols = x.shape
    y = np.zeros_like(x)
    lib().orc_rms_norm(_p(x, F32P), _p(w, F32P), _p(y, F32P), rows, cols, eps)
    return y


def softmax(x):
    x = _f32(np.atleast_2d(x))
    rows, cols = x.shape
    y = np.zeros_like(x)
    lib().orc_softmax(_p(x, F32P), _p(y, F32P), rows, cols)
    return y


def scale(x, v):
    x = _f32(x)
    y = np.zeros_like(x)
    lib().orc_scale(_p(x, F32P), _p(y, F32P), x.size, v)
    return y


def argmax(v):
    v = _f32(v)
    return lib().orc_argmax(_p(v, F32P), v.size)


def sample(logits, recent, penalty, temperature, top_p, u):
    """src/main.rs:192-305 with the caller's uniform draw u: (token, margin)."""
    v = _f32(logits)
    r = np.ascontiguousarray(recent, np.int32)
    m = np.zeros(1, np.float32)
    t = lib().orc_sample(_p(v, F32P), v.size, _p(r, I32P), r.size, float(penalty), float(temperature), float(top_p),
                         float(u), _p(m, F32P))
    return int(t), float(m[0])


def top2_margin(v):
    v = _f32(v)
    return lib().orc_top2_margin(_p(v, F32P), v.size)


# ---- synthetic generator ----------------------------------------------------
def synth_q4(seed, layer, tensor, n, k):
    qs = np.zeros(n * k // 2, np.uint8)
    sc = np.zeros(n * k // 32, np.float32)
    lib().orc_synth_q4(seed, layer, tensor, n, k, _p(qs, U8P), _p(sc, F32P))
    return qs, sc


def synth_q8(seed, layer, tensor, n, k):
    qw = np.zeros(n * k, np.int8)
    sc = np.zeros(n * k // 32, np.float32)
    lib().orc_synth_q8(seed, layer, tensor, n, k, _p(qw, I8P), _p(sc, F32P))
    return qw, sc


def synth_normal(seed, layer, tensor, n, mu=0.0, sd=1.0):
    out = np.zeros(n, np.float32)
    lib().orc_synth_normal(seed, layer, tensor, n, mu, sd, _p(out, F32P))
    return out


def synth_token(seed, i, vocab):
    return int(lib().orc_synth_token(seed, i, vocab))


def f32_to_f16_bits(x):
    return int(lib().orc_f32_to_f16(float(x)))


def f16_bits_to_f32(h):
    return float(lib().orc_f16_to_f32(int(h)))


# ---- model --------------------------------------------------------------------
class Model:
    """Restated LlamaModel (src/core/model.rs) over synthetic weights."""

    def __init__(self, cfg, expand_gqa=False):
        self.cfg = dict(cfg)
        c = OrcConfig(**{f: self.cfg[f] for f, _ in OrcConfig._fields_})
        self._c = c
        self.h = lib().orc_model_create(ctypes.byref(c), int(expand_gqa))
        if not self.h:
            raise MemoryError("orc_model_create failed")

    def close(self):
        if self.h:
            lib().orc_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def init_synthetic(self, seed):
        lib().orc_model_init_synthetic(self.h, seed)

    def kv_fill_synthetic(self, seed, n_pos):
        lib().orc_model_kv_fill_synthetic(self.h, seed, n_pos)

    def forward(self, ids, start_pos):
        ids = np.ascontiguousarray(ids, np.int32)
        out = np.zeros(self.cfg["vocab"], np.float32)
        rc = lib().orc_model_forward(self.h, _p(ids, I32P), ids.size, start_pos, _p(out, F32P))
        if rc != 0:
            raise ValueError("orc_model_forward failed: %d" % rc)
        return out

    def forward_traced(self, ids, start_pos):
        """forward(), also returning the last row's residual stream entering
        each RMSNorm: [2*n_layers+1][hidden] (attention norm of layer l at 2l,
        MLP norm at 2l+1, final norm last)."""
        buf = np.zeros((2 * self.cfg["n_layers"] + 1, self.cfg["hidden"]), np.float32)
        lib().orc_model_set_trace(self.h, _p(buf, F32P))
        try:
            logits = self.forward(ids, start_pos)
        finally:
            lib().orc_model_set_trace(self.h, None)
        return logits, buf

    def norm_weight(self, layer, which):
        """attention (0) / MLP (1) RMSNorm weight of `layer`, or the final norm (layer -1)"""
        w, _ = self.tensor(layer, W_FINAL_NORM if layer < 0 else (W_ATTN_NORM if which == 0 else W_MLP_NORM))
        return np.asarray(w, np.float32).reshape(-1)

    def forward_embeds(self, x, start_pos):
        x = _f32(np.atleast_2d(x))
        out = np.zeros(self.cfg["vocab"], np.float32)
        rc = lib().orc_model_forward_embeds(self.h, _p(x, F32P), x.shape[0], start_pos, _p(out, F32P))
        if rc != 0:
            raise ValueError("orc_model_forward_embeds failed: %d" % rc)
        return out

    def tensor(self, layer, which):
        qs = ctypes.c_void_p()
        sc = ctypes.c_void_p()
        n = ctypes.c_size_t()
        k = ctypes.c_size_t()
        rc = lib().orc_model_tensor(self.h, layer, which, ctypes.byref(qs), ctypes.byref(sc),
                                    ctypes.byref(n), ctypes.byref(k))
        if rc != 0:
            raise ValueError("bad tensor")
        n, k = n.value, k.value
        if not sc.value:
            return np.ctypeslib.as_array(ctypes.cast(qs, F32P), shape=(n * k,)).copy(), None
        if self.cfg["weight_format"] == 0 or (which == W_LM_HEAD and self.cfg["tied_embeddings"]):
            codes = np.ctypeslib.as_array(ctypes.cast(qs, U8P), shape=(n * k // 2,)).copy()
        else:
            codes = np.ctypeslib.as_array(ctypes.cast(qs, I8P), shape=(n * k,)).copy()
        scales = np.ctypeslib.as_array(ctypes.cast(sc, F32P), shape=(n * k // 32,)).copy()
        return codes, scales

    def set_tensor(self, layer, which, codes, scales=None):
        """Overwrite one of the model's tensors in place (the layout tensor()
        returns: quantised codes + f32 scales, or an f32 vector/matrix), e.g.
        with the quantised weights of a checkpoint."""
        qs = ctypes.c_void_p()
        sc = ctypes.c_void_p()
        n = ctypes.c_size_t()
        k = ctypes.c_size_t()
        rc = lib().orc_model_tensor(self.h, layer, which, ctypes.byref(qs), ctypes.byref(sc),
                                    ctypes.byref(n), ctypes.byref(k))
        if rc != 0:
            raise ValueError("bad tensor")
        c = np.ascontiguousarray(codes)
        size = n.value * k.value
        if not sc.value:
            want = size * 4
        elif self.cfg["weight_format"] == 0 or (which == W_LM_HEAD and self.cfg["tied_embeddings"]):
            want = size // 2
        else:
            want = size
        if c.nbytes != want:
            raise ValueError("tensor %d of layer %d takes %d bytes, got %d" % (which, layer, want, c.nbytes))
        ctypes.memmove(qs.value, c.ctypes.data, want)
        if sc.value:
            s32 = np.ascontiguousarray(scales, np.float32)
            if s32.size != size // 32:
                raise ValueError("scales of tensor %d: %d values, need %d" % (which, s32.size, size // 32))
            ctypes.memmove(sc.value, s32.ctypes.data, s32.nbytes)

    def kcache(self, layer):
        c = self.cfg
        heads = lib().orc_model_cache_heads(self.h)
        p = lib().orc_model_kcache(self.h, layer)
        return np.ctypeslib.as_array(p, shape=(heads, c["max_seq"], c["head_dim"])).copy()

    def vcache(self, layer):
        """V cache in the reference's transposed layout [heads][D][max_seq]."""
        c = self.cfg
        heads = lib().orc_model_cache_heads(self.h)
        p = lib().orc_model_vcache(self.h, layer)
        return np.ctypeslib.as_array(p, shape=(heads, c["head_dim"], c["max_seq"])).copy()

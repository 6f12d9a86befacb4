"""ctypes bindings for oracle/_ref/libturbo_ref.so -- test infrastructure only.

The library is the reference Turbo.cpp tensor library compiled from its own
sources (oracle/Makefile) with the extern "C" shim oracle/ref_shim.cpp.  Only the
tests, `__graft_entry__.smoke()` and bench.py's CPU-baseline leg load it.
"""
import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_ref", "libturbo_ref.so")

_P = ctypes.c_void_p
_SZ = ctypes.c_size_t
_SZP = ctypes.POINTER(ctypes.c_size_t)
_I = ctypes.c_int
_F = ctypes.c_float

_SIGS = {
    "ref_add": (_I, [_P, _SZP, _I, _P, _SZP, _I, _P]),
    "ref_add_views": (_I, [_P, _SZ, _SZ, _SZP, _SZP, _I, _P, _SZ, _SZ, _SZP, _SZP, _I, _P]),
    "ref_scale": (_I, [_P, _SZ, _SZ, _SZP, _SZP, _I, _F, _P]),
    "ref_copy": (_I, [_P, _SZ, _SZ, _SZP, _SZP, _I, _P, _SZ, _SZ, _SZP, _SZP, _I]),
    "ref_contiguous": (_I, [_P, _SZ, _SZ, _SZP, _SZP, _I, _P]),
    "ref_rmsnorm": (_I, [_P, _SZ, _SZ, _P, _F, _P]),
    "ref_swiglu": (_I, [_P, _P, _SZ, _P]),
    "ref_softmax": (_I, [_P, _SZ, _SZ, _P]),
    "ref_greedy_sample": (_I, [_P, _SZ]),
    "ref_sample_top_p": (None, [_P, _SZ, _F, _F, _I, _P]),
    "ref_rope": (_I, [_P, _SZ, _SZ, _SZP, _SZP, _I, _SZ, _SZ, _F, _SZ]),
    "ref_rope_tables": (None, [_SZ, _SZ, _F, _P, _P]),
    "ref_embedding": (_I, [_P, _I, _SZ, _SZ, _P, _SZ, _P]),
    "ref_matmul_quant": (_I, [_P, _SZ, _SZ, _P, _I, _SZ, _P]),
    "ref_matmul_quant_repeat": (_I, [_P, _SZ, _SZ, _P, _I, _SZ, _P, _I]),
    "ref_matmul_f32": (_I, [_P, _SZ, _SZ, _SZP, _SZP, _P, _SZ, _SZ, _SZP, _SZP, _I, _P]),
    "ref_linear_f32": (_I, [_P, _SZ, _SZ, _P, _SZ, _P, _P]),
    "ref_dequantize_row_q8_0": (None, [_P, _P, _I]),
    "ref_quantize_row_q8_0": (None, [_P, _P, _I]),
    "ref_vec_dot_q8_0_f32": (_F, [_I, _P, _P]),
    "ref_vec_dot_q4_0_q8_0": (_F, [_I, _P, _P]),
    "ref_vec_dot_q4_0_q8_0_avx2": (_F, [_I, _P, _P]),
    "ref_f32_to_f16": (ctypes.c_ushort, [_F]),
    "ref_f16_to_f32": (_F, [ctypes.c_ushort]),
    "ref_model_load": (_P, [ctypes.c_char_p]),
    "ref_model_free": (None, [_P]),
    "ref_model_generate": (_I, [_P, _P, _SZ, _SZ, _SZ, _P, _P, _P,
                                ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double)]),
}

DT_FP32, DT_Q8_0, DT_Q4_0 = 0, 2, 3
STATUS_EXC = {1: ValueError, 2: IndexError, 3: RuntimeError, 4: RuntimeError}

_lib = None


def available():
    return os.path.exists(LIB_PATH)


def lib():
    global _lib
    if _lib is None:
        if not available():
            raise FileNotFoundError(LIB_PATH + " is not built (make -C oracle ref)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def sz(seq):
    seq = [int(v) for v in seq]
    return (ctypes.c_size_t * max(1, len(seq)))(*seq)


def ptr(a):
    return ctypes.c_void_p(a.ctypes.data)


def check(status, what):
    if status:
        raise STATUS_EXC.get(status, RuntimeError)("reference %s failed with status %d" % (what, status))


# --- convenience wrappers (numpy in, numpy out) --------------------------------

def add(a, b):
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    out = np.zeros(np.broadcast_shapes(a.shape, b.shape), np.float32)
    check(lib().ref_add(ptr(a), sz(a.shape), a.ndim, ptr(b), sz(b.shape), b.ndim, ptr(out)), "add")
    return out


def view_args(base, off, shape, strides):
    return (ptr(base), base.size, off, sz(shape), sz(strides), len(shape))


def scale(base, off, shape, strides, s):
    out = np.zeros(shape, np.float32)
    check(lib().ref_scale(*view_args(base, off, shape, strides), s, ptr(out)), "scale")
    return out


def copy_(dst, dst_off, dst_shape, dst_strides, src, src_off, src_shape, src_strides):
    check(lib().ref_copy(*view_args(dst, dst_off, dst_shape, dst_strides),
                         *view_args(src, src_off, src_shape, src_strides)), "copy_")


def contiguous(base, off, shape, strides):
    out = np.zeros(shape, np.float32)
    check(lib().ref_contiguous(*view_args(base, off, shape, strides), ptr(out)), "contiguous")
    return out


def rmsnorm(x, gamma, eps=1e-5):
    x = np.ascontiguousarray(x, np.float32)
    cols = x.shape[-1]
    rows = x.size // cols
    out = np.zeros_like(x)
    check(lib().ref_rmsnorm(ptr(x), rows, cols, ptr(np.ascontiguousarray(gamma, np.float32)),
                            eps, ptr(out)), "rmsnorm")
    return out


def swiglu(g, u):
    g = np.ascontiguousarray(g, np.float32)
    u = np.ascontiguousarray(u, np.float32)
    out = np.zeros_like(g)
    check(lib().ref_swiglu(ptr(g), ptr(u), g.size, ptr(out)), "swiglu")
    return out


def softmax(x):
    x = np.ascontiguousarray(x, np.float32)
    cols = x.shape[-1]
    out = np.zeros_like(x)
    check(lib().ref_softmax(ptr(x), x.size // cols, cols, ptr(out)), "softmax")
    return out


def greedy_sample(logits):
    logits = np.ascontiguousarray(logits, np.float32)
    return int(lib().ref_greedy_sample(ptr(logits), logits.size))


def sample_top_p(logits, temperature, top_p, draws):
    """`draws` calls of the reference's sample_top_p (its own random stream)."""
    logits = np.ascontiguousarray(logits, np.float32)
    out = np.zeros(int(draws), np.int32)
    lib().ref_sample_top_p(ptr(logits), logits.size, float(temperature), float(top_p), int(draws), ptr(out))
    return out


def rope(base, off, shape, strides, head_dim, max_seq, theta, pos_offset):
    """Applies the reference RoPE in place on the view of `base`."""
    check(lib().ref_rope(*view_args(base, off, shape, strides), head_dim, max_seq,
                         theta, pos_offset), "rope")


def rope_tables(head_dim, max_seq, theta):
    c = np.zeros((max_seq, head_dim // 2), np.float32)
    s = np.zeros((max_seq, head_dim // 2), np.float32)
    lib().ref_rope_tables(head_dim, max_seq, theta, ptr(c), ptr(s))
    return c, s


def embedding(w_bytes, dtype, dim, vocab, ids):
    ids = np.ascontiguousarray(ids, np.float32)
    out = np.zeros((ids.size, dim), np.float32)
    check(lib().ref_embedding(ptr(w_bytes), dtype, dim, vocab, ptr(ids), ids.size, ptr(out)),
          "embedding")
    return out


def matmul_quant(x, w_bytes, dtype, N):
    x = np.ascontiguousarray(x, np.float32)
    M, K = x.shape
    y = np.zeros((M, N), np.float32)
    check(lib().ref_matmul_quant(ptr(x), M, K, ptr(w_bytes), dtype, N, ptr(y)), "matmul")
    return y


def matmul_f32(a, a_off, a_shape, a_strides, b, b_off, b_shape, b_strides):
    out_shape = list(a_shape[:-1]) + [b_shape[-1]]
    out = np.zeros(out_shape, np.float32)
    check(lib().ref_matmul_f32(ptr(a), a.size, a_off, sz(a_shape), sz(a_strides),
                               ptr(b), b.size, b_off, sz(b_shape), sz(b_strides),
                               len(a_shape), ptr(out)), "matmul_f32")
    return out


def linear_f32(x, w, bias=None):
    x = np.ascontiguousarray(x, np.float32)
    M, K = x.shape
    N = w.shape[1]
    y = np.zeros((M, N), np.float32)
    bp = ptr(np.ascontiguousarray(bias, np.float32)) if bias is not None else None
    check(lib().ref_linear_f32(ptr(x), M, K, ptr(np.ascontiguousarray(w, np.float32)), N, bp,
                               ptr(y)), "linear")
    return y


def dequantize_row_q8_0(blocks_bytes, k):
    y = np.zeros(k, np.float32)
    lib().ref_dequantize_row_q8_0(ptr(blocks_bytes), ptr(y), k)
    return y


def quantize_row_q8_0(x):
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros(x.size // 32 * 34, np.uint8)
    lib().ref_quantize_row_q8_0(ptr(x), ptr(out), x.size)
    return out

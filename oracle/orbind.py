"""ctypes bindings for oracle/liboracle.so, the C restatement of the reference
arithmetic (oracle/turbo_oracle.c).  Test infrastructure only: used by the tests,
`__graft_entry__.smoke()` and bench.py's CPU-baseline leg as the checker.
"""
import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "liboracle.so")
MAX_RANK = 8

_P = ctypes.c_void_p
_SZ = ctypes.c_size_t
_I = ctypes.c_int
_F = ctypes.c_float
_I64P = ctypes.POINTER(ctypes.c_int64)


class View(ctypes.Structure):
    _fields_ = [("base", _P), ("offset", ctypes.c_int64), ("rank", _I),
                ("shape", ctypes.c_int64 * MAX_RANK), ("strides", ctypes.c_int64 * MAX_RANK)]


_VP = ctypes.POINTER(View)

_SIGS = {
    "or_f16_to_f32": (_F, [ctypes.c_uint16]),
    "or_f32_to_f16": (ctypes.c_uint16, [_F]),
    "or_dequant_q8_0": (None, [_P, _SZ, _P]),
    "or_dequant_q4_0": (None, [_P, _SZ, _P]),
    "or_quantize_row_q8_0": (None, [_P, _P, _SZ]),
    "or_vec_dot_q8_0_f32": (_F, [_P, _P, _SZ]),
    "or_vec_dot_q4_0_q8_0": (_F, [_P, _P, _SZ]),
    "or_matmul_q8_0": (None, [_P, _SZ, _SZ, _P, _SZ, _P]),
    "or_matmul_q4_0": (None, [_P, _SZ, _SZ, _P, _SZ, _P]),
    "or_broadcast_shape": (_I, [_I64P, _I, _I64P, _I, _I64P, ctypes.POINTER(_I)]),
    "or_add": (_I, [_VP, _VP, _P, _I64P, ctypes.POINTER(_I)]),
    "or_scale": (None, [_VP, _F, _P]),
    "or_copy": (_I, [_P, _VP, _VP]),
    "or_contiguous": (None, [_VP, _P]),
    "or_rmsnorm": (_I, [_P, _SZ, _SZ, _P, _F, _P]),
    "or_swiglu": (None, [_P, _P, _SZ, _P]),
    "or_softmax": (None, [_P, _SZ, _SZ, _P]),
    "or_argmax": (ctypes.c_int64, [_P, _SZ]),
    "or_sample_top_p": (_I, [_P, _SZ, _F, _F, ctypes.c_double, ctypes.POINTER(_I),
                             ctypes.POINTER(_SZ), ctypes.POINTER(_SZ), ctypes.POINTER(ctypes.c_double)]),
    "or_sample_top_p_set": (_I, [_P, _SZ, _F, _F, ctypes.c_double, ctypes.c_double, ctypes.c_double, _I, _P,
                                 ctypes.POINTER(_I)]),
    "or_rope_tables": (None, [_SZ, _SZ, _F, _P, _P]),
    "or_rope": (_I, [_P, _VP, _SZ, _SZ, _P, _P, _SZ]),
    "or_embedding": (_I, [_P, _I, _SZ, _SZ, _P, _SZ, _P]),
    "or_matmul_f32": (_I, [_VP, _VP, _P]),
}

STATUS_EXC = {1: ValueError, 2: IndexError, 3: RuntimeError}
_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(LIB_PATH + " is not built (make -C oracle oracle)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def ptr(a):
    return ctypes.c_void_p(a.ctypes.data)


def view(base, offset, shape, strides):
    v = View()
    v.base = base.ctypes.data
    v.offset = int(offset)
    v.rank = len(shape)
    for i, (s, st) in enumerate(zip(shape, strides)):
        v.shape[i] = int(s)
        v.strides[i] = int(st)
    return v


def check(status, what):
    if status:
        raise STATUS_EXC.get(status, RuntimeError)("oracle %s failed with status %d" % (what, status))


def f32_to_f16(f):
    return int(lib().or_f32_to_f16(float(f)))


def f16_to_f32(h):
    return float(lib().or_f16_to_f32(int(h)))


def dequant_q8_0(blocks_bytes, nblocks):
    y = np.zeros(nblocks * 32, np.float32)
    lib().or_dequant_q8_0(ptr(blocks_bytes), nblocks, ptr(y))
    return y


def dequant_q4_0(blocks_bytes, nblocks):
    y = np.zeros(nblocks * 32, np.float32)
    lib().or_dequant_q4_0(ptr(blocks_bytes), nblocks, ptr(y))
    return y


def quantize_row_q8_0(x):
    x = np.ascontiguousarray(x, np.float32).ravel()
    out = np.zeros(x.size // 32 * 34, np.uint8)
    lib().or_quantize_row_q8_0(ptr(x), ptr(out), x.size)
    return out


def matmul_q8_0(x, w_bytes, N):
    x = np.ascontiguousarray(x, np.float32)
    M, K = x.shape
    y = np.zeros((M, N), np.float32)
    lib().or_matmul_q8_0(ptr(x), M, K, ptr(w_bytes), N, ptr(y))
    return y


def matmul_q4_0(x, w_bytes, N, threads=1):
    """or_matmul_q4_0; with threads > 1 the rows of x are split over host
    threads (ctypes releases the GIL during each call; rows are independent)."""
    x = np.ascontiguousarray(x, np.float32)
    M, K = x.shape
    y = np.zeros((M, N), np.float32)
    L = lib()
    if threads <= 1 or M < 2:
        L.or_matmul_q4_0(ptr(x), M, K, ptr(w_bytes), N, ptr(y))
        return y
    from concurrent.futures import ThreadPoolExecutor
    cuts = np.linspace(0, M, min(threads, M) + 1).astype(int)

    def part(i):
        a, b = int(cuts[i]), int(cuts[i + 1])
        if b > a:
            L.or_matmul_q4_0(ptr(x[a:b]), b - a, K, ptr(w_bytes), N, ptr(y[a:b]))

    with ThreadPoolExecutor(len(cuts) - 1) as ex:
        list(ex.map(part, range(len(cuts) - 1)))
    return y


def add(a, a_off, a_shape, a_strides, b, b_off, b_shape, b_strides):
    va = view(a, a_off, a_shape, a_strides)
    vb = view(b, b_off, b_shape, b_strides)
    oshape = (ctypes.c_int64 * MAX_RANK)()
    orank = ctypes.c_int()
    n = 1
    try:
        n = int(np.prod(np.broadcast_shapes(tuple(a_shape), tuple(b_shape)))) if a_shape and b_shape else 0
    except ValueError:
        n = 1
    out = np.zeros(max(n, 1), np.float32)
    check(lib().or_add(ctypes.byref(va), ctypes.byref(vb), ptr(out), oshape, ctypes.byref(orank)), "add")
    shape = tuple(oshape[i] for i in range(orank.value))
    return out[:n].reshape(shape)


def scale(x, off, shape, strides, s):
    out = np.zeros(shape, np.float32)
    v = view(x, off, shape, strides)
    lib().or_scale(ctypes.byref(v), s, ptr(out))
    return out


def copy_(dst, dst_off, dst_shape, dst_strides, src, src_off, src_shape, src_strides):
    vd = view(dst, dst_off, dst_shape, dst_strides)
    vs = view(src, src_off, src_shape, src_strides)
    check(lib().or_copy(ptr(dst), ctypes.byref(vd), ctypes.byref(vs)), "copy_")


def contiguous(x, off, shape, strides):
    out = np.zeros(shape, np.float32)
    v = view(x, off, shape, strides)
    lib().or_contiguous(ctypes.byref(v), ptr(out))
    return out


def rmsnorm(x, gamma, eps=1e-5):
    x = np.ascontiguousarray(x, np.float32)
    cols = x.shape[-1]
    out = np.zeros_like(x)
    check(lib().or_rmsnorm(ptr(x), x.size // cols, cols, ptr(np.ascontiguousarray(gamma, np.float32)),
                           eps, ptr(out)), "rmsnorm")
    return out


def swiglu(g, u):
    g = np.ascontiguousarray(g, np.float32)
    u = np.ascontiguousarray(u, np.float32)
    out = np.zeros_like(g)
    lib().or_swiglu(ptr(g), ptr(u), g.size, ptr(out))
    return out


def softmax(x):
    x = np.ascontiguousarray(x, np.float32)
    cols = x.shape[-1]
    out = np.zeros_like(x)
    lib().or_softmax(ptr(x), x.size // cols, cols, ptr(out))
    return out


def argmax(x):
    x = np.ascontiguousarray(x, np.float32)
    return int(lib().or_argmax(ptr(x), x.size))


def sample_top_p(logits, temperature, top_p, u):
    """Nucleus sample with the uniform number `u` given.  Returns (id, nucleus
    length, the reference's fp32-running-sum nucleus length, slack)."""
    x = np.ascontiguousarray(logits, np.float32).ravel()
    tid, nuc, nuc32, slack = _I(), _SZ(), _SZ(), ctypes.c_double()
    st = lib().or_sample_top_p(ptr(x), x.size, float(temperature), float(top_p), float(u), ctypes.byref(tid),
                               ctypes.byref(nuc), ctypes.byref(nuc32), ctypes.byref(slack))
    if st == 1:
        raise ValueError("sample_top_p: bad arguments")
    return tid.value, nuc.value, nuc32.value, (slack.value if st == 0 else 0.0)


def sample_top_p_set(logits, temperature, top_p, u, rel_p, abs_u, accurate_sum=False):
    """Every draw reachable when top_p moves by a factor (1 +- rel_p) and u by
    +- abs_u; accurate_sum takes the softmax denominator as the exact sum."""
    x = np.ascontiguousarray(logits, np.float32).ravel()
    ids = np.zeros(x.size, np.int32)
    n = _I()
    st = lib().or_sample_top_p_set(ptr(x), x.size, float(temperature), float(top_p), float(u), float(rel_p),
                                   float(abs_u), int(bool(accurate_sum)), ptr(ids), ctypes.byref(n))
    if st == 1:
        raise ValueError("sample_top_p: bad arguments")
    return set(int(i) for i in ids[:n.value])


def rope_tables(head_dim, max_seq, theta):
    c = np.zeros((max_seq, head_dim // 2), np.float32)
    s = np.zeros((max_seq, head_dim // 2), np.float32)
    lib().or_rope_tables(head_dim, max_seq, theta, ptr(c), ptr(s))
    return c, s


def rope(base, off, shape, strides, head_dim, max_seq, cos_t, sin_t, pos_offset):
    v = view(base, off, shape, strides)
    check(lib().or_rope(ptr(base), ctypes.byref(v), head_dim, max_seq, ptr(cos_t), ptr(sin_t),
                        pos_offset), "rope")


def embedding(w_bytes, dtype, dim, vocab, ids):
    ids = np.ascontiguousarray(ids, np.float32)
    out = np.zeros((ids.size, dim), np.float32)
    check(lib().or_embedding(ptr(w_bytes), dtype, dim, vocab, ptr(ids), ids.size, ptr(out)),
          "embedding")
    return out


def matmul_f32(a, a_off, a_shape, a_strides, b, b_off, b_shape, b_strides):
    out = np.zeros(list(a_shape[:-1]) + [b_shape[-1]], np.float32)
    va = view(a, a_off, a_shape, a_strides)
    vb = view(b, b_off, b_shape, b_strides)
    check(lib().or_matmul_f32(ctypes.byref(va), ctypes.byref(vb), ptr(out)), "matmul_f32")
    return out

"""Python binding of libturbo_b200.so, the C ABI in include/turbo_b200.h.

Used by the tests and bench.py to drive the CUDA kernels through exactly the
entry points a C/C++ caller uses.  Device memory comes from PyTorch tensors
(plumbing only); every computation is a kernel of the library.  There is no
fallback: if the library is missing or the device is not an sm_100 part, the
calls raise.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
PKG_ROOT = os.path.dirname(os.path.dirname(_HERE))  # turbo.cpp_b200/
LIB_PATH = os.path.join(PKG_ROOT, "libturbo_b200.so")
HEADER = os.path.join(os.path.dirname(PKG_ROOT), "include", "turbo_b200.h")

MAX_RANK = 8
F32, F16, Q8_0, Q4_0, I32, BF16 = 0, 1, 2, 3, 4, 5
OK, EINVAL, ERANGE, ERUNTIME, ECUDA, ETIMEOUT, ENOMEM = range(7)


class TbError(RuntimeError):
    def __init__(self, status, msg):
        super().__init__("%s: %s" % (STATUS_NAMES.get(status, status), msg))
        self.status = status


STATUS_NAMES = {0: "TB_OK", 1: "TB_EINVAL", 2: "TB_ERANGE", 3: "TB_ERUNTIME", 4: "TB_ECUDA",
                5: "TB_ETIMEOUT", 6: "TB_ENOMEM"}


class View(ctypes.Structure):
    """tb_view: data, dtype, rank, offset, shape[8], strides[8] (elements)."""
    _fields_ = [("data", ctypes.c_void_p), ("dtype", ctypes.c_int32), ("rank", ctypes.c_int32),
                ("offset", ctypes.c_int64), ("shape", ctypes.c_int64 * MAX_RANK),
                ("strides", ctypes.c_int64 * MAX_RANK)]


_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_F = ctypes.c_float
_SZ = ctypes.c_size_t
_VP = ctypes.POINTER(View)

SIGNATURES = {
    "tb_init": [_I],
    "tb_last_error": None,
    "tb_status_name": [_I],
    "tb_version": [],
    "tb_alloc": [ctypes.POINTER(_P), _SZ],
    "tb_free": [_P],
    "tb_upload": [_P, _P, _SZ, _P],
    "tb_download": [_P, _P, _SZ, _P],
    "tb_memset": [_P, _I, _SZ, _P],
    "tb_sync": [_P],
    "tb_take_device_errors": [ctypes.POINTER(ctypes.c_uint32)],
    "tb_set_wait_limit_ns": [ctypes.c_uint64],
    "tb_binary": [_I, _VP, _VP, _VP, _P],
    "tb_scale": [_VP, _F, _VP, _P],
    "tb_copy": [_VP, _VP, _P],
    "tb_rmsnorm": [_I, _P, _P, _P, _I64, _I64, _F, _P],
    "tb_swiglu": [_I, _P, _P, _P, _I64, _P],
    "tb_softmax": [_P, _P, _I64, _I64, _P],
    "tb_argmax": [_P, _I64, _I64, _P, _P],
    "tb_sample_top_p": [_P, _I64, _F, _F, ctypes.c_double, _P, _P],
    "tb_sample_top_p_at": [_P, _I64, _F, _F, _P, _P, _I64, _P, _P],
    "tb_rope": [_VP, _P, _P, _I64, _I64, _I64, _P],
    "tb_fill_upper": [_P, _I64, _I64, _I64, _I64, _F, _P],
    "tb_dequant": [_I, _P, _I64, _P, _P],
    "tb_quantize_q8_0": [_P, _I64, _I64, _P, _P],
    "tb_embedding": [_I, _P, _I64, _I64, _P, _I64, _P, _P],
    "tb_matmul_quant": [_I, _P, _I64, _I64, _P, _I64, _P, _P],
    "tb_matmul_quant_exact": [_I, _P, _I64, _I64, _P, _I64, _P, _P],
    "tb_matmul_q4_0_static_scratch": [_P, _I64, _I64, _P, _I64, _P, _P],
    "tb_packed_quant_weights_bytes": [_I, _I64, _I64, _P],
    "tb_pack_quant_weights": [_I, _P, _I64, _I64, _P, _SZ, _P],
    "tb_matmul_quant_packed": [_I, _P, _I64, _I64, _P, _I64, _P, _P],
    "tb_matmul_f32": [_VP, _VP, _VP, _P],
    "tb_softmax_shard_stats": [_P, _I64, _I64, _I64, _P, _P, _P],
    "tb_softmax_shard_rescale": [_P, _P, _P, _I64, _P],
    "tb_softmax_shard_finish": [_P, _I64, _I64, _I64, _P, _P, _P, _I64, _P],
    "tb_argmax_shard_keys": [_P, _I64, _I64, _I64, _I64, _P, _P],
    "tb_argmax_key_index": [_P, _I64, _P, _P],
    "tb_shard_group_unique_id": [_P],
    "tb_shard_group_create": [_I, _I, _P, _I64, ctypes.c_double, ctypes.POINTER(_P)],
    "tb_shard_group_wait": [_P, _P, ctypes.c_double],
    "tb_shard_group_abort": [_P],
    "tb_shard_group_destroy": [_P],
    "tb_softmax_vocab_sharded": [_P, _P, _I64, _I64, _I64, _P, _I64, _P],
    "tb_argmax_vocab_sharded": [_P, _P, _I64, _I64, _I64, _I64, _P, _P],
    "tb_shard_group_enable_peer": [_P, _I64],
    "tb_gemv_q8_0_row_sharded": [_P, _P, _I64, _P, _I64, _P, _P],
    "tb_decode_workspace_bytes": [_P, ctypes.POINTER(_SZ)],
    "tb_attention_prefill": [_P, _I64, _P, _P, _I64, _I64, _I64, _I64, _I64, _F, _P, _I64, _P],
    "tb_decode_step_persistent": [_P, _P],
    "tb_rope_at": [_VP, _P, _P, _I64, _I64, _P, _P],
    "tb_kv_append": [_P, _P, _P, _P, _I64, _I64, _P, _P],
    "tb_attention_decode": [_P, _P, _P, _I64, _I64, _I64, _I64, _F, _P, _P, _P],
    "tb_decode_margin": [_P, _I64, _P, _P, _I64, _P, _P],
    "tb_decode_advance": [_P, _P, _P, _P, _I64, _P],
    "tb_stream_create": [ctypes.POINTER(_P)],
    "tb_stream_destroy": [_P],
    "tb_capture_begin": [_P],
    "tb_capture_end": [_P, ctypes.POINTER(_P)],
    "tb_graph_launch": [_P, _P],
    "tb_graph_destroy": [_P],
    "tb_gemv_q8_0_multi": [_P, _I64, _P, _F, _P, _I, _P],
    "tb_gemv_q8_0_swiglu": [_P, _I64, _P, _F, _P, _P, _I64, _P, _P],
    "tb_rope_kv_append": [_P, _P, _P, _I64, _I64, _I64, _P, _P, _I64, _P, _P, _I64, _P, _P],
    "tb_prefetch_l2": [_P, _P, _I, _P],
    "tb_rope_attention_decode": [_P, _P, _P, _I64, _I64, _I64, _P, _P, _I64, _P, _P, _I64, _F, _P, _P, _P],
}


class GemvSegment(ctypes.Structure):
    """tb_gemv_segment: w, n, y, residual."""
    _fields_ = [("w", ctypes.c_void_p), ("n", ctypes.c_int64), ("y", ctypes.c_void_p), ("residual", ctypes.c_void_p)]

_lib = None


def load():
    """Loads the library (raises if it is not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError("libturbo_b200.so is not built: run __graft_entry__.build() or "
                              "python turbo.cpp_b200/build.py")
        L = ctypes.CDLL(LIB_PATH)
        for name, args in SIGNATURES.items():
            fn = getattr(L, name)
            if name in ("tb_last_error", "tb_status_name", "tb_version"):
                fn.restype = ctypes.c_char_p
                fn.argtypes = [] if args is None else args
            else:
                fn.restype = ctypes.c_int
                fn.argtypes = args
        _lib = L
    return _lib


def lib():
    return load()


def check(status, what=""):
    if status != OK:
        msg = load().tb_last_error().decode(errors="replace")
        raise TbError(status, (what + ": " if what else "") + msg)


def call(name, *args):
    check(getattr(load(), name)(*args), name)


# ---- torch helpers -----------------------------------------------------------

def stream_handle(stream=None):
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def dtype_code(t):
    import torch
    return {torch.float32: F32, torch.float16: F16, torch.int32: I32, torch.bfloat16: BF16}[t.dtype]


def view(base, offset=None, shape=None, strides=None, dtype=None):
    """A tb_view over a torch tensor.  With explicit offset/shape/strides the
    view addresses `base`'s storage from its first element (the reference's
    Tensor{storage, offset, shape, strides}); otherwise it describes `base`."""
    v = View()
    if offset is None:
        v.data = base.data_ptr()
        v.offset = 0
        shape = list(base.shape)
        strides = list(base.stride())
    else:
        v.data = base.data_ptr()
        v.offset = int(offset)
    v.dtype = dtype if dtype is not None else dtype_code(base)
    v.rank = len(shape)
    for i, (s, st) in enumerate(zip(shape, strides)):
        v.shape[i] = int(s)
        v.strides[i] = int(st)
    return v


def byref(v):
    return ctypes.byref(v)


def take_device_errors():
    flags = ctypes.c_uint32(0)
    call("tb_take_device_errors", ctypes.byref(flags))
    return flags.value

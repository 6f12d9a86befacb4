"""ctypes binding of libturbo_b200_host.so's model interface (tbm_*): the C++
MiniGPT over the device Tensor, driven like the reference's generate loop."""
import ctypes
import os

import numpy as np

from . import PKG_ROOT

HOST_LIB = os.path.join(PKG_ROOT, "libturbo_b200_host.so")
_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(HOST_LIB):
            raise ImportError("libturbo_b200_host.so is not built (python turbo.cpp_b200/build.py)")
        L = ctypes.CDLL(HOST_LIB)
        L.tbm_last_error.restype = ctypes.c_char_p
        L.tbm_model_load.restype = ctypes.c_void_p
        L.tbm_model_load.argtypes = [ctypes.c_char_p, ctypes.c_int]
        L.tbm_model_free.argtypes = [ctypes.c_void_p]
        L.tbm_set_persistent_decode.argtypes = [ctypes.c_int]
        L.tbm_set_persistent_decode.restype = None
        L.tbm_model_generate.restype = ctypes.c_int
        L.tbm_model_generate.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t,
                                         ctypes.c_size_t, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                         ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double)]
        L.tbm_model_generate_sampled.restype = ctypes.c_int
        L.tbm_model_generate_sampled.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t,
                                                 ctypes.c_size_t, ctypes.c_float, ctypes.c_float, ctypes.c_void_p,
                                                 ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(ctypes.c_double),
                                                 ctypes.POINTER(ctypes.c_double)]
        _lib = L
    return _lib


class Model:
    def __init__(self, path, exact=True, persistent=False):
        """exact: the bit-identical matmul kernels and the op-by-op step;
        otherwise one CUDA graph per token, whose step is a single persistent
        kernel when `persistent` and the model's shapes allow it, else the
        fused per-op kernels."""
        self.h = lib().tbm_model_load(path.encode(), 1 if exact else 0)
        if not self.h:
            raise RuntimeError("tbm_model_load: " + lib().tbm_last_error().decode())
        self.persistent = persistent

    def generate(self, prompt, steps, max_seq=1024, want_margins=True, want_logits=False, vocab=128256,
                 temperature=0.0, top_p=0.9, uniforms=None):
        """Prefill, then `steps` tokens: greedy, or with temperature > 0 nucleus
        sampled (the reference's generate loop), token s drawn with
        uniforms[s] in [0, 1) (steps + 1 numbers; drawn here when not given)."""
        prompt = np.ascontiguousarray(prompt, np.int32)
        ids = np.zeros(steps + 1, np.int32)
        margins = np.zeros(steps + 1, np.float32) if want_margins else None
        logits = np.zeros(vocab, np.float32) if want_logits else None
        pre, dec = ctypes.c_double(), ctypes.c_double()
        lib().tbm_set_persistent_decode(1 if self.persistent else 0)
        if temperature > 0:
            if want_logits:
                raise ValueError("want_logits is for greedy runs")
            if uniforms is None:
                uniforms = np.random.default_rng().random(steps + 1)
            uniforms = np.ascontiguousarray(uniforms, np.float64)
            if uniforms.size != steps + 1:
                raise ValueError("need steps + 1 uniform numbers")
            st = lib().tbm_model_generate_sampled(self.h, prompt.ctypes.data, prompt.size, steps, max_seq,
                                                  float(temperature), float(top_p), uniforms.ctypes.data,
                                                  ids.ctypes.data, margins.ctypes.data if margins is not None else None,
                                                  ctypes.byref(pre), ctypes.byref(dec))
        else:
            st = lib().tbm_model_generate(self.h, prompt.ctypes.data, prompt.size, steps, max_seq, ids.ctypes.data,
                                          margins.ctypes.data if margins is not None else None,
                                          logits.ctypes.data if logits is not None else None,
                                          ctypes.byref(pre), ctypes.byref(dec))
        if st:
            raise RuntimeError("tbm_model_generate: " + lib().tbm_last_error().decode())
        return dict(ids=ids, margins=margins, logits=logits, prefill_ms=pre.value, decode_ms=dec.value)

    def close(self):
        if self.h:
            lib().tbm_model_free(self.h)
            self.h = None

    def __del__(self):
        self.close()

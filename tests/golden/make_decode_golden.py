#!/usr/bin/env python3
"""Generates tests/golden/decode_1b.npz: the REFERENCE MiniGPT's greedy decode
of the Llama-3.2-1B-shaped synthetic Q8_0 model (turbo_b200.gguf_synth, seed 0):
prefill of 512 seeded token ids, then 128 greedy steps, with each step's chosen
id and its top-1 minus top-2 logit margin, plus the final step's logits.

Needs oracle/_ref/libturbo_ref.so (the reference compiled from its sources).
Takes a few minutes on 8 cores.  Usage: make_decode_golden.py [model.gguf]
"""
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "turbo.cpp_b200", "python"))

import ctypes  # noqa: E402

from oracle import refbind as R  # noqa: E402
from turbo_b200 import gguf_synth  # noqa: E402

STEPS = 128
MAX_SEQ = 1024


def main():
    path = sys.argv[1] if len(sys.argv) > 1 else gguf_synth.default_model_path()
    if not os.path.exists(path):
        t0 = time.time()
        gguf_synth.write_model(path)
        print("wrote %s (%.1f s, %d bytes)" % (path, time.time() - t0, os.path.getsize(path)))
    prompt = gguf_synth.prompt_ids(512)
    h = R.lib().ref_model_load(path.encode())
    assert h, "reference failed to load the model"
    ids = np.zeros(STEPS + 1, np.int32)
    margins = np.zeros(STEPS + 1, np.float32)
    logits = np.zeros(gguf_synth.LLAMA_1B["vocab"], np.float32)
    pre = ctypes.c_double()
    dec = ctypes.c_double()
    st = R.lib().ref_model_generate(h, R.ptr(prompt), prompt.size, STEPS, MAX_SEQ, R.ptr(ids), R.ptr(margins),
                                    R.ptr(logits), ctypes.byref(pre), ctypes.byref(dec))
    R.check(st, "generate")
    R.lib().ref_model_free(h)
    print("prefill %.1f s, decode %.1f s (%.2f tok/s)" % (pre.value / 1e3, dec.value / 1e3, STEPS / (dec.value / 1e3)))
    print("ids", ids[:16], "... min margin %.4g" % margins.min())
    np.savez_compressed(os.path.join(HERE, "decode_1b.npz"), prompt=prompt, ids=ids, margins=margins,
                        last_logits=logits, steps=STEPS, max_seq=MAX_SEQ, seed=0,
                        prefill_ms=pre.value, decode_ms=dec.value, threads=os.cpu_count())


if __name__ == "__main__":
    main()

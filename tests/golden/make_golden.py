#!/usr/bin/env python3
"""Generates tests/golden/*.npz: inputs and the REFERENCE library's outputs.

Run in a container where the reference sources were compiled into
oracle/_ref/libturbo_ref.so (make -C oracle ref).  Each fixture stores its
inputs next to the reference outputs, so the tests need neither the reference
nor the random generator to check the oracle and the CUDA path against it.

Cases: the known-answer tests of the reference's gtest suite
(tests/test_tensor.cpp, test_nn.cpp, test_rope.cpp, test_quant.cpp) and seeded
small instances of every hot-path op at the shapes of the benchmark configs.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "turbo.cpp_b200", "python"))

from oracle import refbind as R  # noqa: E402
from turbo_b200 import synth  # noqa: E402


def save(name, **arrays):
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **arrays)


def main():
    # --- known answers of the reference suite ---------------------------------
    sm_in = np.array([[1, 2, 3], [10, 100, 10]], np.float32)  # test_tensor.cpp:17
    rms_in = np.array([[1, 2, 3, 4]], np.float32)  # test_nn.cpp:143-154
    rms_g = np.array([0.5, 1.0, 1.5, 2.0], np.float32)
    rope_in = np.array([[1, 2, 3, 4], [1, 2, 3, 4]], np.float32)  # test_rope.cpp:12-15
    rope_out = rope_in.copy()
    R.rope(rope_out, 0, (2, 4), (4, 1), 4, 10, 10000.0, 0)
    lin_w = np.array([[1, 2], [3, 4], [5, 6]], np.float32)  # test_nn.cpp:16-24
    lin_b = np.array([0.5, -0.5], np.float32)
    lin_x = np.array([[1, 1, 1], [2, 0, 1]], np.float32)
    q8_blk = np.zeros(34, np.uint8)  # test_quant.cpp:9-19: d = 0.5, q = +-2, x = 1
    q8_blk[:2] = np.frombuffer(np.float16(0.5).tobytes(), np.uint8)
    q8_blk[2:] = np.array([2 if i % 2 == 0 else -2 for i in range(32)], np.int8).view(np.uint8)
    q4_blk = np.zeros(18, np.uint8)  # test_quant.cpp:36-55: d = 0.5, byte 0x6A
    q4_blk[:2] = np.frombuffer(np.float16(0.5).tobytes(), np.uint8)
    q4_blk[2:] = 0x6A
    x8_blk = np.zeros(34, np.uint8)
    x8_blk[:2] = np.frombuffer(np.float16(1.0).tobytes(), np.uint8)
    x8_blk[2:] = 1
    ones = np.ones(32, np.float32)
    save("kat",
         softmax_in=sm_in, softmax_out=R.softmax(sm_in),
         rmsnorm_in=rms_in, rmsnorm_gamma=rms_g, rmsnorm_out=R.rmsnorm(rms_in, rms_g),
         rope_in=rope_in, rope_out=rope_out,
         linear_w=lin_w, linear_b=lin_b, linear_x=lin_x, linear_out=R.linear_f32(lin_x, lin_w, lin_b),
         q8_block=q8_blk, q8_dot=np.float32(R.lib().ref_vec_dot_q8_0_f32(32, R.ptr(q8_blk), R.ptr(ones))),
         q4_block=q4_blk, x8_block=x8_blk,
         q4_dot=np.float32(R.lib().ref_vec_dot_q4_0_q8_0(32, R.ptr(q4_blk), R.ptr(x8_blk))),
         q4_dot_avx2=np.float32(R.lib().ref_vec_dot_q4_0_q8_0_avx2(32, R.ptr(q4_blk), R.ptr(x8_blk))))

    # --- quantized matmul / dequant / quantize ------------------------------------
    w8 = synth.quantize_q8_0(synth.normal((64, 2048), 0.02, seed=1))
    x8 = synth.normal((2, 2048), 1.0, seed=2)
    w4 = synth.quantize_q4_0(synth.normal((32, 1024), 0.02, seed=3))
    x4 = synth.normal((3, 1024), 1.0, seed=4)
    xq_in = synth.normal((4, 256), 1.0, seed=5)
    xq_in[0, :32] = 0
    save("quant",
         w8=w8, x8=x8, y8=R.matmul_quant(x8, w8, R.DT_Q8_0, 64),
         w4=w4, x4=x4, y4=R.matmul_quant(x4, w4, R.DT_Q4_0, 32),
         deq8=np.stack([R.dequantize_row_q8_0(w8[r], 2048) for r in range(4)]),
         xq_in=xq_in, xq_out=np.stack([R.quantize_row_q8_0(xq_in[r]) for r in range(4)]))

    # --- elementwise, rows, views -------------------------------------------------
    a = synth.normal((4, 1, 8), 1.0, seed=6)
    b = synth.normal((3, 1), 1.0, seed=7)
    h = synth.normal((4, 2048), 1.0, seed=8)
    g = synth.uniform((2048,), 0.5, 1.5, seed=9)
    gate = synth.normal((4096,), 1.0, seed=10)
    up = synth.normal((4096,), 1.0, seed=11)
    logits = synth.normal((2, 1000), 2.0, seed=12)
    amax_rows = synth.normal((3, 5000), 2.0, seed=13)
    amax_rows[1, 17] = amax_rows[1, 4000] = 99.0
    base = synth.normal((4 * 6 * 5 + 3,), 1.0, seed=14)
    save("elementwise",
         add_a=a, add_b=b, add_out=R.add(a, b),
         rms_x=h, rms_g=g, rms_out=R.rmsnorm(h, g),
         swiglu_g=gate, swiglu_u=up, swiglu_out=R.swiglu(gate, up),
         softmax_x=logits, softmax_out=R.softmax(logits),
         argmax_x=amax_rows, argmax_out=np.array([R.greedy_sample(r) for r in amax_rows], np.int64),
         view_base=base, view_off=np.int64(3), view_shape=np.array([5, 4, 6]), view_strides=np.array([1, 30, 5]),
         scale_out=R.scale(base, 3, (5, 4, 6), (1, 30, 5), 0.125),
         contiguous_out=R.contiguous(base, 3, (5, 4, 6), (1, 30, 5)))

    # --- RoPE 4-D view, embedding, fp32 attention products ------------------------
    hd, S, H = 64, 5, 8
    q = synth.normal((S * H * hd,), 1.0, seed=15)
    q_out = q.copy()
    R.rope(q_out, 0, (1, H, S, hd), (S * H * hd, hd, H * hd, 1), hd, 64, 500000.0, 11)
    cos_t, sin_t = R.rope_tables(hd, 64, 500000.0)
    emb_w = synth.quantize_q8_0(synth.normal((100, 256), 0.02, seed=16)).ravel()
    ids = np.array([3, 99, 0, 3], np.float32)
    qa = synth.normal((1 * 2048 + 64,), 1.0, seed=17)
    kb = synth.normal((40 * 512 + 64,), 1.0, seed=18)
    save("rope_embed_attn",
         rope_x=q, rope_out=q_out, rope_cos=cos_t, rope_sin=sin_t,
         emb_w=emb_w, emb_ids=ids, emb_out=R.embedding(emb_w, R.DT_Q8_0, 256, 100, ids),
         mm_a=qa, mm_b=kb,
         mm_out=R.matmul_f32(qa, 3, (1, 64), (2048, 1), kb, 5, (64, 40), (1, 512)))
    print("wrote", sorted(f for f in os.listdir(HERE) if f.endswith(".npz")))


if __name__ == "__main__":
    main()

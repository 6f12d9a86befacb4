"""Golden vectors: the reference library's own outputs (tests/golden/*.npz,
written by tests/golden/make_golden.py) against the oracle on CPU and the CUDA
path on the GPU.  The known-answer values of the reference's gtest suite are
asserted as the reference asserts them."""
import os

import numpy as np
import pytest

from oracle import orbind as O

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return np.load(os.path.join(HERE, name + ".npz"))


def same_bits(a, b):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


# ------------------------------------------------------------------ CPU -----

def test_reference_kats_hold():
    k = load("kat")
    np.testing.assert_allclose(k["softmax_out"].ravel(), [0.0900, 0.2447, 0.6652, 0, 1, 0], atol=1e-4)
    np.testing.assert_allclose(k["rmsnorm_out"][0], [0.182574, 0.730296, 1.643167, 2.921186], atol=1e-4)
    assert abs(k["rope_out"][1, 0] - -1.9840) < 1e-3 and abs(k["rope_out"][1, 2] - 2.4623) < 1e-3
    np.testing.assert_array_equal(k["rope_out"][0], [1, 2, 3, 4])
    np.testing.assert_array_equal(k["linear_out"], [[9.5, 11.5], [7.5, 9.5]])
    assert abs(float(k["q8_dot"])) < 1e-5 and abs(float(k["q4_dot"])) < 1e-5


def test_oracle_matches_golden_kats():
    k = load("kat")
    assert same_bits(O.softmax(k["softmax_in"]), k["softmax_out"])
    assert same_bits(O.rmsnorm(k["rmsnorm_in"], k["rmsnorm_gamma"]), k["rmsnorm_out"])
    c, s = O.rope_tables(4, 10, 10000.0)
    x = k["rope_in"].copy()
    O.rope(x, 0, (2, 4), (4, 1), 4, 10, c, s, 0)
    assert same_bits(x, k["rope_out"])
    w = k["linear_w"]
    y = O.matmul_f32(k["linear_x"], 0, (2, 3), (3, 1), w, 0, (3, 2), (2, 1)) + k["linear_b"]
    assert same_bits(y, k["linear_out"])
    q4 = k["q4_block"]
    x8 = k["x8_block"]
    assert np.float32(O.lib().or_vec_dot_q4_0_q8_0(O.ptr(q4), O.ptr(x8), 32)) == k["q4_dot_avx2"]


def test_oracle_matches_golden_quant():
    g = load("quant")
    assert same_bits(O.matmul_q8_0(g["x8"], g["w8"], 64), g["y8"])
    assert same_bits(O.matmul_q4_0(g["x4"], g["w4"], 32), g["y4"])
    for r in range(4):
        assert same_bits(O.dequant_q8_0(g["w8"][r], 64), g["deq8"][r])
        assert np.array_equal(O.quantize_row_q8_0(g["xq_in"][r]), g["xq_out"][r])


def test_oracle_matches_golden_elementwise():
    g = load("elementwise")
    a, b = g["add_a"], g["add_b"]
    assert same_bits(O.add(a, 0, a.shape, (8, 8, 1), b, 0, b.shape, (1, 1)), g["add_out"])
    assert same_bits(O.rmsnorm(g["rms_x"], g["rms_g"]), g["rms_out"])
    assert same_bits(O.swiglu(g["swiglu_g"], g["swiglu_u"]), g["swiglu_out"])
    assert same_bits(O.softmax(g["softmax_x"]), g["softmax_out"])
    assert [O.argmax(r) for r in g["argmax_x"]] == list(g["argmax_out"])
    base, off = g["view_base"], int(g["view_off"])
    shape, strides = tuple(g["view_shape"]), tuple(g["view_strides"])
    assert same_bits(O.scale(base, off, shape, strides, 0.125), g["scale_out"])
    assert same_bits(O.contiguous(base, off, shape, strides), g["contiguous_out"])


def test_oracle_matches_golden_rope_embed_attn():
    g = load("rope_embed_attn")
    c, s = O.rope_tables(64, 64, 500000.0)
    assert same_bits(c, g["rope_cos"]) and same_bits(s, g["rope_sin"])
    x = g["rope_x"].copy()
    O.rope(x, 0, (1, 8, 5, 64), (5 * 8 * 64, 64, 8 * 64, 1), 64, 64, c, s, 11)
    assert same_bits(x, g["rope_out"])
    assert same_bits(O.embedding(g["emb_w"], 2, 256, 100, g["emb_ids"]), g["emb_out"])
    assert same_bits(O.matmul_f32(g["mm_a"], 3, (1, 64), (2048, 1), g["mm_b"], 5, (64, 40), (1, 512)),
                     g["mm_out"])


# ------------------------------------------------------------------ GPU -----

@pytest.mark.gpu
def test_cuda_matches_golden():
    import torch

    import turbo_b200 as T
    T.call("tb_init", 0)
    s = T.stream_handle()

    keep = []  # inputs stay alive until the kernels that read them have run

    def dev(a):
        t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
        keep.append(t)
        return t

    q = load("quant")
    for dt, x, w, y, N in ((T.Q8_0, q["x8"], q["w8"], q["y8"], 64), (T.Q4_0, q["x4"], q["w4"], q["y4"], 32)):
        out = torch.empty(y.shape, dtype=torch.float32, device="cuda")
        T.call("tb_matmul_quant_exact", dt, T.ptr(dev(x)), x.shape[0], x.shape[1], T.ptr(dev(w)), N, T.ptr(out), s)
        torch.cuda.synchronize()
        assert same_bits(out.cpu().numpy(), y)
    xq = torch.empty(q["xq_out"].size, dtype=torch.uint8, device="cuda")
    T.call("tb_quantize_q8_0", T.ptr(dev(q["xq_in"])), 4, 256, T.ptr(xq), s)
    torch.cuda.synchronize()
    assert np.array_equal(xq.cpu().numpy().reshape(4, -1), q["xq_out"])

    g = load("elementwise")
    out = torch.empty(g["argmax_x"].shape[0], dtype=torch.int64, device="cuda")
    T.call("tb_argmax", T.ptr(dev(g["argmax_x"])), 3, 5000, T.ptr(out), s)
    torch.cuda.synchronize()
    assert list(out.cpu().numpy()) == list(g["argmax_out"])
    base = dev(g["view_base"])
    o = torch.empty((5, 4, 6), dtype=torch.float32, device="cuda")
    T.call("tb_copy", T.byref(T.view(o)), T.byref(T.view(base, 3, (5, 4, 6), (1, 30, 5))), s)
    torch.cuda.synchronize()
    assert same_bits(o.cpu().numpy(), g["contiguous_out"])

    r = load("rope_embed_attn")
    x = dev(r["rope_x"])
    T.call("tb_rope", T.byref(T.view(x, 0, (1, 8, 5, 64), (5 * 8 * 64, 64, 8 * 64, 1))),
           T.ptr(dev(r["rope_cos"])), T.ptr(dev(r["rope_sin"])), 64, 64, 11, s)
    e = torch.empty((4, 256), dtype=torch.float32, device="cuda")
    T.call("tb_embedding", T.Q8_0, T.ptr(dev(r["emb_w"])), 256, 100,
           T.ptr(dev(r["emb_ids"].astype(np.int32))), 4, T.ptr(e), s)
    torch.cuda.synchronize()
    assert same_bits(x.cpu().numpy(), r["rope_out"])
    assert same_bits(e.cpu().numpy(), r["emb_out"])

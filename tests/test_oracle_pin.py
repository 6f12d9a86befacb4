"""Pins the C restatement (oracle/turbo_oracle.c) to the reference library itself.

The reference Turbo.cpp library is compiled from its own sources into
oracle/_ref/libturbo_ref.so (oracle/Makefile).  Every restated function must
agree with it BIT FOR BIT on seeded inputs, including the edge cases the
reference code reaches (ties, NaN, -inf, broadcast, strided views, tails).
"""
import numpy as np
import pytest

from oracle import orbind as O
from oracle import refbind as R
from turbo_b200 import synth

pytestmark = pytest.mark.skipif(not R.available(), reason="reference library not built")

f32 = np.float32


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def assert_bits(a, b):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    assert a.shape == b.shape
    nan_a, nan_b = np.isnan(a), np.isnan(b)
    assert np.array_equal(nan_a, nan_b)
    diff = (bits(a) != bits(b)) & ~nan_a
    assert not diff.any(), "%d mismatches, first at %s" % (diff.sum(), np.argwhere(diff)[0])


def test_f16_roundtrip_all_halves():
    for h in range(0, 65536, 1):
        o = O.f16_to_f32(h)
        r = float(R.lib().ref_f16_to_f32(h))
        assert (np.isnan(o) and np.isnan(r)) or np.float32(o).view(np.uint32) == np.float32(r).view(np.uint32), h


def test_f32_to_f16_rne_matches_f16c():
    rng = np.random.default_rng(5)
    vals = list(rng.integers(0, 2**32, 20000, dtype=np.uint64).astype(np.uint32).view(np.float32))
    vals += [0.0, -0.0, 65504.0, 65519.99, 65520.0, 1e-8, 2**-25, 2**-24, 3 * 2**-26, 6.1e-5,
             np.inf, -np.inf, 1.0 + 2**-11, 1.0 + 3 * 2**-11]
    for v in vals:
        v = np.float32(v)
        o = O.f32_to_f16(v)
        r = int(R.lib().ref_f32_to_f16(v))
        if np.isnan(v):
            assert (o & 0x7C00) == 0x7C00 and (o & 0x3FF) and (r & 0x3FF)
        else:
            assert o == r, (v, hex(o), hex(r))


def test_quantize_row_q8_0_matches_reference_and_synth():
    x = synth.normal((64, 2048), 1.0, seed=3)
    x[0, :32] = 0.0  # all-zero block: d = 0, id = 0
    x[1, :32] = np.linspace(-3, 3, 32)  # exact .5 multiples after scaling
    for r in range(x.shape[0]):
        ref = R.quantize_row_q8_0(x[r])
        assert np.array_equal(O.quantize_row_q8_0(x[r]), ref)
        assert np.array_equal(synth.quantize_q8_0(x[r]), ref)


def test_dequant_q8_0_bit_exact():
    w = synth.quantize_q8_0(synth.normal((16, 2048), 0.02, seed=4))
    for r in range(w.shape[0]):
        ref = R.dequantize_row_q8_0(w[r], 2048)
        assert_bits(O.dequant_q8_0(w[r], 64), ref)
        assert_bits(synth.dequantize_q8_0(w[r], 2048), ref)


def test_matmul_q8_0_bit_exact():
    N, K, M = 512, 2048, 3
    wq = synth.quantize_q8_0(synth.normal((N, K), 0.02, seed=7))
    x = synth.normal((M, K), 1.0, seed=8)
    assert_bits(O.matmul_q8_0(x, wq, N), R.matmul_quant(x, wq, R.DT_Q8_0, N))


def test_matmul_q4_0_bit_exact():
    N, K, M = 256, 8192, 3
    wq = synth.quantize_q4_0(synth.normal((N, K), 0.02, seed=9))
    x = synth.normal((M, K), 1.0, seed=10)
    assert_bits(O.matmul_q4_0(x, wq, N), R.matmul_quant(x, wq, R.DT_Q4_0, N))


def test_q4_0_dot_kats_agree():
    # the scalar and AVX2 reference dots agree on exact small cases
    w = synth.quantize_q4_0(synth.normal((1, 64), 1.0, seed=11))
    xq = synth.quantize_q8_0(synth.normal((1, 64), 1.0, seed=12))
    a = R.lib().ref_vec_dot_q4_0_q8_0_avx2(64, R.ptr(w), R.ptr(xq))
    o = O.lib().or_vec_dot_q4_0_q8_0(O.ptr(w), O.ptr(xq), 64)
    assert np.float32(a) == np.float32(o)


@pytest.mark.parametrize("sa,sb", [((1, 128, 2048), (1, 128, 2048)), ((4, 1, 8), (3, 1)),
                                   ((2, 3, 4), (4,)), ((5,), (2, 1, 5)), ((7, 1), (1, 9))])
def test_add_broadcast(sa, sb):
    a = synth.normal(sa, 1.0, seed=1)
    b = synth.normal(sb, 1.0, seed=2)
    ref = R.add(a, b)
    ca = np.ascontiguousarray(a)
    cb = np.ascontiguousarray(b)
    out = O.add(ca, 0, sa, [s // 4 for s in ca.strides], cb, 0, sb, [s // 4 for s in cb.strides])
    assert_bits(out, ref)


def test_add_not_broadcastable_raises_invalid_argument():
    a = synth.normal((3, 4), 1.0, seed=1)
    b = synth.normal((5,), 1.0, seed=2)
    with pytest.raises(ValueError):
        R.add(a, b)
    with pytest.raises(ValueError):
        O.add(a, 0, (3, 4), (4, 1), b, 0, (5,), (1,))


def test_strided_views_scale_copy_contiguous():
    base = synth.normal((4 * 6 * 5 + 3,), 1.0, seed=13)
    shape, strides, off = (5, 4, 6), (1, 30, 5), 3  # a transposed view
    assert_bits(O.scale(base, off, shape, strides, 0.125), R.scale(base, off, shape, strides, 0.125))
    assert_bits(O.contiguous(base, off, shape, strides), R.contiguous(base, off, shape, strides))
    d_ref = np.zeros(200, np.float32)
    d_or = np.zeros(200, np.float32)
    dshape, dstrides, doff = shape, (24, 6, 1), 7
    R.copy_(d_ref, doff, dshape, dstrides, base, off, shape, strides)
    O.copy_(d_or, doff, dshape, dstrides, base, off, shape, strides)
    assert_bits(d_or, d_ref)


def test_copy_shape_mismatch_raises():
    a = np.zeros(12, np.float32)
    with pytest.raises(ValueError):
        R.copy_(a, 0, (3, 4), (4, 1), a, 0, (4, 3), (3, 1))
    with pytest.raises(ValueError):
        O.copy_(a, 0, (3, 4), (4, 1), a, 0, (4, 3), (3, 1))


def test_kv_cache_copy_view():
    # attention.cpp:66-84: cache.slice(0, p, p+S).copy_(K.squeeze(0).transpose(0, 1))
    S, H, D, ctx, p = 7, 8, 64, 32, 5
    k = synth.normal((1, S, H, D), 1.0, seed=14).ravel()
    src_shape, src_strides = (S, H, D), (H * D, D, 1)
    c_ref = synth.normal((ctx * H * D,), 1.0, seed=15)
    c_or = c_ref.copy()
    R.copy_(c_ref, p * H * D, src_shape, (H * D, D, 1), k, 0, src_shape, src_strides)
    O.copy_(c_or, p * H * D, src_shape, (H * D, D, 1), k, 0, src_shape, src_strides)
    assert_bits(c_or, c_ref)


def test_rmsnorm_bit_exact():
    x = synth.normal((64, 2048), 1.0, seed=0)
    g = synth.uniform((2048,), 0.5, 1.5, seed=1)
    assert_bits(O.rmsnorm(x, g), R.rmsnorm(x, g))


def test_swiglu_bit_exact():
    g = synth.normal((8192 * 4,), 1.0, seed=2)
    u = synth.normal((8192 * 4,), 1.0, seed=3)
    g[:6] = [0.0, -0.0, 88.0, -88.0, -104.0, np.inf]
    assert_bits(O.swiglu(g, u), R.swiglu(g, u))


def test_softmax_bit_exact():
    x = synth.normal((3, 128256), 2.0, seed=4)
    assert_bits(O.softmax(x), R.softmax(x))
    y = synth.normal((16, 37), 1.0, seed=5)
    assert_bits(O.softmax(y), R.softmax(y))


def test_argmax_semantics():
    x = synth.normal((128256,), 2.0, seed=6)
    assert O.argmax(x) == R.greedy_sample(x) == int(np.argmax(x))
    t = np.array([1.0, 3.0, np.nan, 3.0, -np.inf], np.float32)
    assert O.argmax(t) == R.greedy_sample(t) == 1
    t = np.array([np.nan, -np.inf, np.nan], np.float32)
    assert O.argmax(t) == R.greedy_sample(t) == 0


def test_rope_tables_bit_exact():
    c_r, s_r = R.rope_tables(64, 1024, 500000.0)
    c_o, s_o = O.rope_tables(64, 1024, 500000.0)
    assert_bits(c_o, c_r)
    assert_bits(s_o, s_r)


@pytest.mark.parametrize("rank", [2, 4])
def test_rope_apply_bit_exact(rank):
    hd, max_seq, theta, pos = 64, 256, 500000.0, 17
    c, s = O.rope_tables(hd, max_seq, theta)
    if rank == 2:
        S = 9
        shape, strides, off, n = (S, hd), (hd, 1), 0, S * hd
    else:
        B, S, H = 1, 9, 8  # [1, S, H, D] storage viewed as [1, H, S, D] (transpose(1, 2))
        shape, strides, off, n = (B, H, S, hd), (S * H * hd, hd, H * hd, 1), 0, S * H * hd
    x = synth.normal((n,), 1.0, seed=20)
    xr, xo = x.copy(), x.copy()
    R.rope(xr, off, shape, strides, hd, max_seq, theta, pos)
    O.rope(xo, off, shape, strides, hd, max_seq, c, s, pos)
    assert_bits(xo, xr)


def test_rope_out_of_range():
    c, s = O.rope_tables(4, 10, 10000.0)
    x = np.zeros(8, np.float32)
    with pytest.raises(IndexError):
        R.rope(x.copy(), 0, (2, 4), (4, 1), 4, 10, 10000.0, 9)
    with pytest.raises(IndexError):
        O.rope(x.copy(), 0, (2, 4), (4, 1), 4, 10, c, s, 9)


@pytest.mark.parametrize("dtype", [0, 2, 3])
def test_embedding_bit_exact(dtype):
    dim, vocab = 256, 1000
    w = synth.normal((vocab, dim), 0.02, seed=21)
    if dtype == 0:
        wb = np.ascontiguousarray(w.T).view(np.uint8).ravel()  # logical {dim, vocab}
    elif dtype == 2:
        wb = synth.quantize_q8_0(w).ravel()
    else:
        wb = synth.quantize_q4_0(w).ravel()
    for ids in ([7.0], [0.0, 999.0, 5.0, 5.0, 123.0]):
        ids = np.array(ids, np.float32)
        assert_bits(O.embedding(wb, dtype, dim, vocab, ids), R.embedding(wb, dtype, dim, vocab, ids))
    with pytest.raises(IndexError):
        R.embedding(wb, dtype, dim, vocab, np.array([1000.0], np.float32))
    with pytest.raises(IndexError):
        O.embedding(wb, dtype, dim, vocab, np.array([1000.0], np.float32))


@pytest.mark.parametrize("M,K,N", [(1, 64, 37), (5, 64, 70), (3, 130, 9), (1, 64, 640)])
def test_matmul_f32_strided_bit_exact(M, K, N):
    # q_head[M, K] (row stride 2048) times k_head^T [K, N] (strides (1, 512)): the
    # attention score product of attention.cpp:110-117.
    a = synth.normal((M * 2048 + K,), 1.0, seed=30)
    b = synth.normal((N * 512 + K,), 1.0, seed=31)
    args = (a, 3, (M, K), (2048, 1), b, 5, (K, N), (1, 512))
    assert_bits(O.matmul_f32(*args), R.matmul_f32(*args))


def test_matmul_f32_batched_bit_exact():
    a = synth.normal((2 * 3 * 5 * 7,), 1.0, seed=32)
    b = synth.normal((2 * 3 * 7 * 11,), 1.0, seed=33)
    args = (a, 0, (2, 3, 5, 7), (105, 35, 7, 1), b, 0, (2, 3, 7, 11), (231, 77, 11, 1))
    assert_bits(O.matmul_f32(*args), R.matmul_f32(*args))


# -------------------------------------------------------------- sampling ----
# The reference draws its uniform number from a random_device-seeded mt19937,
# so its draws are pinned statistically: every draw lies in the oracle's
# nucleus, and the draw frequencies match the oracle's renormalised
# probabilities.

def _sorted_probs(x, temperature):
    p = O.softmax((np.asarray(x, f32) / f32(temperature)).astype(f32)[None])[0]
    order = np.lexsort((np.arange(p.size), -p))
    return p, order


@pytest.mark.parametrize("V,temperature,top_p", [(1000, 0.8, 0.9), (4000, 1.0, 0.9), (1000, 1.3, 0.5),
                                                 (600, 0.7, 0.95)])
def test_sample_top_p_reference_draws_lie_in_oracle_nucleus(V, temperature, top_p):
    x = synth.normal((V,), 2.0, seed=V + int(100 * top_p))
    _, nuc, nuc32, slack = O.sample_top_p(x, temperature, top_p, 0.5)
    assert nuc == nuc32  # the exact prefix mass and the reference's fp32 running sum agree here
    p, order = _sorted_probs(x, temperature)
    nucleus = order[:nuc]
    draws = R.sample_top_p(x, temperature, top_p, 4000)
    assert np.isin(draws, nucleus).all()
    freq = np.bincount(draws, minlength=V)[nucleus] / draws.size
    want = p[nucleus].astype(np.float64) / p[nucleus].astype(np.float64).sum()
    sigma = np.sqrt(want * (1 - want) / draws.size)
    assert (np.abs(freq - want) <= 5 * sigma + 2e-3).all()
    # the oracle's draw for u is the inverse of the same distribution function
    us = (np.arange(400) + 0.5) / 400
    ids = np.array([O.sample_top_p(x, temperature, top_p, u)[0] for u in us])
    cdf = np.cumsum(want)
    expect = nucleus[np.minimum(np.searchsorted(cdf, us), nuc - 1)]
    close = np.abs(cdf[np.minimum(np.searchsorted(cdf, us), nuc - 1)] - us) < 1e-6
    assert (ids[~close] == expect[~close]).all()


def test_sample_top_p_tiny_top_p_is_greedy():
    x = synth.normal((5000,), 2.0, seed=11)
    g = R.greedy_sample(x)
    assert (R.sample_top_p(x, 0.9, 1e-6, 200) == g).all()
    for u in (0.0, 0.3, 0.999999):
        tid, nuc, _, _ = O.sample_top_p(x, 0.9, 1e-6, u)
        assert tid == g and nuc == 1


def test_sample_top_p_oracle_ties_by_id_and_nan():
    V = 1000
    x = np.zeros(V, f32)  # every probability 1/V: ties ordered by id
    q = int(np.float64(f32(1) / f32(V)) * 2.0**62)
    for u in (0.0, 0.1234, 0.5, 0.9999):
        tid, nuc, _, _ = O.sample_top_p(x, 1.0, 0.5, u)
        assert nuc == -(-int(np.ceil(0.5 * 2.0**62)) // q)
        C = nuc * q
        t2 = int(np.ceil(u * float(C)))
        assert tid == max(1, -(-t2 // q)) - 1
    y = synth.normal((300,), 1.0, seed=2)
    y[7] = np.nan  # the reference's sum turns NaN: no positive probability, greedy's choice
    tid, _, _, slack = O.sample_top_p(y, 1.0, 0.9, 0.5)
    assert tid == O.argmax(y) and slack == 0.0

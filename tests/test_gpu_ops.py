"""GPU parity of every hot-path op against the oracle, through the C ABI.

Bit-exact (integer, byte, index work and the ops whose order the kernels keep):
dequant, quantize, Q8_0 / Q4_0 matmul on CUDA cores, copies, broadcast add,
scale, RoPE, embedding, fp32 matmul, argmax.  Tolerance-bound (tree reductions):
RMSNorm and softmax at 1e-5 relative (fp32), 1e-2 for bf16.  SwiGLU uses a
correctly rounded exp; it differs from glibc's expf only where glibc misrounds.
"""
import ctypes
import os

import numpy as np
import pytest

from oracle import orbind as O
from turbo_b200 import synth

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import turbo_b200 as T  # noqa: E402

F32_REL = 1e-5
BF16_REL = 1e-2


_KEEP = []  # device copies stay alive until the test's kernels have run


def dev(a):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    _KEEP.append(t)
    return t


@pytest.fixture(autouse=True)
def _release_inputs():
    yield
    torch.cuda.synchronize()
    _KEEP.clear()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def S():
    return T.stream_handle()


def assert_bits(a, b):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    assert a.shape == b.shape, (a.shape, b.shape)
    na, nb_ = np.isnan(a), np.isnan(b)
    assert np.array_equal(na, nb_)
    diff = (a.view(np.uint32) != b.view(np.uint32)) & ~na
    assert not diff.any(), "%d of %d differ; first at %s: %r vs %r" % (
        diff.sum(), diff.size, np.argwhere(diff)[0], a[tuple(np.argwhere(diff)[0])],
        b[tuple(np.argwhere(diff)[0])])


def assert_rel(a, b, tol):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    err = np.abs(a - b)
    scale = np.maximum(np.abs(b), np.abs(b).max() * 1e-3 + 1e-30)
    assert (err / scale).max() <= tol, "max rel err %g > %g" % ((err / scale).max(), tol)


def softmax_exact(x):
    x = np.asarray(x, np.float64)
    e = np.exp(x - x.max(axis=-1, keepdims=True))
    return e / e.sum(axis=-1, keepdims=True)


def assert_softmax(got, x):
    """Softmax tolerance.  The reference sums exp() sequentially in fp32; over
    128k columns that sum is itself ~1e-4 away from the exact value.  The CUDA
    result must be within 1e-5 (relative) of the exact softmax, and within the
    reference's own error (+1e-5) of the reference."""
    ref = O.softmax(x)
    exact = softmax_exact(x)
    assert_rel(got, exact, F32_REL)
    ref_err = np.max(np.abs(ref - exact) / np.maximum(exact, exact.max() * 1e-3))
    assert_rel(got, ref, ref_err + F32_REL)


@pytest.fixture(scope="module", autouse=True)
def _init():
    T.call("tb_init", 0)
    yield
    assert T.take_device_errors() == 0


# ----------------------------------------------------------------- quant ----

@pytest.mark.parametrize("dtype", [T.Q8_0, T.Q4_0])
@pytest.mark.parametrize("nblocks", [1, 31, 64 * 37, 8192 * 64 + 5])
def test_dequant_bit_exact(dtype, nblocks):
    w = synth.normal((nblocks * 32,), 0.02, seed=nblocks)
    q = synth.quantize_q8_0(w) if dtype == T.Q8_0 else synth.quantize_q4_0(w)
    out = torch.empty(nblocks * 32, dtype=torch.float32, device="cuda")
    T.call("tb_dequant", dtype, T.ptr(dev(q)), nblocks, T.ptr(out), S())
    ref = O.dequant_q8_0(q, nblocks) if dtype == T.Q8_0 else O.dequant_q4_0(q, nblocks)
    assert_bits(host(out), ref)


def test_quantize_q8_0_bit_exact():
    x = synth.normal((37, 2048), 1.0, seed=3)
    x[0, :32] = 0.0
    x[1, :32] = np.linspace(-3, 3, 32)
    x[2, 5] = np.nan
    q = torch.empty(37 * 64 * 34, dtype=torch.uint8, device="cuda")
    T.call("tb_quantize_q8_0", T.ptr(dev(x)), 37, 2048, T.ptr(q), S())
    got = host(q).reshape(37, -1)
    for r in range(37):
        ref = O.quantize_row_q8_0(x[r])
        if r == 2:  # the NaN element's own byte is unspecified (float->int8 of NaN)
            got[r, 2 + 5] = ref[2 + 5]
        assert np.array_equal(got[r], ref), r


# ----------------------------------------------------------------- matmul ----

def run_matmul(dtype, x, wq, N, entry="tb_matmul_quant_exact"):
    M, K = x.shape
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    T.call(entry, dtype, T.ptr(dev(x)), M, K, T.ptr(dev(wq)), N, T.ptr(y), S())
    return host(y)


def assert_dot_tol(got, x, wq, K, tol=F32_REL):
    """GEMV/GEMM tolerance: |y - y_ref| <= tol * sum_k |w_k x_k| per output (the
    conditioning of each dot product), with y_ref the reference's result."""
    N = wq.shape[0]
    scale = np.empty((x.shape[0], N))
    for r0 in range(0, N, 8192):  # chunked: the lm_head shape has 128256 rows
        wd = np.abs(synth.dequantize_q8_0(wq[r0:r0 + 8192], K)).astype(np.float64)
        scale[:, r0:r0 + 8192] = np.abs(x.astype(np.float64)) @ wd.T
    ref = O.matmul_q8_0(x, wq, N)
    err = np.abs(got.astype(np.float64) - ref)
    assert (err / scale).max() <= tol, "max scaled err %g" % (err / scale).max()


MATMUL_SHAPES = [(1, 2048, 8192), (1, 8192, 2048), (3, 2048, 515), (1, 64, 5), (2, 2080, 77),
                 (16, 1024, 300), (1, 2048, 128256), (1, 4096, 1000)]


@pytest.mark.parametrize("M,K,N", MATMUL_SHAPES)
def test_matmul_q8_0_exact_bit_exact(M, K, N):
    wq = synth.quantize_q8_0(synth.normal((N, K), 0.02, seed=K + N))
    x = synth.normal((M, K), 1.0, seed=M)
    assert_bits(run_matmul(T.Q8_0, x, wq, N), O.matmul_q8_0(x, wq, N))


@pytest.mark.parametrize("M,K,N", MATMUL_SHAPES)
def test_matmul_q8_0_default_within_tolerance(M, K, N):
    wq = synth.quantize_q8_0(synth.normal((N, K), 0.02, seed=K + N))
    x = synth.normal((M, K), 1.0, seed=M)
    assert_dot_tol(run_matmul(T.Q8_0, x, wq, N, "tb_matmul_quant"), x, wq, K)


@pytest.mark.parametrize("N,K", [(8192, 2048), (2048, 8192), (3000, 4096)])
def test_matmul_q8_0_digit_path_and_its_fallbacks(N, K):
    # M = 1 at K = 2048 takes x as int8 digits per block (dp4a); a block that
    # digits cannot hold (NaN, infinity, a tiny nonzero maximum) sends the
    # whole product to the fp32 dot; a block of wide range stays on digits.
    # K = 4096 and 8192 (the decode's down projection) take the fp32 dot with
    # the same special values.
    wq = synth.quantize_q8_0(synth.normal((N, K), 0.02, seed=41))
    base = synth.normal((1, K), 1.0, seed=42)
    cases = {"plain": base.copy(), "zeros": np.zeros((1, K), np.float32), "wide": base.copy(),
             "tiny": base.copy(), "nan": base.copy(), "inf": base.copy()}
    cases["wide"][0, 64:96] *= 1e-4
    cases["wide"][0, 70] = 1e3
    cases["tiny"][0, 128:160] *= 1e-33
    cases["nan"][0, 300] = np.nan
    cases["inf"][0, 5] = np.inf
    for name, x in cases.items():
        got = run_matmul(T.Q8_0, x, wq, N, "tb_matmul_quant")
        ref = O.matmul_q8_0(x, wq, N)
        if name in ("nan", "inf"):
            assert np.array_equal(np.isnan(got), np.isnan(ref)), name
            assert np.array_equal(got[~np.isnan(got)], ref[~np.isnan(ref)]), name
            continue
        if name == "zeros":
            assert np.array_equal(got, ref), name
            continue
        assert_dot_tol(got, x, wq, K)


def test_matmul_q8_0_unaligned_weight_base():
    N, K = 33, 2048
    wq = synth.quantize_q8_0(synth.normal((N, K), 0.02, seed=1)).ravel()
    x = synth.normal((1, K), 1.0, seed=2)
    buf = torch.zeros(wq.size + 16, dtype=torch.uint8, device="cuda")
    buf[6:6 + wq.size] = dev(wq)
    y = torch.empty((1, N), dtype=torch.float32, device="cuda")
    T.call("tb_matmul_quant_exact", T.Q8_0, T.ptr(dev(x)), 1, K, buf.data_ptr() + 6, N, T.ptr(y), S())
    assert_bits(host(y), O.matmul_q8_0(x, wq, N))


# (512, 8192, 2048): the prefill down projection X[512, 8192] . W_down
@pytest.mark.parametrize("M,K,N", [(1, 8192, 2048), (3, 8192, 130), (5, 64, 7), (512, 8192, 2048)])
def test_matmul_q4_0_bit_exact(M, K, N):
    wq = synth.quantize_q4_0(synth.normal((N, K), 0.02, seed=K + N))
    x = synth.normal((M, K), 1.0, seed=M + 1)
    assert_bits(run_matmul(T.Q4_0, x, wq, N), O.matmul_q4_0(x, wq, N, threads=os.cpu_count() or 1))


def test_matmul_q4_0_wait_timeout_is_reported():
    # A bounded wait that gives up (wait limit 0: no waiting allowed) leaves the
    # rows unwritten and sets bit 0 of the device error word; the context stays
    # usable and the next call, with the default limit, is exact again.
    M, K, N = 4, 2048, 300
    wq = synth.quantize_q4_0(synth.normal((N, K), 0.02, seed=3))
    x = synth.normal((M, K), 1.0, seed=4)
    dx, dw = dev(x), dev(wq)
    assert T.take_device_errors() == 0
    y = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    T.call("tb_set_wait_limit_ns", 0)
    try:
        T.call("tb_matmul_quant_exact", T.Q4_0, T.ptr(dx), M, K, T.ptr(dw), N, T.ptr(y), S())
        torch.cuda.synchronize()
    finally:
        T.call("tb_set_wait_limit_ns", 2000000000)
    assert T.take_device_errors() & 1
    assert np.isnan(host(y)).all()
    T.call("tb_matmul_quant_exact", T.Q4_0, T.ptr(dx), M, K, T.ptr(dw), N, T.ptr(y), S())
    assert_bits(host(y), O.matmul_q4_0(x, wq, N))
    assert T.take_device_errors() == 0


def assert_gemm_tol(got, xd, wd, tol=F32_REL):
    """|y - y_exact| <= tol * sum_k |w_k x_k| per output, y_exact in float64
    from the exactly dequantised operands (the reference is itself within
    ~1e-7 of it)."""
    x64, w64 = xd.astype(np.float64), wd.astype(np.float64)
    ref = x64 @ w64.T
    scale = np.abs(x64) @ np.abs(w64).T
    err = np.abs(got.astype(np.float64) - ref) / np.maximum(scale, 1e-30)
    assert err.max() <= tol, "max scaled err %g" % err.max()
    return err.max()


# prefill shapes on the tcgen05 path (M >= 32, K % 256 == 0): the benchmark's
# gate/up and down GEMMs, ragged M and N, a K range split over several CTAs
TC_SHAPES = [(512, 2048, 8192), (32, 256, 128), (130, 512, 300), (64, 2048, 1000), (200, 8192, 256),
             (33, 4096, 2049)]


@pytest.mark.parametrize("M,K,N", TC_SHAPES)
def test_matmul_q8_0_tensor_cores_within_tolerance(M, K, N):
    w = synth.normal((N, K), 0.02, seed=K + N)
    wq = synth.quantize_q8_0(w)
    x = synth.normal((M, K), 1.0, seed=M)
    got = run_matmul(T.Q8_0, x, wq, N, "tb_matmul_quant")
    # 1e-5 is the bar; exact block products keep the tensor-core path near 7e-8
    err = assert_gemm_tol(got, x, synth.dequantize_q8_0(wq, K), tol=1e-6)
    print("Q8_0 %dx%dx%d: max scaled error %.3g" % (M, K, N, err))
    if M * N * K <= 64 * 2048 * 1000:  # and against the oracle's own result
        assert_dot_tol(got, x, wq, K)


@pytest.mark.parametrize("M,K,N", [(512, 8192, 2048), (64, 256, 130), (96, 1024, 640)])
def test_matmul_q4_0_tensor_cores_within_tolerance(M, K, N):
    wq = synth.quantize_q4_0(synth.normal((N, K), 0.02, seed=K + N))
    x = synth.normal((M, K), 1.0, seed=M + 1)
    got = run_matmul(T.Q4_0, x, wq, N, "tb_matmul_quant")
    xd = synth.dequantize_q8_0(synth.quantize_q8_0(x), K)  # the reference quantises X rows
    err = assert_gemm_tol(got, xd, synth.dequantize_q4_0(wq, K), tol=1e-6)
    print("Q4_0 %dx%dx%d: max scaled error %.3g" % (M, K, N, err))
    if M <= 96:
        ref = O.matmul_q4_0(x, wq, N)
        scale = np.abs(xd.astype(np.float64)) @ np.abs(synth.dequantize_q4_0(wq, K).astype(np.float64)).T
        assert (np.abs(got - ref) / scale).max() <= F32_REL


# packed weights: the same kernel as tb_matmul_quant, W converted once.  The
# shapes reach both token tiles (128, 256) and K split over clusters of 2-8.
@pytest.mark.parametrize("dtype,M,K,N", [("q8", 512, 2048, 1000), ("q4", 300, 8192, 640), ("q4", 33, 4096, 2049),
                                         ("q8", 64, 2048, 1000), ("q4", 200, 8192, 256)])
def test_matmul_quant_packed_matches_unpacked(dtype, M, K, N):
    dt = T.Q8_0 if dtype == "q8" else T.Q4_0
    w = synth.normal((N, K), 0.02, seed=K + 3 * N)
    wq = synth.quantize_q8_0(w) if dtype == "q8" else synth.quantize_q4_0(w)
    x = synth.normal((M, K), 1.0, seed=M + 7)
    want = run_matmul(dt, x, wq, N, "tb_matmul_quant")
    nbytes = ctypes.c_size_t(0)
    T.call("tb_packed_quant_weights_bytes", dt, N, K, ctypes.byref(nbytes))
    packed = torch.empty(nbytes.value, dtype=torch.uint8, device="cuda")
    T.call("tb_pack_quant_weights", dt, T.ptr(dev(wq)), N, K, T.ptr(packed), nbytes.value, S())
    xd = dev(x)
    for _ in range(2):  # the packed copy is reusable
        y = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
        T.call("tb_matmul_quant_packed", dt, T.ptr(xd), M, K, T.ptr(packed), N, T.ptr(y), S())
        assert_bits(host(y), want)


def test_matmul_quant_packed_rejects_bad_arguments():
    K, N = 512, 130
    wq = synth.quantize_q8_0(synth.normal((N, K), 0.02, seed=5))
    nbytes = ctypes.c_size_t(0)
    T.call("tb_packed_quant_weights_bytes", T.Q8_0, N, K, ctypes.byref(nbytes))
    packed = torch.empty(nbytes.value, dtype=torch.uint8, device="cuda")
    with pytest.raises(T.TbError) as e:  # too small a buffer
        T.call("tb_pack_quant_weights", T.Q8_0, T.ptr(dev(wq)), N, K, T.ptr(packed), nbytes.value - 16, S())
    assert e.value.status == T.EINVAL
    T.call("tb_pack_quant_weights", T.Q8_0, T.ptr(dev(wq)), N, K, T.ptr(packed), nbytes.value, S())
    x = dev(synth.normal((31, K), 1.0, seed=1))
    y = torch.empty((31, N), dtype=torch.float32, device="cuda")
    with pytest.raises(T.TbError) as e:  # M < 32 belongs to tb_matmul_quant
        T.call("tb_matmul_quant_packed", T.Q8_0, T.ptr(x), 31, K, T.ptr(packed), N, T.ptr(y), S())
    assert e.value.status == T.EINVAL
    with pytest.raises(T.TbError) as e:  # K not a multiple of 256
        T.call("tb_matmul_quant_packed", T.Q8_0, T.ptr(x), 32, 480, T.ptr(packed), N, T.ptr(y), S())
    assert e.value.status == T.EINVAL


def test_matmul_quant_rejects_bad_k():
    x = torch.zeros((1, 40), device="cuda")
    with pytest.raises(T.TbError) as e:
        T.call("tb_matmul_quant", T.Q8_0, T.ptr(x), 1, 40, T.ptr(x), 1, T.ptr(x), S())
    assert e.value.status == T.EINVAL


@pytest.mark.parametrize("M,K,N", [(1, 64, 37), (5, 64, 70), (3, 130, 9), (1, 64, 640)])
def test_matmul_f32_attention_views_bit_exact(M, K, N):
    a = synth.normal((M * 2048 + K,), 1.0, seed=30)
    b = synth.normal((N * 512 + K,), 1.0, seed=31)
    ref = O.matmul_f32(a, 3, (M, K), (2048, 1), b, 5, (K, N), (1, 512))
    out = torch.empty((M, N), dtype=torch.float32, device="cuda")
    da, db = dev(a), dev(b)
    T.call("tb_matmul_f32", T.byref(T.view(da, 3, (M, K), (2048, 1))),
           T.byref(T.view(db, 5, (K, N), (1, 512))), T.byref(T.view(out)), S())
    assert_bits(host(out), ref)


def test_matmul_f32_batched_bit_exact():
    a = synth.normal((2 * 3 * 5 * 7,), 1.0, seed=32)
    b = synth.normal((2 * 3 * 7 * 11,), 1.0, seed=33)
    ref = O.matmul_f32(a, 0, (2, 3, 5, 7), (105, 35, 7, 1), b, 0, (2, 3, 7, 11), (231, 77, 11, 1))
    out = torch.empty((2, 3, 5, 11), dtype=torch.float32, device="cuda")
    T.call("tb_matmul_f32", T.byref(T.view(dev(a), 0, (2, 3, 5, 7), (105, 35, 7, 1))),
           T.byref(T.view(dev(b), 0, (2, 3, 7, 11), (231, 77, 11, 1))), T.byref(T.view(out)), S())
    assert_bits(host(out), ref)


@pytest.mark.parametrize("case", ["scores", "context", "odd", "a_transposed", "batched", "wide"])
def test_matmul_f32_tiled_bit_exact(case):
    # from 32 rows and 32 columns on: 64x64 (or, with at least one per SM,
    # 128x128) output tiles staged through shared memory, each output still the
    # k-ordered fma chain (attention.cpp:115-132 at prefill shapes: Q_h K_h^T,
    # then P V_h)
    if case == "batched":
        a = synth.normal((2 * 3 * 70 * 33,), 1.0, seed=40)
        b = synth.normal((2 * 3 * 33 * 45,), 1.0, seed=41)
        sa, sta = (2, 3, 70, 33), (6930, 2310, 33, 1)
        sb, stb = (2, 3, 33, 45), (4455, 1485, 45, 1)
        oa = ob = 0
    else:
        M, K, N, sta, stb, oa, ob = {
            "scores": (512, 64, 512, (2048, 1), (1, 512), 3, 5),    # Q_h [S,64] x K_h^T (cache rows of 512)
            "context": (512, 512, 64, (512, 1), (512, 1), 0, 7),    # P [S,ctx] x V_h [ctx,64]
            "odd": (96, 130, 77, (2048, 1), (1, 512), 3, 5),
            "a_transposed": (64, 40, 70, (1, 64), (70, 1), 0, 0),
            "wide": (1600, 37, 1700, (37, 1), (1, 37), 0, 0),       # 128x128 tiles, B read along k
        }[case]
        sa, sb = (M, K), (K, N)
        a = synth.normal((oa + (sa[0] - 1) * sta[0] + (sa[1] - 1) * sta[1] + 1,), 1.0, seed=42)
        b = synth.normal((ob + (sb[0] - 1) * stb[0] + (sb[1] - 1) * stb[1] + 1,), 1.0, seed=43)
    ref = O.matmul_f32(a, oa, sa, sta, b, ob, sb, stb)
    out = torch.empty(tuple(sa[:-1]) + (sb[-1],), dtype=torch.float32, device="cuda")
    T.call("tb_matmul_f32", T.byref(T.view(dev(a), oa, sa, sta)), T.byref(T.view(dev(b), ob, sb, stb)),
           T.byref(T.view(out)), S())
    assert_bits(host(out), ref)


@pytest.mark.parametrize("nbytes", [16, 8192, 32768, 262144, 262160, 100])
def test_upload_download_pinned_and_pageable(nbytes):
    # page-locked buffers of up to 256 KB in 16-byte units move by a copy kernel
    # through the host mapping; pageable, larger or unaligned ones by DMA: the
    # bytes arrive unchanged either way
    src = np.random.default_rng(nbytes).integers(0, 256, nbytes + 4, dtype=np.uint8)
    d = torch.empty(nbytes + 64, dtype=torch.uint8, device="cuda")
    pin = torch.from_numpy(src.copy()).pin_memory()
    back = torch.zeros(nbytes + 4, dtype=torch.uint8).pin_memory()
    for off in (0, 4):  # 4: a host address not on a 16-byte boundary (DMA)
        L = T.load()
        T.check(L.tb_upload(T.ptr(d), ctypes.c_void_p(pin.data_ptr() + off), nbytes, S()))
        T.check(L.tb_download(ctypes.c_void_p(back.data_ptr() + off), T.ptr(d), nbytes, S()))
        torch.cuda.synchronize()
        assert np.array_equal(back.numpy()[off:off + nbytes], src[off:off + nbytes])
        page = np.zeros(nbytes, np.uint8)
        T.check(L.tb_download(ctypes.c_void_p(page.ctypes.data), T.ptr(d), nbytes, S()))
        torch.cuda.synchronize()
        assert np.array_equal(page, src[off:off + nbytes])


def test_small_upload_waits_for_the_previous_reader():
    # x is read by a GEMV and then overwritten by a small upload from pinned
    # memory, then read again, all on one stream: each GEMV sees its own x
    N, K = 4096, 2048
    wq = synth.quantize_q8_0(synth.normal((N, K), 0.02, seed=70))
    xa, xb = synth.normal((1, K), 1.0, seed=71), synth.normal((1, K), 1.0, seed=72)
    dw = dev(wq)
    x = dev(xa)
    pa, pb = torch.from_numpy(xa).pin_memory(), torch.from_numpy(xb).pin_memory()
    y1 = torch.empty((1, N), device="cuda")
    y2 = torch.empty((1, N), device="cuda")
    L = T.load()
    for _ in range(3):
        T.call("tb_matmul_quant_exact", T.Q8_0, T.ptr(x), 1, K, T.ptr(dw), N, T.ptr(y1), S())
        T.check(L.tb_upload(T.ptr(x), ctypes.c_void_p(pb.data_ptr()), K * 4, S()))
        T.call("tb_matmul_quant_exact", T.Q8_0, T.ptr(x), 1, K, T.ptr(dw), N, T.ptr(y2), S())
        T.check(L.tb_upload(T.ptr(x), ctypes.c_void_p(pa.data_ptr()), K * 4, S()))
        torch.cuda.synchronize()
        assert_bits(host(y1), O.matmul_q8_0(xa, wq, N))
        assert_bits(host(y2), O.matmul_q8_0(xb, wq, N))


# ------------------------------------------------------------ elementwise ----

@pytest.mark.parametrize("sa,sb", [((1, 128, 2048), (1, 128, 2048)), ((4, 1, 8), (3, 1)),
                                   ((2, 3, 4), (4,)), ((5,), (2, 1, 5)), ((7, 1), (1, 9)),
                                   ((64, 4096), (4096,)), ((4096,), (3, 4096)), ((3, 5), (3, 5))])
def test_add_broadcast_bit_exact(sa, sb):
    a = synth.normal(sa, 1.0, seed=1)
    b = synth.normal(sb, 1.0, seed=2)
    ref = O.add(a, 0, sa, [s // 4 for s in a.strides], b, 0, sb, [s // 4 for s in b.strides])
    out = torch.empty(ref.shape, dtype=torch.float32, device="cuda")
    T.call("tb_binary", 0, T.byref(T.view(dev(a))), T.byref(T.view(dev(b))), T.byref(T.view(out)), S())
    assert_bits(host(out), ref)


def test_mul_rowvector_and_bf16_add():
    a = synth.normal((64, 4096), 1.0, seed=5)
    g = synth.normal((4096,), 1.0, seed=6)
    out = torch.empty((64, 4096), dtype=torch.float32, device="cuda")
    T.call("tb_binary", 1, T.byref(T.view(dev(a))), T.byref(T.view(dev(g))), T.byref(T.view(out)), S())
    assert_bits(host(out), (a * g).astype(np.float32))
    ab = dev(a).to(torch.bfloat16)
    bb = dev(synth.normal((64, 4096), 1.0, seed=7)).to(torch.bfloat16)
    ob = torch.empty_like(ab)
    T.call("tb_binary", 0, T.byref(T.view(ab)), T.byref(T.view(bb)), T.byref(T.view(ob)), S())
    ref = O.add(*(lambda x, y: (x, 0, x.shape, (4096, 1), y, 0, y.shape, (4096, 1)))(
        ab.float().cpu().numpy(), bb.float().cpu().numpy()))
    assert_rel(ob.float().cpu().numpy(), ref, BF16_REL)


def test_add_not_broadcastable():
    a = torch.zeros((3, 4), device="cuda")
    b = torch.zeros((5,), device="cuda")
    out = torch.zeros((3, 4), device="cuda")
    with pytest.raises(T.TbError) as e:
        T.call("tb_binary", 0, T.byref(T.view(a)), T.byref(T.view(b)), T.byref(T.view(out)), S())
    assert e.value.status == T.EINVAL


def test_scale_and_contiguous_and_copy_strided_bit_exact():
    base = synth.normal((4 * 6 * 5 + 3,), 1.0, seed=13)
    shape, strides, off = (5, 4, 6), (1, 30, 5), 3
    db = dev(base)
    out = torch.empty(shape, dtype=torch.float32, device="cuda")
    T.call("tb_scale", T.byref(T.view(db, off, shape, strides)), 0.125, T.byref(T.view(out)), S())
    assert_bits(host(out), O.scale(base, off, shape, strides, 0.125))
    T.call("tb_copy", T.byref(T.view(out)), T.byref(T.view(db, off, shape, strides)), S())
    assert_bits(host(out), O.contiguous(base, off, shape, strides))
    dst = np.zeros(200, np.float32)
    dd = dev(dst)
    T.call("tb_copy", T.byref(T.view(dd, 7, shape, (24, 6, 1))), T.byref(T.view(db, off, shape, strides)), S())
    O.copy_(dst, 7, shape, (24, 6, 1), base, off, shape, strides)
    assert_bits(host(dd), dst)


@pytest.mark.parametrize("S_,H,D", [(1, 32, 64), (512, 32, 64), (7, 8, 64)])
def test_contiguous_of_transposed_attention_context(S_, H, D):
    # context [1, H, S, D] -> transpose(1, 2) -> contiguous (attention.cpp:144-145)
    ctx = synth.normal((H * S_ * D,), 1.0, seed=S_)
    shape, strides = (1, S_, H, D), (H * S_ * D, D, S_ * D, 1)
    out = torch.empty(shape, dtype=torch.float32, device="cuda")
    T.call("tb_copy", T.byref(T.view(out)), T.byref(T.view(dev(ctx), 0, shape, strides)), S())
    assert_bits(host(out), O.contiguous(ctx, 0, shape, strides))


def test_kv_cache_append_and_transpose_copy():
    S_, H, D, ctx, p = 7, 8, 64, 64, 5
    k = synth.normal((S_ * H * D,), 1.0, seed=14)
    cache = synth.normal((ctx * H * D,), 1.0, seed=15)
    dc = dev(cache)
    T.call("tb_copy", T.byref(T.view(dc, p * H * D, (S_, H, D), (H * D, D, 1))),
           T.byref(T.view(dev(k), 0, (S_, H, D), (H * D, D, 1))), S())
    O.copy_(cache, p * H * D, (S_, H, D), (H * D, D, 1), k, 0, (S_, H, D), (H * D, D, 1))
    assert_bits(host(dc), cache)
    # a truly strided source: K viewed [S, H, D] with strides (D, S*D, 1)
    dc2 = dev(cache)
    T.call("tb_copy", T.byref(T.view(dc2, p * H * D, (S_, H, D), (H * D, D, 1))),
           T.byref(T.view(dev(k), 0, (S_, H, D), (D, S_ * D, 1))), S())
    O.copy_(cache, p * H * D, (S_, H, D), (H * D, D, 1), k, 0, (S_, H, D), (D, S_ * D, 1))
    assert_bits(host(dc2), cache)


@pytest.mark.parametrize("shape", [(300, 200), (3, 100, 90), (64, 64), (2, 33, 70), (130, 258), (4, 66, 2050)])
def test_contiguous_of_transpose_tiles_bit_exact(shape):
    # contiguous() of a view whose last two dims are swapped: the tiled
    # transpose path (64x64 tiles when both extents reach 64, else 32x32;
    # 16-bit elements move as 32-bit pairs when every extent and offset is
    # even, partial tiles included)
    *lead, R, C = shape
    n = int(np.prod(shape))
    src = synth.normal((n,), 1.0, seed=n)
    # source memory is [lead..., C, R] contiguous; the view is [lead..., R, C]
    mem_shape = tuple(lead) + (C, R)
    mst = [1] * len(mem_shape)
    for i in range(len(mem_shape) - 2, -1, -1):
        mst[i] = mst[i + 1] * mem_shape[i + 1]
    vstrides = tuple(mst[:-2]) + (1, R)
    for dt in (torch.float32, torch.bfloat16):
        ds = dev(src).to(dt)
        out = torch.empty(shape, dtype=dt, device="cuda")
        T.call("tb_copy", T.byref(T.view(out)), T.byref(T.view(ds, 0, shape, vstrides)), S())
        want = ds.as_strided(shape, vstrides).contiguous()
        assert torch.equal(out.view(torch.int16) if dt == torch.bfloat16 else out.view(torch.int32),
                           want.view(torch.int16) if dt == torch.bfloat16 else want.view(torch.int32))
    ref = O.contiguous(src, 0, shape, vstrides)
    got = torch.empty(shape, dtype=torch.float32, device="cuda")
    T.call("tb_copy", T.byref(T.view(got)), T.byref(T.view(dev(src), 0, shape, vstrides)), S())
    assert_bits(host(got), ref)


def test_copy_shape_mismatch():
    a = torch.zeros(12, device="cuda")
    with pytest.raises(T.TbError) as e:
        T.call("tb_copy", T.byref(T.view(a, 0, (3, 4), (4, 1))), T.byref(T.view(a, 0, (4, 3), (3, 1))), S())
    assert e.value.status == T.EINVAL


@pytest.mark.parametrize("n", [1, 5, 8192 * 128, 8192 * 128 + 3])
def test_swiglu_matches_libm(n):
    g = synth.normal((n,), 1.0, seed=2)
    u = synth.normal((n,), 1.0, seed=3)
    if n > 8:
        g[:6] = [0.0, -0.0, 88.0, -88.0, -104.0, 20.0]
    y = torch.empty(n, dtype=torch.float32, device="cuda")
    T.call("tb_swiglu", T.F32, T.ptr(dev(g)), T.ptr(dev(u)), T.ptr(y), n, S())
    got, ref = host(y), O.swiglu(g, u)
    # The kernel's exp is correctly rounded; glibc's expf (used by the
    # reference and the oracle) misrounds on ~0.03% of inputs by one ulp, which
    # the division and product carry to at most a few ulps of the result.
    diff = got.view(np.uint32).astype(np.int64) - ref.view(np.uint32).astype(np.int64)
    assert np.abs(diff).max() <= 4
    assert np.count_nonzero(diff) <= max(1, n // 1000)
    assert_rel(got, ref, F32_REL)


def test_swiglu_bf16():
    g = synth.normal((8192 * 16,), 1.0, seed=4)
    u = synth.normal((8192 * 16,), 1.0, seed=5)
    gb, ub = dev(g).to(torch.bfloat16), dev(u).to(torch.bfloat16)
    y = torch.empty_like(gb)
    T.call("tb_swiglu", T.BF16, T.ptr(gb), T.ptr(ub), T.ptr(y), g.size, S())
    ref = O.swiglu(gb.float().cpu().numpy(), ub.float().cpu().numpy())
    assert_rel(y.float().cpu().numpy(), ref, BF16_REL)


# ------------------------------------------------------------------ rows ----

@pytest.mark.parametrize("rows,cols", [(128, 2048), (1, 2048), (3, 4096), (5, 100), (2, 16384)])
def test_rmsnorm(rows, cols):
    x = synth.normal((rows, cols), 1.0, seed=rows)
    g = synth.uniform((cols,), 0.5, 1.5, seed=cols)
    y = torch.empty((rows, cols), dtype=torch.float32, device="cuda")
    T.call("tb_rmsnorm", T.F32, T.ptr(dev(x)), T.ptr(dev(g)), T.ptr(y), rows, cols, 1e-5, S())
    assert_rel(host(y), O.rmsnorm(x, g), F32_REL)


def test_rmsnorm_kat_and_bf16():
    # reference test_nn.cpp RMSNormForwardPass: [1,2,3,4], gamma [.5,1,1.5,2]
    y = torch.empty((1, 4), dtype=torch.float32, device="cuda")
    T.call("tb_rmsnorm", T.F32, T.ptr(dev(np.array([[1, 2, 3, 4]], np.float32))),
           T.ptr(dev(np.array([0.5, 1, 1.5, 2], np.float32))), T.ptr(y), 1, 4, 1e-5, S())
    np.testing.assert_allclose(host(y)[0], [0.182574, 0.730296, 1.643167, 2.921186], atol=1e-4)
    x = synth.normal((64, 4096), 1.0, seed=9)
    g = synth.uniform((4096,), 0.5, 1.5, seed=10)
    xb = dev(x).to(torch.bfloat16)
    yb = torch.empty_like(xb)
    T.call("tb_rmsnorm", T.BF16, T.ptr(xb), T.ptr(dev(g)), T.ptr(yb), 64, 4096, 1e-5, S())
    assert_rel(yb.float().cpu().numpy(), O.rmsnorm(xb.float().cpu().numpy(), g), BF16_REL)


@pytest.mark.parametrize("rows,cols", [(1, 128256), (3, 37), (64, 128256), (16, 640), (2, 300000), (8, 65536)])
def test_softmax(rows, cols):
    x = synth.normal((rows, cols), 2.0, seed=cols)
    y = torch.empty((rows, cols), dtype=torch.float32, device="cuda")
    T.call("tb_softmax", T.ptr(dev(x)), T.ptr(y), rows, cols, S())
    assert_softmax(host(y), x)


@pytest.mark.parametrize("rows,cols", [(200, 128256), (160, 100004), (300, 8000), (170, 60000)])
def test_softmax_many_rows_two_pass(rows, cols):
    # at least one row per SM: the persistent CTA-per-row kernel; 8000 columns
    # stay in registers between the passes, 60000 in registers and shared
    # memory, the longer rows also re-read part of the row from L2
    check_softmax_special_rows(rows, cols)


@pytest.mark.parametrize("rows,cols", [(40, 128256), (64, 128256), (15, 300000), (100, 4004), (100, 128256)])
def test_softmax_few_rows_special_values(rows, cols):
    # 8 rows to one per SM: the two-launch chunked kernels (rows split into
    # chunks of at most 8192 columns, statistics combined in the second
    # launch), or clusters for rows wider than 16 chunks
    check_softmax_special_rows(rows, cols)


def check_softmax_special_rows(rows, cols):
    from oracle import refbind as R
    x = synth.normal((rows, cols), 2.0, seed=rows)
    x[7, min(12345, cols - 1)] = 30.0
    x[11, ::3] = -np.inf
    x[12, 5] = np.nan
    x[13, :] = -np.inf
    x[14, 99] = np.inf
    y = torch.empty((rows, cols), dtype=torch.float32, device="cuda")
    T.call("tb_softmax", T.ptr(dev(x)), T.ptr(y), rows, cols, S())
    got = host(y)
    ref = R.softmax(x) if R.available() else O.softmax(x)
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    ok = [r for r in range(rows) if r not in (12, 13, 14)]
    assert not got[11, ::3].any()
    assert_softmax(got[ok], x[ok])
    assert T.take_device_errors() == 0


def test_softmax_many_short_rows():
    # more clusters than SMs: the 256-thread CTA variant
    x = synth.normal((160, 4099), 2.0, seed=5)
    y = torch.empty((160, 4099), dtype=torch.float32, device="cuda")
    T.call("tb_softmax", T.ptr(dev(x)), T.ptr(y), 160, 4099, S())
    assert_softmax(host(y), x)


@pytest.mark.parametrize("cols", [9, 128256])
def test_softmax_special_values_match_reference(cols):
    # -inf entries give 0; a NaN, an all -inf row or a +inf make the row NaN
    from oracle import refbind as R
    x = synth.normal((4, cols), 2.0, seed=cols)
    x[0, 3] = -np.inf
    x[1, cols // 2] = np.nan
    x[2, :] = -np.inf
    x[3, cols - 1] = np.inf
    y = torch.empty((4, cols), dtype=torch.float32, device="cuda")
    T.call("tb_softmax", T.ptr(dev(x)), T.ptr(y), 4, cols, S())
    got = host(y)
    ref = R.softmax(x) if R.available() else O.softmax(x)
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    assert got[0, 3] == 0.0
    assert_softmax(got[:1], x[:1])


def test_exp_selfcheck_every_float():
    # a test-only library (turbo.cpp_b200/csrc/test), built beside the product one
    lib = ctypes.CDLL(os.path.join(os.path.dirname(T.LIB_PATH), "libturbo_b200_selfcheck.so"))
    lib.tb_selfcheck_exp.argtypes = [ctypes.c_void_p]
    lib.tb_selfcheck_exp.restype = ctypes.c_int
    torch.cuda.init()
    counts = (ctypes.c_uint64 * 4)()
    assert lib.tb_selfcheck_exp(ctypes.cast(counts, ctypes.c_void_p)) == 0
    n_cr, max_cr, n_fast, max_fast = list(counts)
    print("exp_cr: %d of 2^32 inputs differ from the double-precision exp (max %d ulp); "
          "__expf: %d beyond its documented bound on [-87, 0] (max %d ulp on [-20, 0])"
          % (n_cr, max_cr, n_fast, max_fast))
    assert max_cr <= 1 and n_cr <= 1024
    assert n_fast == 0 and max_fast <= 26


def test_softmax_kat():
    # reference test_tensor.cpp NumericallyStableSoftmax
    x = np.array([[1, 2, 3], [10, 100, 10]], np.float32)
    y = torch.empty((2, 3), dtype=torch.float32, device="cuda")
    T.call("tb_softmax", T.ptr(dev(x)), T.ptr(y), 2, 3, S())
    np.testing.assert_allclose(host(y).ravel(), [0.0900, 0.2447, 0.6652, 0, 1, 0], atol=1e-4)


def argmax_gpu(x):
    x = np.ascontiguousarray(x, np.float32)
    rows, cols = x.shape
    idx = torch.empty(rows, dtype=torch.int64, device="cuda")
    T.call("tb_argmax", T.ptr(dev(x)), rows, cols, T.ptr(idx), S())
    return host(idx)


@pytest.mark.parametrize("rows,cols", [(1, 128256), (64, 128256), (5, 3), (2, 9000), (1, 1)])
def test_argmax_random(rows, cols):
    x = synth.normal((rows, cols), 2.0, seed=rows * cols)
    got = argmax_gpu(x)
    for r in range(rows):
        assert got[r] == O.argmax(x[r])


def test_argmax_ties_nan_inf():
    rows = [
        [1.0, 3.0, np.nan, 3.0, -np.inf],
        [np.nan, -np.inf, np.nan],
        [np.nan, 2.0, 2.0],
        [-np.inf, -np.inf, -np.inf],
        [np.inf, np.inf, 1.0],
        [-0.0, 0.0, -0.0],
    ]
    for r in rows:
        x = np.array([r], np.float32)
        assert argmax_gpu(x)[0] == O.argmax(x[0]), r
    big = np.full((1, 128256), -1.0, np.float32)
    big[0, 77777] = 5.0
    big[0, 100000] = 5.0
    big[0, 5] = np.nan
    assert argmax_gpu(big)[0] == 77777 == O.argmax(big[0])


# -------------------------------------------------------------- sampling ----
# Nucleus sampling with the uniform number given.  The device's exp is within
# 2 ulp and its softmax sum is a tree, so its probabilities differ from the
# reference's by rounding, which can move a cut point when top_p or u sits
# close to a prefix boundary.  The oracle therefore returns the set of draws
# reachable under a perturbation of that size:
# - against the exact-sum oracle: top_p x (1 +- 1e-5), u +- 1e-6 -- most
#   cases have a single answer, so this checks the selection itself;
# - against the reference-faithful oracle (its sequential fp32 sum, whose own
#   error reaches 5e-4 at 300k terms): top_p x (1 +- that error + 1e-5).
# Rows whose probabilities are exact on both sides (equal logits, -inf) are
# compared exactly.

def sample_many(xd, V, temperature, top_p, us):
    out = torch.full((len(us),), -1, dtype=torch.int32, device="cuda")
    for i, u in enumerate(us):
        T.call("tb_sample_top_p", T.ptr(xd), V, float(temperature), float(top_p), float(u), T.ptr(out[i:]), S())
    return host(out)


US = [0.0] + list((np.arange(16) + 0.37) / 16) + [0.999999]


def reference_sum_error(x, temperature):
    s = (np.asarray(x, np.float32) / np.float32(temperature)).astype(np.float32)
    e = np.exp((s - s.max()).astype(np.float32))
    return abs(float(np.cumsum(e, dtype=np.float32)[-1]) / e.astype(np.float64).sum() - 1.0)


@pytest.mark.parametrize("V", [1, 7, 1000, 32000, 128256, 151936, 262144, 300001])
def test_sample_top_p_matches_oracle(V):
    x = synth.normal((V,), 2.5, seed=V)
    xd = dev(x)
    single = total = 0
    for temperature, top_p in [(0.8, 0.9), (1.0, 0.5), (1.3, 0.99), (0.6, 0.0), (1.0, 1.5), (0.9, 0.95)]:
        got = sample_many(xd, V, temperature, top_p, US)
        rel_ref = 2 * reference_sum_error(x, temperature) + 1e-5
        for u, g in zip(US, got):
            exact = O.sample_top_p_set(x, temperature, top_p, u, 1e-5, 1e-6, accurate_sum=True)
            faithful = O.sample_top_p_set(x, temperature, top_p, u, rel_ref, 1e-6)
            assert g in exact and g in faithful, (temperature, top_p, u, g, exact, faithful)
            total += 1
            single += len(exact) == 1
    assert single >= 0.75 * total, (single, total)


@pytest.mark.parametrize("V,every", [(1000, 1), (128256, 1), (128256, 5), (300001, 7), (262144, 3)])
def test_sample_top_p_ties_across_slices(V, every):
    # equal logits (every `every`-th id, the rest -inf): exact equal probabilities,
    # ordered by id across the cluster's slices
    x = np.full(V, -np.inf, np.float32)
    x[::every] = 0.0
    xd = dev(x)
    for top_p in (0.5, 0.9, 0.0, 2.0):
        got = sample_many(xd, V, 1.0, top_p, US)
        for u, g in zip(US, got):
            assert g == O.sample_top_p(x, 1.0, top_p, u)[0], (top_p, u)


def test_sample_top_p_at_reads_uniform_of_position():
    # the graph form: u = u_dev[*pos_dev] (clamped into [0, max_seq)), id as int64
    V, max_seq = 32000, 64
    x = synth.normal((V,), 2.5, seed=5)
    xd = dev(x)
    us = np.random.default_rng(3).random(max_seq)
    ud = dev(us)
    for pos in (0, 17, 63, 200, -5):
        pd = dev(np.array([pos], np.int32))
        idx = torch.full((1,), -1, dtype=torch.int64, device="cuda")
        T.call("tb_sample_top_p_at", T.ptr(xd), V, 0.8, 0.9, T.ptr(ud), T.ptr(pd), max_seq, T.ptr(idx), S())
        u = us[min(max(pos, 0), max_seq - 1)]
        assert int(host(idx)[0]) == int(sample_many(xd, V, 0.8, 0.9, [u])[0]), pos
    with pytest.raises(T.TbError):
        T.call("tb_sample_top_p_at", T.ptr(xd), V, 0.8, 0.9, None, T.ptr(ud), max_seq, T.ptr(idx), S())


def test_sample_top_p_degenerate_rows():
    cases = [np.array([1.0, np.nan, 3.0, 3.0], np.float32),       # NaN: greedy's first maximum
             np.full(5, -np.inf, np.float32),                     # no finite logit: 0
             np.array([0.0, np.inf, 1.0, np.inf], np.float32),    # +inf: first +inf
             np.array([2.0], np.float32)]
    for x in cases:
        got = sample_many(dev(x), x.size, 0.7, 0.9, [0.3])[0]
        assert got == O.sample_top_p(x, 0.7, 0.9, 0.3)[0] == O.argmax(x), x


def test_sample_top_p_unaligned_row_and_errors():
    V = 5001
    x = synth.normal((V + 1,), 2.0, seed=9)
    xd = dev(x)
    out = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    T.call("tb_sample_top_p", T.ptr(xd[1:]), V, 0.8, 0.9, 0.4, T.ptr(out), S())  # a row 4 bytes past 16-byte alignment
    assert O.sample_top_p_set(x[1:], 0.8, 0.9, 0.4, 1e-5, 1e-6, accurate_sum=True) == {int(host(out)[0])}
    for args in [(0.0, 0.9), (-1.0, 0.9), (float("nan"), 0.9)]:
        with pytest.raises(T.TbError):
            T.call("tb_sample_top_p", T.ptr(xd), V, args[0], args[1], 0.5, T.ptr(out), S())
    with pytest.raises(T.TbError):
        T.call("tb_sample_top_p", T.ptr(xd), 0, 1.0, 0.9, 0.5, T.ptr(out), S())
    with pytest.raises(T.TbError):  # larger than a 16-CTA cluster holds; rejected before any launch
        T.call("tb_sample_top_p", T.ptr(xd), 10**6, 1.0, 0.9, 0.5, T.ptr(out), S())


# ------------------------------------------------------------------ RoPE ----

@pytest.mark.parametrize("rank", [2, 4])
def test_rope_bit_exact(rank):
    hd, max_seq, theta, pos = 64, 256, 500000.0, 17
    c, s = O.rope_tables(hd, max_seq, theta)
    if rank == 2:
        S_ = 9
        shape, strides, n = (S_, hd), (hd, 1), S_ * hd
    else:
        B, S_, H = 1, 9, 32
        shape, strides, n = (B, H, S_, hd), (S_ * H * hd, hd, H * hd, 1), S_ * H * hd
    x = synth.normal((n,), 1.0, seed=20)
    dx = dev(x)
    T.call("tb_rope", T.byref(T.view(dx, 0, shape, strides)), T.ptr(dev(c)), T.ptr(dev(s)), hd, max_seq, pos, S())
    O.rope(x, 0, shape, strides, hd, max_seq, c, s, pos)
    assert_bits(host(dx), x)


def test_rope_kat_and_range():
    # reference test_rope.cpp: head_dim 4, max_seq 10, theta 10000, token 1
    c, s = O.rope_tables(4, 10, 10000.0)
    x = dev(np.array([[1, 2, 3, 4], [1, 2, 3, 4]], np.float32))
    T.call("tb_rope", T.byref(T.view(x)), T.ptr(dev(c)), T.ptr(dev(s)), 4, 10, 0, S())
    h = host(x)
    np.testing.assert_array_equal(h[0], [1, 2, 3, 4])
    assert abs(h[1, 0] - -1.9840) < 1e-3 and abs(h[1, 2] - 2.4623) < 1e-3
    with pytest.raises(T.TbError) as e:
        T.call("tb_rope", T.byref(T.view(x)), T.ptr(dev(c)), T.ptr(dev(s)), 4, 10, 9, S())
    assert e.value.status == T.ERANGE


# -------------------------------------------------------------- embedding ----

@pytest.mark.parametrize("dtype", [T.F32, T.Q8_0, T.Q4_0])
def test_embedding_bit_exact(dtype):
    dim, vocab = 2048, 1000
    w = synth.normal((vocab, dim), 0.02, seed=21)
    if dtype == T.F32:
        wb = np.ascontiguousarray(w.T).view(np.uint8).ravel()
    elif dtype == T.Q8_0:
        wb = synth.quantize_q8_0(w).ravel()
    else:
        wb = synth.quantize_q4_0(w).ravel()
    ids = np.array([0, 999, 5, 5, 123], np.int32)
    out = torch.empty((ids.size, dim), dtype=torch.float32, device="cuda")
    T.call("tb_embedding", dtype, T.ptr(dev(wb)), dim, vocab, T.ptr(dev(ids)), ids.size, T.ptr(out), S())
    assert_bits(host(out), O.embedding(wb, dtype, dim, vocab, ids.astype(np.float32)))
    assert T.take_device_errors() == 0
    bad = np.array([3, 1000], np.int32)
    out2 = torch.empty((2, dim), dtype=torch.float32, device="cuda")
    T.call("tb_embedding", dtype, T.ptr(dev(wb)), dim, vocab, T.ptr(dev(bad)), 2, T.ptr(out2), S())
    torch.cuda.synchronize()
    assert T.take_device_errors() & 2
    assert not out2[1].any()


# ------------------------------------------------- vocab-sharded (one GPU) ----

@pytest.mark.parametrize("shards", [2, 4, 8])
def test_sharded_softmax_and_argmax_emulated(shards):
    rows, V = 64, 128256
    x = synth.normal((rows, V), 2.0, seed=shards)
    x[3, 1000] = 50.0
    x[3, 90000] = 50.0  # tie across shards: first index wins
    dx = dev(x)
    w = V // shards
    maxes, sums, keys = [], [], []
    for g in range(shards):
        part = dx[:, g * w:(g + 1) * w]
        m = torch.empty(rows, device="cuda")
        s_ = torch.empty(rows, device="cuda")
        T.call("tb_softmax_shard_stats", part.data_ptr(), rows, w, V, T.ptr(m), T.ptr(s_), S())
        k = torch.empty(rows, dtype=torch.int64, device="cuda")
        T.call("tb_argmax_shard_keys", part.data_ptr(), rows, w, V, g * w, T.ptr(k), S())
        maxes.append(m)
        sums.append(s_)
        keys.append(k)
    gmax = torch.stack(maxes).max(0).values.contiguous()  # stands in for the max all-reduce
    for g in range(shards):
        T.call("tb_softmax_shard_rescale", T.ptr(maxes[g]), T.ptr(gmax), T.ptr(sums[g]), rows, S())
    gsum = torch.stack(sums).sum(0).contiguous()  # the sum all-reduce
    y = torch.empty_like(dx)
    for g in range(shards):
        T.call("tb_softmax_shard_finish", dx.data_ptr() + 4 * g * w, rows, w, V, T.ptr(gmax),
               T.ptr(gsum), y.data_ptr() + 4 * g * w, V, S())
    assert_softmax(host(y), x)
    kmax = torch.stack(keys).max(0).values  # stands in for the int64 MAX all-reduce
    idx = torch.empty(rows, dtype=torch.int64, device="cuda")
    T.call("tb_argmax_key_index", T.ptr(kmax.contiguous()), rows, T.ptr(idx), S())
    got = host(idx)
    for r in range(rows):
        assert got[r] == O.argmax(x[r]), r


# ------------------------------------------------ decode step (device position) ----

def _pos(p):
    return dev(np.array([p], np.int32))


def test_rope_at_matches_rope_and_checks_range():
    H, D, max_seq = 32, 64, 1024
    c, s_ = O.rope_tables(D, max_seq, 500000.0)
    dc, ds = dev(c), dev(s_)
    x = synth.normal((H * D,), 1.0, seed=40)
    a, b = dev(x), dev(x)
    va = T.view(a, 0, (1, H, 1, D), (H * D, D, H * D, 1))
    vb = T.view(b, 0, (1, H, 1, D), (H * D, D, H * D, 1))
    T.call("tb_rope", T.byref(va), T.ptr(dc), T.ptr(ds), D, max_seq, 517, S())
    T.call("tb_rope_at", T.byref(vb), T.ptr(dc), T.ptr(ds), D, max_seq, T.ptr(_pos(517)), S())
    assert_bits(host(b), host(a))
    assert T.take_device_errors() == 0
    c2 = dev(x)
    vc = T.view(c2, 0, (1, H, 1, D), (H * D, D, H * D, 1))
    T.call("tb_rope_at", T.byref(vc), T.ptr(dc), T.ptr(ds), D, max_seq, T.ptr(_pos(max_seq)), S())
    torch.cuda.synchronize()
    assert T.take_device_errors() & 2
    assert_bits(host(c2), x)  # left unchanged


def test_kv_append_and_range():
    row, max_seq = 8 * 64, 40
    kc = torch.zeros(max_seq * row, device="cuda")
    vc = torch.zeros(max_seq * row, device="cuda")
    k = synth.normal((row,), 1.0, seed=41)
    v = synth.normal((row,), 1.0, seed=42)
    T.call("tb_kv_append", T.ptr(kc), T.ptr(vc), T.ptr(dev(k)), T.ptr(dev(v)), row, max_seq, T.ptr(_pos(7)), S())
    hk, hv = host(kc).reshape(max_seq, row), host(vc).reshape(max_seq, row)
    assert_bits(hk[7], k)
    assert_bits(hv[7], v)
    assert not hk[:7].any() and not hk[8:].any()
    T.call("tb_kv_append", T.ptr(kc), T.ptr(vc), T.ptr(dev(k)), T.ptr(dev(v)), row, max_seq, T.ptr(_pos(max_seq)), S())
    torch.cuda.synchronize()
    assert T.take_device_errors() & 2
    assert np.count_nonzero(host(kc)) == np.count_nonzero(hk)


@pytest.mark.parametrize("pos", [0, 1, 255, 640, 1023])
def test_attention_decode_against_float64(pos):
    H, KVH, D, max_seq = 32, 8, 64, 1024
    q = synth.normal((H, D), 1.0, seed=pos)
    kc = synth.normal((max_seq, KVH, D), 1.0, seed=pos + 1)
    vc = synth.normal((max_seq, KVH, D), 1.0, seed=pos + 2)
    out = torch.empty((H, D), device="cuda")
    scale = np.float32(1.0) / np.sqrt(np.float32(D))
    T.call("tb_attention_decode", T.ptr(dev(q)), T.ptr(dev(kc)), T.ptr(dev(vc)), H, KVH, D, max_seq,
           float(scale), T.ptr(_pos(pos)), T.ptr(out), S())
    got = host(out)
    ctx = pos + 1
    want = np.empty((H, D))
    for h in range(H):
        kh = kc[:ctx, h // (H // KVH)].astype(np.float64)
        vh = vc[:ctx, h // (H // KVH)].astype(np.float64)
        s = (kh @ q[h].astype(np.float64)) * float(scale)
        p = np.exp(s - s.max())
        p /= p.sum()
        want[h] = p @ vh
    # per output: |err| <= 1e-5 * sum_c p_c |v_c| (the conditioning of p . V)
    cond = np.empty((H, D))
    for h in range(H):
        kh = kc[:ctx, h // (H // KVH)].astype(np.float64)
        s = (kh @ q[h].astype(np.float64)) * float(scale)
        p = np.exp(s - s.max())
        p /= p.sum()
        cond[h] = p @ np.abs(vc[:ctx, h // (H // KVH)].astype(np.float64))
    assert (np.abs(got - want) / cond).max() <= F32_REL


def test_decode_margin_and_advance():
    V, max_seq = 1000, 16
    logits = synth.normal((V,), 1.0, seed=43)
    logits[123] = 9.0
    logits[7] = 8.5
    dl = dev(logits)
    idx = torch.empty(1, dtype=torch.int64, device="cuda")
    T.call("tb_argmax", T.ptr(dl), 1, V, T.ptr(idx), S())
    pos = _pos(5)
    margins = torch.zeros(max_seq, device="cuda")
    ids = torch.zeros(1, dtype=torch.int32, device="cuda")
    hist = torch.zeros(max_seq, dtype=torch.int32, device="cuda")
    T.call("tb_decode_margin", T.ptr(dl), V, T.ptr(idx), T.ptr(pos), max_seq, T.ptr(margins), S())
    T.call("tb_decode_advance", T.ptr(idx), T.ptr(ids), T.ptr(pos), T.ptr(hist), max_seq, S())
    assert host(margins)[5] == np.float32(9.0) - np.float32(8.5)
    assert host(ids)[0] == 123 and host(hist)[5] == 123 and host(pos)[0] == 6


def test_graph_capture_and_replay():
    st = ctypes.c_void_p()
    T.call("tb_stream_create", ctypes.byref(st))
    x = dev(synth.normal((4096,), 1.0, seed=44))
    y = torch.empty(4096, device="cuda")
    vx, vy = T.view(x), T.view(y)
    g = ctypes.c_void_p()
    T.call("tb_capture_begin", st)
    T.call("tb_scale", T.byref(vx), 2.0, T.byref(vy), st)
    T.call("tb_binary", 0, T.byref(vy), T.byref(vx), T.byref(vy), st)
    T.call("tb_capture_end", st, ctypes.byref(g))
    for _ in range(3):
        T.call("tb_graph_launch", g, st)
    T.call("tb_sync", st)
    xs = host(x)
    assert_bits(host(y), xs * np.float32(2.0) + xs)
    T.call("tb_graph_destroy", g)
    T.call("tb_stream_destroy", st)


# --------------------------------------------------- fused decode-step GEMVs ----

def _q8_dev(N, K, seed):
    wq = synth.quantize_q8_0(synth.normal((N, K), 0.02, seed=seed))
    return wq, dev(wq)


@pytest.mark.parametrize("sizes,K", [((2048, 512, 512), 2048), ((37, 100, 5), 256), ((300,), 8192), ((2048,), 8192)])
def test_gemv_multi_segments_and_residual(sizes, K):
    # each segment within tolerance of the oracle; the residual epilogue is
    # exactly tb_binary(add) of the residual and the plain product
    xh = synth.normal((K,), 1.0, seed=K)
    x = dev(xh)
    plain, fused, refs, res, wqs = [], [], [], [], []
    for i, n in enumerate(sizes):
        wq, dw = _q8_dev(n, K, seed=n + i)
        wqs.append((wq, dw))
        plain.append(torch.empty(n, device="cuda"))
        fused.append(torch.empty(n, device="cuda"))
        res.append(dev(synth.normal((n,), 1.0, seed=i)) if i == 0 else None)
    seg0 = (T.GemvSegment * len(sizes))(*[T.GemvSegment(dw.data_ptr(), n, y.data_ptr(), None)
                                          for (wq, dw), n, y in zip(wqs, sizes, plain)])
    seg1 = (T.GemvSegment * len(sizes))(*[T.GemvSegment(dw.data_ptr(), n, y.data_ptr(),
                                                        r.data_ptr() if r is not None else None)
                                          for (wq, dw), n, y, r in zip(wqs, sizes, fused, res)])
    T.call("tb_gemv_q8_0_multi", T.ptr(x), K, None, 0.0, ctypes.cast(seg0, ctypes.c_void_p), len(sizes), S())
    T.call("tb_gemv_q8_0_multi", T.ptr(x), K, None, 0.0, ctypes.cast(seg1, ctypes.c_void_p), len(sizes), S())
    for i, n in enumerate(sizes):
        assert_dot_tol(host(plain[i]).reshape(1, n), xh.reshape(1, K), wqs[i][0], K)
        if res[i] is None:
            assert_bits(host(fused[i]), host(plain[i]))
        else:
            out = torch.empty(n, device="cuda")
            T.call("tb_binary", 0, T.byref(T.view(res[i])), T.byref(T.view(plain[i])), T.byref(T.view(out)), S())
            assert_bits(host(fused[i]), host(out))


@pytest.mark.parametrize("N,K", [(40000, 2048), (1, 2048), (5, 256), (1024, 16384), (3000, 4096)])
def test_gemv_stream_ring_multipass_and_tiny(N, K):
    # 40000 x 2048 through tb_gemv_q8_0_multi runs the span buffers as a ring
    # (more spans per CTA than buffers); K = 16384 and 4096 take several
    # 64-block passes per row and fewer CTAs per SM; 1 and 5 rows leave most
    # warps without a row
    xh = synth.normal((K,), 1.0, seed=K + N)
    x = dev(xh)
    wq, dw = _q8_dev(N, K, seed=N)
    y = torch.empty(N, device="cuda")
    seg = (T.GemvSegment * 1)(T.GemvSegment(dw.data_ptr(), N, y.data_ptr(), None))
    T.call("tb_gemv_q8_0_multi", T.ptr(x), K, None, 0.0, ctypes.cast(seg, ctypes.c_void_p), 1, S())
    assert_dot_tol(host(y).reshape(1, N), xh.reshape(1, K), wq, K)
    if N < 32768:  # tb_matmul_quant's M = 1 path below the tensor-core size is the same kernel
        y2 = torch.empty(N, device="cuda")
        T.call("tb_matmul_quant", T.Q8_0, T.ptr(x), 1, K, T.ptr(dw), N, T.ptr(y2), S())
        assert_bits(host(y2), host(y))


def test_prefetch_l2_is_only_a_hint():
    K, N = 2048, 4096
    xh = synth.normal((K,), 1.0, seed=77)
    x = dev(xh)
    wq, dw = _q8_dev(N, K, seed=78)
    y0, y1 = torch.empty(N, device="cuda"), torch.empty(N, device="cuda")
    T.call("tb_matmul_quant", T.Q8_0, T.ptr(x), 1, K, T.ptr(dw), N, T.ptr(y0), S())
    # ranges trimmed inward to 16 bytes (an unaligned start, a ragged end, one
    # range shorter than 16 bytes, a null pointer) are accepted
    base = dw.data_ptr()
    ptrs = (ctypes.c_void_p * 4)(base + 3, base, base + 5, None)
    sizes = (ctypes.c_int64 * 4)(dw.numel() - 3, 1000, 7, 64)
    T.call("tb_prefetch_l2", ctypes.cast(ptrs, ctypes.c_void_p), ctypes.cast(sizes, ctypes.c_void_p), 4, S())
    T.call("tb_prefetch_l2", None, None, 0, S())
    T.call("tb_matmul_quant", T.Q8_0, T.ptr(x), 1, K, T.ptr(dw), N, T.ptr(y1), S())
    assert_bits(host(y1), host(y0))
    ptrs9 = (ctypes.c_void_p * 9)(*([base] * 9))
    sizes9 = (ctypes.c_int64 * 9)(*([64] * 9))
    with pytest.raises(T.TbError) as e:
        T.call("tb_prefetch_l2", ctypes.cast(ptrs9, ctypes.c_void_p), ctypes.cast(sizes9, ctypes.c_void_p), 9, S())
    assert e.value.status == T.EINVAL


@pytest.mark.parametrize("K,N", [(2048, 3072), (8192, 2048), (16384, 600)])
def test_gemv_multi_with_rmsnorm_within_tolerance(K, N):
    # K = 8192 and 16384 take the split-K form (x normalised while loaded
    # into registers, one or two passes per warp)
    xh = synth.normal((K,), 1.0, seed=50)
    g = synth.uniform((K,), 0.5, 1.5, seed=51)
    wq, dw = _q8_dev(N, K, seed=52)
    x, dg = dev(xh), dev(g)
    y = torch.empty(N, device="cuda")
    seg = (T.GemvSegment * 1)(T.GemvSegment(dw.data_ptr(), N, y.data_ptr(), None))
    T.call("tb_gemv_q8_0_multi", T.ptr(x), K, T.ptr(dg), 1e-5, ctypes.cast(seg, ctypes.c_void_p), 1, S())
    xn = O.rmsnorm(xh.reshape(1, K), g)
    assert_dot_tol(host(y).reshape(1, N), xn, wq, K)


def test_gemv_swiglu_within_tolerance_with_and_without_norm():
    K, N = 2048, 8192
    xh = synth.normal((K,), 1.0, seed=53)
    x = dev(xh)
    wg, dg = _q8_dev(N, K, seed=54)
    wu, du = _q8_dev(N, K, seed=55)
    y = torch.empty(N, device="cuda")
    for gam in (None, synth.uniform((K,), 0.5, 1.5, seed=56)):
        _check_swiglu(xh, x, gam, wg, dg, wu, du, y, K, N)


def _check_swiglu(xh, x, gam, wg, dg, wu, du, y, K, N):
    gp = T.ptr(dev(gam)) if gam is not None else None
    T.call("tb_gemv_q8_0_swiglu", T.ptr(x), K, gp, 1e-5, T.ptr(dg), T.ptr(du), N, T.ptr(y), S())
    xn = O.rmsnorm(xh.reshape(1, K), gam) if gam is not None else xh.reshape(1, K)
    g_ref, u_ref = O.matmul_q8_0(xn, wg, N)[0], O.matmul_q8_0(xn, wu, N)[0]
    want = O.swiglu(g_ref, u_ref)
    # g and u are each within 1e-5 of their sum |w x|; propagate through
    # y = silu(g) * u (|d silu / dg| <= 1.1)
    xa = np.abs(xn[0].astype(np.float64))
    sg = np.abs(synth.dequantize_q8_0(wg, K)).astype(np.float64) @ xa
    su = np.abs(synth.dequantize_q8_0(wu, K)).astype(np.float64) @ xa
    silu = np.abs(g_ref.astype(np.float64)) / (1 + np.exp(-g_ref.astype(np.float64)))
    bound = F32_REL * (1.1 * np.abs(u_ref) * sg + silu * su) + 1e-30
    assert (np.abs(host(y).astype(np.float64) - want) / bound).max() <= 1.0


def test_rope_kv_append_equals_separate_ops():
    H, KVH, D, max_seq = 32, 8, 64, 1024
    c, s_ = O.rope_tables(D, max_seq, 500000.0)
    dc, ds = dev(c), dev(s_)
    qh = synth.normal((H * D,), 1.0, seed=57)
    kh = synth.normal((KVH * D,), 1.0, seed=58)
    vh = synth.normal((KVH * D,), 1.0, seed=59)
    pos = _pos(300)
    q1, k1, v1 = dev(qh), dev(kh), dev(vh)
    kc1, vc1 = torch.zeros(max_seq * KVH * D, device="cuda"), torch.zeros(max_seq * KVH * D, device="cuda")
    T.call("tb_rope_kv_append", T.ptr(q1), T.ptr(k1), T.ptr(v1), H, KVH, D, T.ptr(dc), T.ptr(ds), max_seq,
           T.ptr(kc1), T.ptr(vc1), max_seq, T.ptr(pos), S())
    q2, k2, v2 = dev(qh), dev(kh), dev(vh)
    kc2, vc2 = torch.zeros_like(kc1), torch.zeros_like(vc1)
    vq = T.view(q2, 0, (1, H, 1, D), (H * D, D, H * D, 1))
    vk = T.view(k2, 0, (1, KVH, 1, D), (KVH * D, D, KVH * D, 1))
    T.call("tb_rope_at", T.byref(vq), T.ptr(dc), T.ptr(ds), D, max_seq, T.ptr(pos), S())
    T.call("tb_rope_at", T.byref(vk), T.ptr(dc), T.ptr(ds), D, max_seq, T.ptr(pos), S())
    T.call("tb_kv_append", T.ptr(kc2), T.ptr(vc2), T.ptr(k2), T.ptr(v2), KVH * D, max_seq, T.ptr(pos), S())
    for a, b in ((q1, q2), (k1, k2), (kc1, kc2), (vc1, vc2)):
        assert_bits(host(a), host(b))
    assert T.take_device_errors() == 0


@pytest.mark.parametrize("p", [0, 1, 300, 1023])
def test_rope_attention_decode_equals_separate_ops(p):
    # tb_rope_attention_decode == tb_rope_kv_append then tb_attention_decode,
    # bit for bit: the output and both caches (the prefix rows random, so the
    # new row is not the only one that counts); q, k, v are left unchanged
    H, KVH, D, max_seq = 32, 8, 64, 1024
    c, s_ = O.rope_tables(D, max_seq, 500000.0)
    dc, ds = dev(c), dev(s_)
    qh = synth.normal((H * D,), 1.0, seed=60 + p)
    kh = synth.normal((KVH * D,), 1.0, seed=61 + p)
    vh = synth.normal((KVH * D,), 1.0, seed=62 + p)
    prefix_k = synth.normal((max_seq * KVH * D,), 1.0, seed=63)
    prefix_v = synth.normal((max_seq * KVH * D,), 1.0, seed=64)
    pos = _pos(p)
    scale = 1.0 / 8.0
    q1, k1, v1 = dev(qh), dev(kh), dev(vh)
    kc1, vc1 = dev(prefix_k), dev(prefix_v)
    out1 = torch.empty(H * D, device="cuda")
    T.call("tb_rope_kv_append", T.ptr(q1), T.ptr(k1), T.ptr(v1), H, KVH, D, T.ptr(dc), T.ptr(ds), max_seq,
           T.ptr(kc1), T.ptr(vc1), max_seq, T.ptr(pos), S())
    T.call("tb_attention_decode", T.ptr(q1), T.ptr(kc1), T.ptr(vc1), H, KVH, D, max_seq, scale, T.ptr(pos),
           T.ptr(out1), S())
    q2, k2, v2 = dev(qh), dev(kh), dev(vh)
    kc2, vc2 = dev(prefix_k), dev(prefix_v)
    out2 = torch.empty(H * D, device="cuda")
    T.call("tb_rope_attention_decode", T.ptr(q2), T.ptr(k2), T.ptr(v2), H, KVH, D, T.ptr(dc), T.ptr(ds), max_seq,
           T.ptr(kc2), T.ptr(vc2), max_seq, scale, T.ptr(pos), T.ptr(out2), S())
    for a, b in ((out1, out2), (kc1, kc2), (vc1, vc2)):
        assert_bits(host(a), host(b))
    for t, h_ in ((q2, qh), (k2, kh), (v2, vh)):
        assert_bits(host(t), h_)
    assert T.take_device_errors() == 0
    # a position outside the RoPE table is refused on the device: error bit, caches untouched
    bad = _pos(max_seq)
    T.call("tb_rope_attention_decode", T.ptr(q2), T.ptr(k2), T.ptr(v2), H, KVH, D, T.ptr(dc), T.ptr(ds), max_seq,
           T.ptr(kc2), T.ptr(vc2), max_seq, scale, T.ptr(bad), T.ptr(out2), S())
    assert T.take_device_errors() & 2
    assert_bits(host(kc2), host(kc1))


# ---- causal GQA prefill attention (attention.cpp:104-141, all heads at once) ------
def attention_ref(q, kc, vc, S, pos0, H, KVH, D, scale):
    """float64 causal attention and, per output, sum_t p_t |v_t| (the scale of
    its rounding error)."""
    G = H // KVH
    out = np.zeros((S, H * D))
    mag = np.zeros((S, H * D))
    for h in range(H):
        kvh = h // G
        qh = q[:, h * D:(h + 1) * D].astype(np.float64)
        K = kc[:pos0 + S, kvh * D:(kvh + 1) * D].astype(np.float64)
        V = vc[:pos0 + S, kvh * D:(kvh + 1) * D].astype(np.float64)
        sc = (qh @ K.T) * scale
        mask = np.arange(pos0 + S)[None, :] > (pos0 + np.arange(S))[:, None]
        sc[mask] = -np.inf
        p = np.exp(sc - sc.max(axis=1, keepdims=True))
        p /= p.sum(axis=1, keepdims=True)
        out[:, h * D:(h + 1) * D] = p @ V
        mag[:, h * D:(h + 1) * D] = p @ np.abs(V)
    return out, mag


@pytest.mark.parametrize("n,pos0,H,KVH", [(512, 0, 32, 8), (37, 100, 32, 8), (1, 600, 32, 8), (200, 0, 8, 8),
                                          (64, 1200, 32, 8), (100, 1900, 32, 8)])
def test_attention_prefill(n, pos0, H, KVH):
    D, max_seq = 64, 2048
    q = synth.normal((n, H * D), 1.0, seed=n + pos0)
    kc = synth.normal((max_seq, KVH * D), 1.0, seed=7)
    vc = synth.normal((max_seq, KVH * D), 1.0, seed=8)
    scale = np.float32(1.0 / np.sqrt(D))
    out = torch.full((n, H * D), float("nan"), dtype=torch.float32, device="cuda")
    T.call("tb_attention_prefill", T.ptr(dev(q)), H * D, T.ptr(dev(kc)), T.ptr(dev(vc)), n, pos0, H, KVH, D,
           float(scale), T.ptr(out), H * D, S())
    ref, mag = attention_ref(q, kc, vc, n, pos0, H, KVH, D, float(scale))
    got = host(out).astype(np.float64)
    err = np.abs(got - ref) / np.maximum(mag, 1e-30)
    assert err.max() <= 1e-5, err.max()

"""tb_matmul_q4_0_static_scratch: the Q4_0 matmul for callers that cannot
allocate device memory during a call -- a serving process that reserves its
whole device-memory budget at start-up and may not grow it per request, or a
latency-critical loop in which an allocator call could synchronize or fail.

It keeps the quantized copy of X in a fixed buffer compiled into the library
instead of scratch from the allocator.  Its output must equal the regular
bit-exact entry point's (tb_matmul_quant_exact, TB_Q4_0) bit for bit -- the
tolerance the Q4_0 tests use -- on two calls in a row, so that whatever the
first call left in the shared buffer cannot leak into the second; a sample of
the prefill shape's rows is also compared with the oracle directly, and below
32 rows it equals tb_matmul_quant (which takes the tensor cores from 32 rows
on).  This file is named to be collected last; it passes alone in a fresh
process as well.
"""
import os

import numpy as np
import pytest

from oracle import orbind as O
from turbo_b200 import synth

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import turbo_b200 as T  # noqa: E402


def _dev(a, keep):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    keep.append(t)
    return t


def test_static_scratch_matches_regular_entry_two_calls():
    T.call("tb_init", 0)
    s = T.stream_handle()
    keep = []
    cases = [(512, 8192, 2048, 11), (7, 2048, 515, 12)]  # the prefill shape, then a small one
    for i, (M, K, N, seed) in enumerate(cases):
        wq = synth.quantize_q4_0(synth.normal((N, K), 0.02, seed=seed))
        x = synth.normal((M, K), 1.0, seed=seed + 100)
        dx, dw = _dev(x, keep), _dev(wq, keep)
        y_reg = torch.empty((M, N), dtype=torch.float32, device="cuda")
        y_fix = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
        T.call("tb_matmul_quant_exact", T.Q4_0, T.ptr(dx), M, K, T.ptr(dw), N, T.ptr(y_reg), s)
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        T.call("tb_matmul_q4_0_static_scratch", T.ptr(dx), M, K, T.ptr(dw), N, T.ptr(y_fix), s)
        torch.cuda.synchronize()
        # After the first call (which may load the library's module that holds
        # the buffer), a call takes no device memory from the driver.
        if i > 0:
            assert torch.cuda.mem_get_info()[0] == free_before, (M, K, N)
        a = y_reg.cpu().numpy()
        b = y_fix.cpu().numpy()
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), (M, K, N)
        rows = np.unique(np.linspace(0, M - 1, min(M, 24)).astype(int))
        ref = O.matmul_q4_0(x[rows], wq, N, threads=os.cpu_count() or 1)
        assert np.array_equal(b[rows].view(np.uint32), ref.view(np.uint32)), (M, K, N)
        if M < 32:
            y_def = torch.empty((M, N), dtype=torch.float32, device="cuda")
            T.call("tb_matmul_quant", T.Q4_0, T.ptr(dx), M, K, T.ptr(dw), N, T.ptr(y_def), s)
            torch.cuda.synchronize()
            assert np.array_equal(y_def.cpu().numpy().view(np.uint32), b.view(np.uint32)), (M, K, N)
    assert T.take_device_errors() == 0


def test_static_scratch_reports_a_wait_that_gave_up():
    # With no waiting allowed (wait limit 0) the kernel's bounded wait gives up:
    # the output stays unwritten and the entry point's own error word says so
    # through tb_take_device_errors; with the default limit the next call is
    # exact again.
    T.call("tb_init", 0)
    s = T.stream_handle()
    keep = []
    M, K, N = 5, 2048, 260
    wq = synth.quantize_q4_0(synth.normal((N, K), 0.02, seed=21))
    x = synth.normal((M, K), 1.0, seed=22)
    dx, dw = _dev(x, keep), _dev(wq, keep)
    y = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    assert T.take_device_errors() == 0
    T.call("tb_set_wait_limit_ns", 0)
    try:
        T.call("tb_matmul_q4_0_static_scratch", T.ptr(dx), M, K, T.ptr(dw), N, T.ptr(y), s)
        torch.cuda.synchronize()
    finally:
        T.call("tb_set_wait_limit_ns", 2000000000)
    assert T.take_device_errors() & 1
    assert np.isnan(y.cpu().numpy()).all()
    T.call("tb_matmul_q4_0_static_scratch", T.ptr(dx), M, K, T.ptr(dw), N, T.ptr(y), s)
    torch.cuda.synchronize()
    ref = O.matmul_q4_0(x, wq, N)
    assert np.array_equal(y.cpu().numpy().view(np.uint32), ref.view(np.uint32))
    assert T.take_device_errors() == 0


def test_static_scratch_rejects_oversize():
    T.call("tb_init", 0)
    x = torch.zeros((1, 32), device="cuda")
    M, K = 1024, 8192  # 8.5 MiB of Q8_0 scratch: above the fixed 8 MiB
    with pytest.raises(T.TbError) as e:
        T.call("tb_matmul_q4_0_static_scratch", T.ptr(x), M, K, T.ptr(x), 1, T.ptr(x), T.stream_handle())
    assert e.value.status == T.EINVAL
    assert "8388608-byte buffer" in str(e.value)

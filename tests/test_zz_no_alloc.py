"""tb_matmul_q4_0_static_scratch: the Q4_0 matmul for callers that cannot
allocate device memory during a call.

It keeps the quantized copy of X in a fixed buffer compiled into the library
instead of scratch from the allocator.  Its output must equal the regular
bit-exact entry point's (tb_matmul_quant_exact, TB_Q4_0) bit for bit -- the
tolerance the Q4_0 tests use -- on two calls in a row, so that whatever the
first call left in the shared buffer cannot leak into the second; below 32 rows
it also equals tb_matmul_quant (which takes the tensor cores from 32 rows on).
This file is named to be collected last; it passes alone in a fresh process as
well.
"""
import numpy as np
import pytest

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
    for M, K, N, seed in cases:
        wq = synth.quantize_q4_0(synth.normal((N, K), 0.02, seed=seed))
        x = synth.normal((M, K), 1.0, seed=seed + 100)
        dx, dw = _dev(x, keep), _dev(wq, keep)
        y_reg = torch.empty((M, N), dtype=torch.float32, device="cuda")
        y_fix = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
        T.call("tb_matmul_quant_exact", T.Q4_0, T.ptr(dx), M, K, T.ptr(dw), N, T.ptr(y_reg), s)
        T.call("tb_matmul_q4_0_static_scratch", T.ptr(dx), M, K, T.ptr(dw), N, T.ptr(y_fix), s)
        torch.cuda.synchronize()
        a = y_reg.cpu().numpy()
        b = y_fix.cpu().numpy()
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), (M, K, N)
        if M < 32:
            y_def = torch.empty((M, N), dtype=torch.float32, device="cuda")
            T.call("tb_matmul_quant", T.Q4_0, T.ptr(dx), M, K, T.ptr(dw), N, T.ptr(y_def), s)
            torch.cuda.synchronize()
            assert np.array_equal(y_def.cpu().numpy().view(np.uint32), b.view(np.uint32)), (M, K, N)


def test_static_scratch_rejects_oversize():
    T.call("tb_init", 0)
    x = torch.zeros((1, 32), device="cuda")
    M, K = 1024, 8192  # 8.5 MiB of Q8_0 scratch: above the fixed 8 MiB
    with pytest.raises(T.TbError) as e:
        T.call("tb_matmul_q4_0_static_scratch", T.ptr(x), M, K, T.ptr(x), 1, T.ptr(x), T.stream_handle())
    assert e.value.status == T.EINVAL
    assert "8388608-byte buffer" in str(e.value)

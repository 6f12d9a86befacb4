"""The vocab-sharded softmax/argmax and the tensor-parallel Q8_0 GEMV over
NCCL on two GPUs (one process per GPU), with the per-shard halves as the CUDA
kernels: turbo_b200.sharded on [64, 128256] logits, a row-split 8192 x 2048
GEMV and a vocab-split 128256 x 2048 LM head feeding the sharded argmax,
against the oracle's single-process results.  Skipped on machines with fewer
than two GPUs."""
import ctypes
import os
import socket
import sys
from datetime import timedelta

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, rows, vocab):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "turbo.cpp_b200", "python"))
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method="tcp://127.0.0.1:%d" % port, rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=torch.device("cuda", rank))
    try:
        import turbo_b200 as T
        from oracle import orbind as O
        from turbo_b200 import synth
        from turbo_b200.sharded import VocabShardGroup
        T.call("tb_init", rank)
        x = synth.normal((rows, vocab), 2.0, seed=7)
        x[5, 17] = 40.0
        x[5, vocab - 2] = 40.0  # a tie across the shards
        g = VocabShardGroup(vocab)
        local = torch.from_numpy(np.ascontiguousarray(x[:, g.col_base:g.col_base + g.cols])).cuda()
        idx = g.argmax(local).cpu().numpy()
        y = g.softmax(local).cpu().numpy()
        for r in range(rows):
            assert idx[r] == O.argmax(x[r]), (rank, r)
        a = x.astype(np.float64)
        e = np.exp(a - a.max(axis=1, keepdims=True))
        want = (e / e.sum(axis=1, keepdims=True))[:, g.col_base:g.col_base + g.cols]
        assert np.max(np.abs(y - want) / np.maximum(want, want.max() * 1e-3)) <= 1e-5
        assert T.take_device_errors() == 0
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_vocab_sharded_nccl_two_gpus():
    mp.start_processes(_rank, args=(2, _free_port(), 64, 128256), nprocs=2, join=True, start_method="spawn")


def _tp_rank(rank, world, port):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "turbo.cpp_b200", "python"))
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method="tcp://127.0.0.1:%d" % port, rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=torch.device("cuda", rank))
    try:
        import turbo_b200 as T
        from oracle import orbind as O
        from turbo_b200 import synth
        from turbo_b200.sharded import RowShardedGemv, VocabShardGroup
        T.call("tb_init", rank)
        N, K, V = 8192, 2048, 128256
        wq = synth.quantize_q8_0(synth.normal((N, K), 0.02, seed=31))
        xh = synth.normal((K,), 1.0, seed=32)
        x = torch.from_numpy(xh).cuda()
        tp = RowShardedGemv(N, K)
        w_local = tp.local_rows(torch.from_numpy(wq.ravel())).cuda()
        y = tp(x, w_local).cpu().numpy()
        ref = O.matmul_q8_0(xh.reshape(1, K), wq, N)[0].astype(np.float64)
        scale = np.abs(synth.dequantize_q8_0(wq, K)).astype(np.float64) @ np.abs(xh).astype(np.float64)
        assert np.max(np.abs(y - ref) / scale) <= 1e-5
        # vocab-split LM head -> sharded argmax == argmax of the full product on one GPU
        wl = synth.quantize_q8_0(synth.normal((V, K), 0.02, seed=33))
        g = VocabShardGroup(V)
        rb = K // 32 * 34
        mine = torch.from_numpy(wl.ravel()[g.col_base * rb:(g.col_base + g.cols) * rb].copy()).cuda()
        logits = torch.empty((1, g.cols), dtype=torch.float32, device="cuda")
        T.call("tb_matmul_quant", T.Q8_0, T.ptr(x), 1, K, T.ptr(mine), g.cols, T.ptr(logits),
               ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        idx = int(g.argmax(logits)[0])
        wl_d = torch.from_numpy(wl.ravel()).cuda()
        full = torch.empty((1, V), dtype=torch.float32, device="cuda")
        T.call("tb_matmul_quant", T.Q8_0, T.ptr(x), 1, K, T.ptr(wl_d), V, T.ptr(full),
               ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        assert idx == O.argmax(full.cpu().numpy()[0])
        assert T.take_device_errors() == 0
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_tensor_parallel_gemv_nccl_two_gpus():
    mp.start_processes(_tp_rank, args=(2, _free_port()), nprocs=2, join=True, start_method="spawn")


# ---- the same protocol through the C ABI (tb_shard_group_*), as a C++ host
# would call it: no torch.distributed on the path

def _abi_case(T, O, synth, group, rank, world, stream, rows=64, vocab=128256):
    """softmax and argmax of [rows, vocab] logits split by columns, and the
    row-split GEMV, on this rank's shard, against the oracle."""
    _vocab_case(T, O, synth, group, rank, world, stream, rows, vocab)
    _gemv_case(T, O, synth, group, rank, world, stream)


def _vocab_case(T, O, synth, group, rank, world, stream, rows=64, vocab=128256, seed=7):
    """softmax and argmax of [rows, vocab] logits split by columns against the
    oracle: a tie across the shards, a row without candidates."""
    x = synth.normal((rows, vocab), 2.0, seed=seed)
    x[5, 17] = 40.0
    x[5, vocab - 2] = 40.0  # a tie across the shards
    x[9, :] = -np.inf       # no candidate: index 0
    base, cols = rank * vocab // world, (rank + 1) * vocab // world - rank * vocab // world
    local = torch.from_numpy(np.ascontiguousarray(x[:, base:base + cols])).cuda()
    y = torch.empty_like(local)
    idx = torch.empty(rows, dtype=torch.int64, device="cuda")
    T.call("tb_argmax_vocab_sharded", group, T.ptr(local), rows, cols, cols, base, T.ptr(idx), stream)
    x[9, :] = 0.0  # the softmax check uses a row with finite values
    local[9].zero_()
    T.call("tb_softmax_vocab_sharded", group, T.ptr(local), rows, cols, cols, T.ptr(y), cols, stream)
    T.call("tb_shard_group_wait", group, stream, 30.0)
    idx = idx.cpu().numpy()
    x9 = x.copy()
    x9[9, :] = -np.inf
    for r in range(rows):
        assert idx[r] == O.argmax(x9[r]), (rank, r, idx[r])
    a = x.astype(np.float64)
    e = np.exp(a - a.max(axis=1, keepdims=True))
    want = (e / e.sum(axis=1, keepdims=True))[:, base:base + cols]
    got = y.cpu().numpy()
    assert np.max(np.abs(got - want) / np.maximum(want, want.max() * 1e-3)) <= 1e-5
    assert T.take_device_errors() == 0


def _gemv_case(T, O, synth, group, rank, world, stream):
    """the row-split Q8_0 GEMV, 8192 x 2048, against the oracle"""
    N, K = 8192, 2048
    wq = synth.quantize_q8_0(synth.normal((N, K), 0.02, seed=31))
    xh = synth.normal((K,), 1.0, seed=32)
    n_local = N // world
    rb = K // 32 * 34
    w_local = torch.from_numpy(wq.ravel()[rank * n_local * rb:(rank + 1) * n_local * rb].copy()).cuda()
    xd = torch.from_numpy(xh).cuda()
    yv = torch.empty(N, dtype=torch.float32, device="cuda")
    T.call("tb_gemv_q8_0_row_sharded", group, T.ptr(xd), K, T.ptr(w_local), n_local, T.ptr(yv), stream)
    T.call("tb_shard_group_wait", group, stream, 30.0)
    ref = O.matmul_q8_0(xh.reshape(1, K), wq, N)[0].astype(np.float64)
    scale = np.abs(synth.dequantize_q8_0(wq, K)).astype(np.float64) @ np.abs(xh).astype(np.float64)
    assert np.max(np.abs(yv.cpu().numpy() - ref) / scale) <= 1e-5
    assert T.take_device_errors() == 0


def _q8_scale(wq, xh, N, K):
    """sum_k |w_nk x_k| per row, in chunks of rows (the tolerance's scale)."""
    from turbo_b200 import synth
    out = np.empty(N)
    rb = K // 32 * 34
    flat = wq.reshape(-1)
    for r0 in range(0, N, 8192):
        r1 = min(N, r0 + 8192)
        wd = synth.dequantize_q8_0(flat[r0 * rb:r1 * rb].reshape(r1 - r0, rb), K).astype(np.float64)
        out[r0:r1] = np.abs(wd) @ np.abs(xh).astype(np.float64)
    return out


def _peer_case(T, O, synth, group, rank, world, stream):
    """The row-split GEMV with the rows exchanged by NVLink peer stores
    (tb_shard_group_enable_peer): the decode projections' shapes and the
    vocabulary-sized LM head (tensor-core GEMV per shard), several calls so
    that both exchange buffers are used, each against the oracle; between
    them the vocab-sharded softmax and argmax, whose (m, s) pairs and keys
    take the same exchange (and its call numbers)."""
    T.call("tb_shard_group_enable_peer", group, 128256)
    _vocab_case(T, O, synth, group, rank, world, stream, seed=8)
    for i, (N, K) in enumerate([(8192, 2048), (2048, 8192), (8192, 2048), (128256, 2048), (2048, 8192)]):
        wq = synth.quantize_q8_0(synth.normal((N, K), 0.02, seed=40 + i))
        xh = synth.normal((K,), 1.0, seed=50 + i)
        n_local = N // world
        rb = K // 32 * 34
        w_local = torch.from_numpy(wq.ravel()[rank * n_local * rb:(rank + 1) * n_local * rb].copy()).cuda()
        xd = torch.from_numpy(xh).cuda()
        yv = torch.full((N,), float("nan"), dtype=torch.float32, device="cuda")
        T.call("tb_gemv_q8_0_row_sharded", group, T.ptr(xd), K, T.ptr(w_local), n_local, T.ptr(yv), stream)
        T.call("tb_shard_group_wait", group, stream, 30.0)
        assert T.take_device_errors() == 0, (rank, N, K)
        ref = O.matmul_q8_0(xh.reshape(1, K), wq, N)[0].astype(np.float64)
        got = yv.cpu().numpy()
        assert not np.isnan(got).any(), (rank, N, K)
        assert np.max(np.abs(got - ref) / _q8_scale(wq, xh, N, K)) <= 1e-5, (rank, N, K)
        if i == 1:
            _vocab_case(T, O, synth, group, rank, world, stream, rows=13, seed=9)


def test_shard_group_abi_one_rank():
    import turbo_b200 as T
    from oracle import orbind as O
    from turbo_b200 import synth
    T.call("tb_init", 0)
    uid = ctypes.create_string_buffer(128)
    T.call("tb_shard_group_unique_id", uid)
    g = ctypes.c_void_p()
    T.call("tb_shard_group_create", 1, 0, uid, 64, 30.0, ctypes.byref(g))
    try:
        _abi_case(T, O, synth, g, 0, 1, T.stream_handle())
        T.call("tb_shard_group_enable_peer", g, 8192)  # a group of one: nothing to map
        with pytest.raises(T.TbError):  # rows above the group's bound
            T.call("tb_argmax_vocab_sharded", g, None, 65, 8, 8, 0, None, T.stream_handle())
    finally:
        T.call("tb_shard_group_destroy", g)


def _abi_rank(rank, world, q_id, q_done, q_sync):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "turbo.cpp_b200", "python"))
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    import turbo_b200 as T
    from oracle import orbind as O
    from turbo_b200 import synth
    T.call("tb_init", rank)
    if rank == 0:
        uid = ctypes.create_string_buffer(128)
        T.call("tb_shard_group_unique_id", uid)
        for _ in range(world - 1):
            q_id.put(uid.raw)
    else:
        uid = ctypes.create_string_buffer(q_id.get(timeout=60), 128)
    g = ctypes.c_void_p()
    T.call("tb_shard_group_create", world, rank, uid, 64, 60.0, ctypes.byref(g))
    try:
        _abi_case(T, O, synth, g, rank, world, T.stream_handle())
        _peer_case(T, O, synth, g, rank, world, T.stream_handle())
        # a rank that skips a call: the others' waits give up (bounded) and
        # report it in the device error word; nothing faults or hangs
        if rank == 0:
            K, n_local = 2048, 4096
            w_local = torch.zeros(n_local * (K // 32) * 34, dtype=torch.uint8, device="cuda")
            xd = torch.zeros(K, dtype=torch.float32, device="cuda")
            yv = torch.zeros(world * n_local, dtype=torch.float32, device="cuda")
            T.call("tb_set_wait_limit_ns", 50_000_000)
            try:
                T.call("tb_gemv_q8_0_row_sharded", g, T.ptr(xd), K, T.ptr(w_local), n_local, T.ptr(yv),
                       T.stream_handle())
                T.call("tb_shard_group_wait", g, T.stream_handle(), 30.0)
            finally:
                T.call("tb_set_wait_limit_ns", 2_000_000_000)
            assert T.take_device_errors() & 1
            for _ in range(world - 1):
                q_sync.put("done")
        else:
            q_sync.get(timeout=120)  # rank 0's stores into this rank's buffer have landed
    finally:
        T.call("tb_shard_group_destroy", g)
    q_done.put(rank)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_shard_group_abi_two_gpus():
    ctx = mp.get_context("spawn")
    q_id, q_done, q_sync = ctx.Queue(), ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_abi_rank, args=(r, 2, q_id, q_done, q_sync)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert sorted(q_done.get(timeout=5) for _ in range(2)) == [0, 1]

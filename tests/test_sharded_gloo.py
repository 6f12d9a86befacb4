"""The vocab-sharded softmax/argmax protocol (turbo_b200.sharded) on 2 and 3
gloo ranks on CPU, with the per-shard halves restated on the CPU
(oracle/shard_ops.py).  Checks the column split, the two softmax all-reduces
and the int64 key all-reduce against the single-process reference semantics:
softmax of the whole row, and greedy_sample's first maximum (ties across shard
boundaries, +-0.0, NaN and -inf entries, a row without candidates).
"""
import os
import socket
import sys
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def make_logits(rows, vocab, seed):
    x = np.random.default_rng(seed).normal(0.0, 2.0, (rows, vocab)).astype(np.float32)
    x[1, :] = -np.inf
    x[1, 7] = np.nan          # no candidate at all -> column 0
    x[2, 5] = 40.0
    x[2, vocab - 3] = 40.0    # tie across shards: the first column wins
    x[3, :] = -1.0
    x[3, vocab // 2] = 0.0
    x[3, vocab // 2 - 1] = -0.0  # -0.0 before +0.0: they tie, the first wins
    x[4, vocab - 1] = 60.0    # winner in the last column
    x[5, 0] = 60.0
    x[5, 1] = np.nan
    return x


def greedy(row):
    best, idx = -np.inf, 0
    for i, v in enumerate(row):
        if v > best:
            best, idx = v, i
    return idx


def _rank_main(rank, world, port, rows, vocab, seed):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "turbo.cpp_b200", "python"))
    from oracle.shard_ops import OracleShardOps
    from turbo_b200.sharded import VocabShardGroup, shard_range
    dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % port, rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    try:
        x = make_logits(rows, vocab, seed)
        g = VocabShardGroup(vocab, ops=OracleShardOps())
        assert (g.col_base, g.cols) == shard_range(vocab, world, rank)
        full = torch.from_numpy(x)
        local = full[:, g.col_base:g.col_base + g.cols]
        idx = g.argmax(local).numpy()
        for r in range(rows):
            assert idx[r] == greedy(x[r]), (rank, r, idx[r], greedy(x[r]))
        ok_rows = [r for r in range(rows) if np.isfinite(x[r]).all()]
        xs = torch.from_numpy(np.ascontiguousarray(x[ok_rows]))
        y = g.softmax(xs[:, g.col_base:g.col_base + g.cols])
        a = x[ok_rows].astype(np.float64)
        e = np.exp(a - a.max(axis=1, keepdims=True))
        want = (e / e.sum(axis=1, keepdims=True))[:, g.col_base:g.col_base + g.cols]
        err = np.abs(y.numpy() - want).max() / want.max()
        assert err < 1e-5, err
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,vocab", [(1, 1001), (2, 128256), (3, 1001)])
def test_vocab_sharded_gloo(world, vocab):
    mp.start_processes(_rank_main, args=(world, _free_port(), 8, vocab, world), nprocs=world, join=True,
                       start_method="spawn")


def test_shard_range_covers_vocab():
    from turbo_b200.sharded import shard_range
    for vocab in (1, 7, 1001, 128256):
        for world in (1, 2, 3, 4, 8):
            spans = [shard_range(vocab, world, r) for r in range(world)]
            assert spans[0][0] == 0
            for (b0, c0), (b1, _) in zip(spans, spans[1:]):
                assert b0 + c0 == b1
            assert spans[-1][0] + spans[-1][1] == vocab
            assert max(c for _, c in spans) - min(c for _, c in spans) <= 1
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


def test_oracle_keys_match_greedy_sample():
    """The key packing restated on the CPU against the reference's own
    greedy_sample (oracle/_ref) on the same rows."""
    from oracle import refbind as R
    from oracle.shard_ops import candidate_keys
    if not R.available():
        pytest.skip("oracle/_ref not built")
    x = make_logits(8, 4099, 0)
    for r in range(8):
        k = candidate_keys(x[r], 0).max()
        got = 0 if k == 0 else int(np.uint64(0xFFFFFFFF) - (k & np.uint64(0xFFFFFFFF)))
        assert got == R.greedy_sample(x[r]), r


def _tp_rank_main(rank, world, port, n, k, vocab, seed):
    # tensor-parallel GEMV (row split + all-gather) and the vocab-split LM head
    # feeding the sharded argmax, with the per-rank products from the oracle
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "turbo.cpp_b200", "python"))
    from oracle import orbind as O
    from oracle.shard_ops import OracleShardOps
    from turbo_b200 import synth
    from turbo_b200.sharded import RowShardedGemv, VocabShardGroup
    dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % port, rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    try:
        ops = OracleShardOps()
        wq = synth.quantize_q8_0(synth.normal((n, k), 0.02, seed=seed))
        x = synth.normal((k,), 1.0, seed=seed + 1)
        tp = RowShardedGemv(n, k, ops=ops)
        w_local = tp.local_rows(torch.from_numpy(wq.ravel()))
        y = tp(torch.from_numpy(x), w_local)
        want = O.matmul_q8_0(x.reshape(1, k), wq, n)[0]
        assert np.array_equal(y.numpy().view(np.uint32), want.view(np.uint32))  # the same per-row order
        # LM head split by vocabulary rows: each rank's logits slice -> sharded argmax
        wl = synth.quantize_q8_0(synth.normal((vocab, k), 0.02, seed=seed + 2))
        g = VocabShardGroup(vocab, ops=ops)
        rb = k // 32 * 34
        mine = torch.from_numpy(wl.ravel()[g.col_base * rb:(g.col_base + g.cols) * rb].copy())
        logits = torch.empty(g.cols, dtype=torch.float32)
        ops.gemv_q8_0(torch.from_numpy(x), mine, g.cols, logits)
        idx = int(g.argmax(logits.reshape(1, g.cols))[0])
        full = O.matmul_q8_0(x.reshape(1, k), wl, vocab)[0]
        assert idx == greedy(full)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [1, 2, 3])
def test_tensor_parallel_gemv_gloo(world):
    mp.start_processes(_tp_rank_main, args=(world, _free_port(), 96 * world, 256, 1003, 11), nprocs=world,
                       join=True, start_method="spawn")


def test_tensor_parallel_gemv_checks_k():
    from turbo_b200.sharded import RowShardedGemv
    port = _free_port()
    dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % port, rank=0, world_size=1,
                            timeout=timedelta(seconds=30))
    try:
        RowShardedGemv(100, 256, ops=object())  # one rank: any row count divides
        with pytest.raises(ValueError):
            RowShardedGemv(100, 250, ops=object())
    finally:
        dist.destroy_process_group()

"""The vocab-sharded softmax/argmax over NCCL on two GPUs (one process per
GPU), with the per-shard halves as the CUDA kernels: turbo_b200.sharded on
[64, 128256] logits against the oracle's single-process results.  Skipped on
machines with fewer than two GPUs."""
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

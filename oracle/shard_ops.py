"""CPU restatement of the per-shard halves of the vocab-sharded softmax and
argmax -- test infrastructure only (the multi-rank CPU tests drive the
torch.distributed protocol of turbo_b200.sharded with these on gloo ranks).

Each method has the meaning of the CUDA entry point of the same role:
  stats      tb_softmax_shard_stats: row max m and sum of exp(x - m) of a slice
  rescale    tb_softmax_shard_rescale: s *= exp(m_local - m_global)
  finish     tb_softmax_shard_finish: y = exp(x - M) / S
  keys       tb_argmax_shard_keys: the 64-bit candidate key, top bit flipped
  key_index  tb_argmax_key_index: the column of a winning key
  gemv_q8_0  tb_matmul_quant(Q8_0, M = 1) on a rank's rows (the oracle's
             reference-order product)
The argmax key restates greedy_sample (src/core/sampler.cpp:13-26): only
values > -inf that are not NaN are candidates, the first (lowest-column) maximum
wins, +0.0 and -0.0 tie, and a row without candidates selects column 0.
Sums are taken in float64 here, so the softmax agrees with the kernels within
the fp32 tolerance, not bit for bit.
"""
import numpy as np
import torch

SIGN_FLIP = np.uint64(0x8000000000000000)


def candidate_keys(x, col_base):
    """uint64 keys of a float32 row slice (0 = not a candidate)."""
    x = np.asarray(x, np.float32)
    cand = x > -np.inf  # False for NaN and -inf
    b = np.where(x == 0.0, np.float32(0.0), x).view(np.uint32).astype(np.uint64)
    neg = (b & np.uint64(0x80000000)) != 0
    b = np.where(neg, (~b) & np.uint64(0xFFFFFFFF), b | np.uint64(0x80000000))
    cols = np.arange(x.shape[-1], dtype=np.uint64) + np.uint64(col_base)
    k = (b << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - cols)
    return np.where(cand, k, np.uint64(0))


class OracleShardOps:
    """Same interface as turbo_b200.sharded.DeviceShardOps, on CPU tensors."""

    def stats(self, x, ld):
        a = x.numpy().astype(np.float64)
        m = a.max(axis=1)
        s = np.exp(a - m[:, None]).sum(axis=1)
        return torch.from_numpy(m.astype(np.float32)), torch.from_numpy(s.astype(np.float32))

    def rescale(self, m_local, m_global, s):
        f = np.exp(m_local.numpy().astype(np.float64) - m_global.numpy().astype(np.float64))
        s.copy_(torch.from_numpy((s.numpy().astype(np.float64) * f).astype(np.float32)))

    def finish(self, x, ld, m_global, s_global, y, ld_y):
        a = x.numpy().astype(np.float64)
        r = np.exp(a - m_global.numpy().astype(np.float64)[:, None]) / s_global.numpy().astype(np.float64)[:, None]
        y.copy_(torch.from_numpy(r.astype(np.float32)))

    def keys(self, x, ld, col_base):
        k = candidate_keys(x.numpy(), col_base).max(axis=1)
        return torch.from_numpy((k ^ SIGN_FLIP).view(np.int64).copy())

    def key_index(self, keys):
        k = keys.numpy().view(np.uint64) ^ SIGN_FLIP
        idx = np.where(k == 0, 0, np.uint64(0xFFFFFFFF) - (k & np.uint64(0xFFFFFFFF))).astype(np.int64)
        return torch.from_numpy(idx)

    def gemv_q8_0(self, x, w_rows, n, y):
        from oracle import orbind as O
        K = x.numel()
        r = O.matmul_q8_0(x.numpy().reshape(1, K).astype(np.float32), w_rows.numpy(), n)
        y.copy_(torch.from_numpy(np.asarray(r, np.float32).reshape(n)))

"""Vocab-sharded softmax and greedy argmax across GPUs, one process per GPU.

Each rank owns a contiguous column slice of logits[rows, vocab] (the lm_head
split of a tensor-parallel decode, or the sharded [64, 128256] sweep).  The
per-shard halves run as kernels of libturbo_b200 (tb_softmax_shard_stats /
_rescale / _finish, tb_argmax_shard_keys / tb_argmax_key_index); the cross-shard
steps are all-reduces issued through torch.distributed (NCCL over NVLink on
GPUs):

  softmax: local row max m_g and s_g = sum exp(x - m_g); all-reduce MAX of m
           -> M; s_g *= exp(m_g - M); all-reduce SUM of s -> S; y = exp(x - M) / S
  argmax:  local 64-bit key per row (value order, then lowest global column);
           all-reduce MAX of the int64 keys; decode the winning column

The single-process forms these replace are Softmax::forward
(src/nn/softmax.cpp:13-54) and greedy_sample (src/core/sampler.cpp:13-26).

RowShardedGemv is the tensor-parallel Q8_0 GEMV: W's rows split over the ranks,
each rank multiplying its rows with the full x (tb_matmul_quant) straight into
its slot of the output, then one in-place all-gather of y.  Its vocab-split
LM-head form (each rank's logits slice) feeds VocabShardGroup.argmax directly,
with no gather.
The per-shard operations are an object (`ops`) so the protocol can be driven by
any implementation of them; the default is the CUDA kernels, and there is no
other implementation in this package.
"""
import ctypes

import torch
import torch.distributed as dist


def shard_range(vocab, world, rank):
    """Columns [base, base + cols) of rank `rank` when `vocab` columns are split
    over `world` ranks: equal slices, the first vocab % world ranks one wider."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank %d of %d" % (rank, world))
    q, r = divmod(vocab, world)
    cols = q + (1 if rank < r else 0)
    base = rank * q + min(rank, r)
    return base, cols


class DeviceShardOps:
    """The per-shard halves as libturbo_b200 kernels on torch CUDA tensors,
    launched on the current stream."""

    def __init__(self):
        from . import load
        self.L = load()

    @staticmethod
    def _s():
        return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def _check(self, st, what):
        from . import check
        check(st, what)

    def stats(self, x, ld):
        rows, cols = x.shape
        m = torch.empty(rows, dtype=torch.float32, device=x.device)
        s = torch.empty(rows, dtype=torch.float32, device=x.device)
        self._check(self.L.tb_softmax_shard_stats(x.data_ptr(), rows, cols, ld, m.data_ptr(), s.data_ptr(),
                                                  self._s()), "tb_softmax_shard_stats")
        return m, s

    def rescale(self, m_local, m_global, s):
        self._check(self.L.tb_softmax_shard_rescale(m_local.data_ptr(), m_global.data_ptr(), s.data_ptr(),
                                                    s.shape[0], self._s()), "tb_softmax_shard_rescale")

    def finish(self, x, ld, m_global, s_global, y, ld_y):
        rows, cols = x.shape
        self._check(self.L.tb_softmax_shard_finish(x.data_ptr(), rows, cols, ld, m_global.data_ptr(),
                                                   s_global.data_ptr(), y.data_ptr(), ld_y, self._s()),
                    "tb_softmax_shard_finish")

    def keys(self, x, ld, col_base):
        rows, cols = x.shape
        k = torch.empty(rows, dtype=torch.int64, device=x.device)
        self._check(self.L.tb_argmax_shard_keys(x.data_ptr(), rows, cols, ld, col_base, k.data_ptr(), self._s()),
                    "tb_argmax_shard_keys")
        return k

    def key_index(self, keys):
        idx = torch.empty(keys.shape[0], dtype=torch.int64, device=keys.device)
        self._check(self.L.tb_argmax_key_index(keys.data_ptr(), keys.shape[0], idx.data_ptr(), self._s()),
                    "tb_argmax_key_index")
        return idx

    def gemv_q8_0(self, x, w_rows, n, y):
        """y[:n] = W_rows . x for n Q8_0 rows of K = x.numel() (tb_matmul_quant, M = 1)."""
        from . import Q8_0
        K = x.numel()
        self._check(self.L.tb_matmul_quant(Q8_0, x.data_ptr(), 1, K, w_rows.data_ptr(), n, y.data_ptr(), self._s()),
                    "tb_matmul_quant")


class VocabShardGroup:
    """Softmax and argmax over logits whose columns are split across the ranks
    of a torch.distributed group.  Every rank calls the same methods in the same
    order (each issues the same collectives)."""

    def __init__(self, vocab, group=None, ops=None):
        if not dist.is_initialized():
            raise RuntimeError("VocabShardGroup needs an initialised torch.distributed process group")
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.vocab = int(vocab)
        self.col_base, self.cols = shard_range(self.vocab, self.world, self.rank)
        self.ops = ops if ops is not None else DeviceShardOps()

    def _check_local(self, x):
        if x.dim() != 2 or x.shape[1] != self.cols:
            raise ValueError("local logits must be [rows, %d] (rank %d of %d), got %s"
                             % (self.cols, self.rank, self.world, tuple(x.shape)))
        if x.stride(1) != 1:
            raise ValueError("local logits must have unit column stride")

    def softmax(self, x, out=None):
        """Softmax of the full rows; writes (and returns) this rank's columns."""
        self._check_local(x)
        if out is None:
            out = torch.empty_like(x)
        m, s = self.ops.stats(x, x.stride(0))
        if self.world == 1:  # a group of one: the local statistics are the global ones
            self.ops.finish(x, x.stride(0), m, s, out, out.stride(0))
            return out
        gmax = m.clone()
        dist.all_reduce(gmax, op=dist.ReduceOp.MAX, group=self.group)
        self.ops.rescale(m, gmax, s)
        dist.all_reduce(s, op=dist.ReduceOp.SUM, group=self.group)
        self.ops.finish(x, x.stride(0), gmax, s, out, out.stride(0))
        return out

    def argmax(self, x):
        """Global first-maximum column per row (greedy_sample's choice); the
        same int64 tensor [rows] on every rank."""
        self._check_local(x)
        keys = self.ops.keys(x, x.stride(0), self.col_base)
        if self.world > 1:
            dist.all_reduce(keys, op=dist.ReduceOp.MAX, group=self.group)
        return self.ops.key_index(keys)


class RowShardedGemv:
    """Tensor-parallel Q8_0 GEMV y[N] = W[N, K] . x[K] over the ranks of a
    torch.distributed group: rank r holds rows [r N/G, (r + 1) N/G) of W (its
    Q8_0 blocks, contiguous) and the full x; it writes its rows straight into
    its slot of y, then one in-place all-gather gives every rank the full y.
    N must be a multiple of the world size (equal slots for the all-gather).
    Every rank calls in the same order."""

    def __init__(self, n, k, group=None, ops=None):
        if not dist.is_initialized():
            raise RuntimeError("RowShardedGemv needs an initialised torch.distributed process group")
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if n <= 0 or n % self.world != 0:
            raise ValueError("rows %d must be a positive multiple of the world size %d" % (n, self.world))
        if k <= 0 or k % 32 != 0:
            raise ValueError("K=%d must be a positive multiple of 32" % k)
        self.n, self.k = int(n), int(k)
        self.rows = self.n // self.world
        self.row_base = self.rank * self.rows
        self.ops = ops if ops is not None else DeviceShardOps()

    def local_rows(self, w_full_blocks):
        """This rank's slice of W's Q8_0 bytes (N rows of K/32 34-byte blocks)."""
        rb = self.k // 32 * 34
        return w_full_blocks[self.row_base * rb:(self.row_base + self.rows) * rb]

    def __call__(self, x, w_local, y=None):
        if x.numel() != self.k:
            raise ValueError("x must hold K=%d values" % self.k)
        if w_local.numel() != self.rows * (self.k // 32) * 34:
            raise ValueError("w_local must hold this rank's %d rows of Q8_0 blocks" % self.rows)
        if y is None:
            y = torch.empty(self.n, dtype=torch.float32, device=x.device)
        slot = y[self.row_base:self.row_base + self.rows]
        self.ops.gemv_q8_0(x, w_local, self.rows, slot)
        if self.world > 1:
            dist.all_gather_into_tensor(y, slot, group=self.group)
        return y

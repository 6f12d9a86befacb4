"""Per-op throughput of the hot-path kernels against the HBM roofline.

Every case calls the C ABI entry point the host layer uses, on seeded
synthetic inputs at the benchmark-config shapes and at large sweep sizes.
Inputs whose working set is below 512 MB are replicated and rotated so that
each call reads from HBM, not L2.  Calls are captured in a CUDA graph and
timed with CUDA events on the launching stream; the per-call time is the
graph time divided by the number of calls.  Prints one JSON line per case.
"""
import ctypes
import json
import math
import os

import numpy as np

from . import synth

ROT_BYTES = 512 << 20


def _peak():
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))),
                     "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class Case:
    def __init__(self, name, config, make, algo_bytes, flops=None):
        self.name, self.config, self.make, self.algo_bytes, self.flops = name, config, make, algo_bytes, flops


def _cases(T, torch):
    dev = "cuda"
    cases = []

    def f32(shape, seed, std=1.0):
        return torch.randn(shape, device=dev, generator=torch.Generator(dev).manual_seed(seed)) * std

    def qblocks(nblocks, bsz, seed):
        """Random quantized blocks generated on the device; every scale is the
        finite half 0x1419 (about 1e-3)."""
        g = torch.Generator(dev).manual_seed(seed)
        w = torch.randint(0, 256, (nblocks, bsz), dtype=torch.uint8, device=dev, generator=g)
        w[:, 0] = 0x19
        w[:, 1] = 0x14
        return w.reshape(-1)

    def rot(nbytes):
        return max(1, min(64, math.ceil(ROT_BYTES / max(nbytes, 1))))

    # ---- A3/A4: broadcast add / row-vector multiply ---------------------------------
    def add_case(rows, cols, dtype, tag, cfg):
        es = 2 if dtype == torch.bfloat16 else 4
        n = rows * cols
        k = rot(3 * n * es)

        def make():
            A = [f32((rows, cols), 1 + i).to(dtype) for i in range(k)]
            B = [f32((rows, cols), 100 + i).to(dtype) for i in range(k)]
            O = [torch.empty((rows, cols), dtype=dtype, device=dev) for _ in range(k)]
            va = [T.view(a) for a in A]
            vb = [T.view(b) for b in B]
            vo = [T.view(o) for o in O]
            keep = (A, B, O, va, vb, vo)
            return (lambda i, s: T.load().tb_binary(0, T.byref(va[i % k]), T.byref(vb[i % k]), T.byref(vo[i % k]), s)), keep
        cases.append(Case("add_" + tag, cfg, make, 3 * n * es))

    add_case(128, 2048, torch.float32, "f32_1x128x2048", "small shapes: x+a fp32 [1,128,2048]")
    add_case(1 << 20, 4096, torch.float32, "f32_16GiB", "sweep: [1048576,4096] fp32 (16 GiB per tensor)")
    add_case(1 << 18, 4096, torch.bfloat16, "bf16_2GiB", "sweep: [262144,4096] bf16")

    def mul_case(rows, cols):
        n = rows * cols

        def make():
            A = f32((rows, cols), 3)
            g = f32((cols,), 4)
            O = torch.empty_like(A)
            va, vg, vo = T.view(A), T.view(g), T.view(O)
            return (lambda i, s: T.load().tb_binary(1, T.byref(va), T.byref(vg), T.byref(vo), s)), (A, g, O, va, vg, vo)
        cases.append(Case("mul_rowvec_f32_4GiB", "sweep: [262144,4096] * [4096] fp32", make, 2 * n * 4 + cols * 4))

    mul_case(1 << 18, 4096)

    # ---- A12: fp32 matmul (the reference's benchmark_gemm shape, and the prefill
    # attention's per-head products) ---------------------------------------------
    def mm_case(M, K, N, tag, cfg):
        def make():
            A, B = f32((M, K), 6), f32((K, N), 7)
            Y = torch.empty((M, N), device=dev)
            va, vb, vy = T.view(A), T.view(B), T.view(Y)
            return (lambda i, s: T.load().tb_matmul_f32(T.byref(va), T.byref(vb), T.byref(vy), s)), (A, B, Y, va, vb, vy)
        cases.append(Case("matmul_f32_" + tag, cfg, make, 4 * (M * K + K * N + M * N), flops=2 * M * K * N))

    mm_case(2048, 2048, 2048, "2048x2048x2048", "reference benchmark_gemm: fp32 2048^3")
    mm_case(512, 64, 512, "512x64x512", "prefill attention scores of one head (S = 512, head_dim 64)")

    # ---- A5/A6: copies ----------------------------------------------------------------
    def transpose_copy(rows, cols):
        n = rows * cols

        def make():
            src = f32((cols, rows), 5)  # contiguous() of its transpose: [rows, cols] strided
            dst = torch.empty((rows, cols), device=dev)
            vs = T.view(src, 0, (rows, cols), (1, rows))
            vd = T.view(dst)
            return (lambda i, s: T.load().tb_copy(T.byref(vd), T.byref(vs), s)), (src, dst, vs, vd)
        cases.append(Case("contiguous_transpose_f32_1GiB", "sweep: [16384,16384]^T -> contiguous fp32", make, 2 * n * 4))

    transpose_copy(16384, 16384)

    def kv_copy():
        S, H, D, ctx = 512, 8, 64, 1024
        k = rot(2 * S * H * D * 4)

        def make():
            Ks = [f32((S, H, D), 6 + i) for i in range(k)]
            Cs = [torch.zeros((ctx, H, D), device=dev) for _ in range(k)]
            vk = [T.view(x) for x in Ks]
            vc = [T.view(c, 0, (S, H, D), (H * D, D, 1)) for c in Cs]
            return (lambda i, s: T.load().tb_copy(T.byref(vc[i % k]), T.byref(vk[i % k]), s)), (Ks, Cs, vk, vc)
        cases.append(Case("kv_append_512x8x64", "KV cache copy_ [512,8,64] into cache[0:512]", make, 2 * S * H * D * 4))

    kv_copy()

    # ---- A7 RMSNorm, A8 SwiGLU ----------------------------------------------------------
    def rms_case(rows, cols, tag, cfg):
        n = rows * cols
        k = rot(2 * n * 4)

        def make():
            X = [f32((rows, cols), 7 + i) for i in range(k)]
            g = torch.rand(cols, device=dev) + 0.5
            Y = [torch.empty_like(x) for x in X]
            return (lambda i, s: T.load().tb_rmsnorm(T.F32, T.ptr(X[i % k]), T.ptr(g), T.ptr(Y[i % k]), rows, cols,
                                                      1e-5, s)), (X, g, Y)
        cases.append(Case("rmsnorm_" + tag, cfg, make, 2 * n * 4 + cols * 4))

    rms_case(128, 2048, "128x2048", "small shapes: RMSNorm [128,2048] eps 1e-5")
    rms_case(1 << 18, 4096, "4GiB", "sweep: [262144,4096] fp32")

    def swiglu_case(n, tag, cfg):
        k = rot(3 * n * 4)

        def make():
            G = [f32((n,), 8 + i) for i in range(k)]
            U = [f32((n,), 50 + i) for i in range(k)]
            Y = [torch.empty_like(g) for g in G]
            return (lambda i, s: T.load().tb_swiglu(T.F32, T.ptr(G[i % k]), T.ptr(U[i % k]), T.ptr(Y[i % k]), n, s)), (G, U, Y)
        cases.append(Case("swiglu_" + tag, cfg, make, 3 * n * 4))

    swiglu_case(128 * 8192, "1x128x8192", "small shapes: SwiGLU [1,128,8192]")
    swiglu_case((1 << 18) * 4096, "4GiB", "sweep: [262144,4096] fp32")

    # ---- A9 softmax, A15 argmax -----------------------------------------------------------
    def rows_case(kind, rows, cols, tag, cfg):
        n = rows * cols
        k = rot((2 if kind == "softmax" else 1) * n * 4)

        def make():
            X = [f32((rows, cols), 9 + i, 2.0) for i in range(k)]
            if kind == "softmax":
                Y = [torch.empty_like(x) for x in X]
                return (lambda i, s: T.load().tb_softmax(T.ptr(X[i % k]), T.ptr(Y[i % k]), rows, cols, s)), (X, Y)
            idx = torch.empty(rows, dtype=torch.int64, device=dev)
            return (lambda i, s: T.load().tb_argmax(T.ptr(X[i % k]), rows, cols, T.ptr(idx), s)), (X, idx)
        cases.append(Case(kind + "_" + tag, cfg, make, (2 if kind == "softmax" else 1) * n * 4 + (0 if kind == "softmax" else 8 * rows)))

    rows_case("softmax", 1, 128256, "1x128256", "small shapes: softmax logits[1,128256]")
    rows_case("softmax", 64, 128256, "64x128256", "sweep: softmax [64,128256]")
    rows_case("softmax", 1024, 128256, "1024x128256", "sweep: softmax [1024,128256] (525 MB)")
    rows_case("softmax", 8192, 128256, "8192x128256", "large: softmax [8192,128256] (4.2 GB)")
    rows_case("argmax", 1, 128256, "1x128256", "small shapes: argmax [1,128256]")
    rows_case("argmax", 64, 128256, "64x128256", "sweep: argmax [64,128256]")
    rows_case("argmax", 8192, 128256, "8192x128256", "large: argmax [8192,128256] (4.2 GB)")

    # ---- nucleus sampling of one row: sample_top_p(logits, 128256, 0.8, 0.9) ----------------
    def sample_case(V, tag, cfg):
        k = rot(V * 4)

        def make():
            X = [f32((V,), 21 + i, 2.5) for i in range(k)]
            out = torch.empty(1, dtype=torch.int32, device=dev)
            return (lambda i, s: T.load().tb_sample_top_p(T.ptr(X[i % k]), V, ctypes.c_float(0.8), ctypes.c_float(0.9),
                                                          ctypes.c_double(((i * 0.6180339887) % 1.0)), T.ptr(out), s)), (X, out)
        cases.append(Case("sample_top_p_" + tag, cfg, make, V * 4 + 4))

    sample_case(128256, "128256", "decode: sample_top_p over logits[128256], T 0.8, top_p 0.9")
    sample_case(262144, "262144", "sweep: sample_top_p over logits[262144]")

    # ---- A14/A17 dequant, quantize, embedding; A13 RoPE ---------------------------------
    def dequant_case(N, K):
        nb = N * K // 32
        k = rot(nb * 34 + N * K * 4)

        def make():
            kk = min(k, 4)
            W = [qblocks(nb, 34, 11 + i) for i in range(kk)]
            Y = [torch.empty(N * K, device=dev) for _ in range(kk)]
            return (lambda i, s: T.load().tb_dequant(T.Q8_0, T.ptr(W[i % kk]), nb, T.ptr(Y[i % kk]), s)), (W, Y)
        cases.append(Case("dequant_q8_0_8192x2048", "decode: exact block dequant of W[8192,2048]", make, nb * 34 + N * K * 4))

    dequant_case(8192, 2048)

    def quantize_case(M, K, cfg):
        nbytes = M * K * 4 + M * K // 32 * 34
        k = rot(nbytes)

        def make():
            X = [f32((M, K), 12 + i) for i in range(k)]
            Q = [torch.empty(M * K // 32 * 34, dtype=torch.uint8, device=dev) for _ in range(k)]
            return (lambda i, s: T.load().tb_quantize_q8_0(T.ptr(X[i % k]), M, K, T.ptr(Q[i % k]), s)), (X, Q)
        cases.append(Case("quantize_q8_0_%dx%d" % (M, K), cfg, make, nbytes))

    quantize_case(512, 8192, "prefill: X[512,8192] -> Q8_0")
    quantize_case(65536, 8192, "sweep: X[65536,8192] -> Q8_0 (2.1 GB in)")

    def embed_case(n, dim, vocab):
        def make():
            W = qblocks(vocab * dim // 32, 34, 13)
            ids = torch.from_numpy(np.random.default_rng(0).integers(0, vocab, n).astype(np.int32)).to(dev)
            Y = torch.empty((n, dim), device=dev)
            return (lambda i, s: T.load().tb_embedding(T.Q8_0, T.ptr(W), dim, vocab, T.ptr(ids), n, T.ptr(Y), s)), (W, ids, Y)
        cases.append(Case("embedding_q8_0_512ids", "1B model: token_embd gather of 512 ids, dim 2048", make,
                          n * (dim // 32 * 34 + dim * 4)))

    embed_case(512, 2048, 128256)

    def rope_case(H, S, D):
        def make():
            X = f32((S, H, D), 14)
            c = torch.rand(1024 * D // 2, device=dev)
            s_ = torch.rand(1024 * D // 2, device=dev)
            v = T.view(X, 0, (1, H, S, D), (S * H * D, D, H * D, 1))
            return (lambda i, s: T.load().tb_rope(T.byref(v), T.ptr(c), T.ptr(s_), D, 1024, 0, s)), (X, c, s_, v)
        cases.append(Case("rope_q_1x32x512x64", "1B model: RoPE on Q [1,32,512,64] view", make, 2 * H * S * D * 4 + S * D * 4))

    rope_case(32, 512, 64)

    # ---- A10/A11: quantized matmul ----------------------------------------------------------
    def gemv_case(N, K, entry, tag, cfg):
        wb = N * K // 32 * 34
        k = rot(wb)

        def make():
            W = [qblocks(N * K // 32, 34, 15 + i) for i in range(k)]
            x = f32((1, K), 16)
            y = torch.empty((1, N), device=dev)
            fn = getattr(T.load(), entry)
            return (lambda i, s: fn(T.Q8_0, T.ptr(x), 1, K, T.ptr(W[i % k]), N, T.ptr(y), s)), (W, x, y)
        cases.append(Case(tag, cfg, make, wb + K * 4 + N * 4))

    gemv_case(8192, 2048, "tb_matmul_quant", "gemv_q8_0_8192x2048", "decode: decode GEMV (default, 1e-5)")
    gemv_case(8192, 2048, "tb_matmul_quant_exact", "gemv_q8_0_8192x2048_exact", "decode: decode GEMV, bit-exact")
    gemv_case(2048, 8192, "tb_matmul_quant", "gemv_q8_0_2048x8192", "1B model: ffn_down GEMV")
    gemv_case(128256, 2048, "tb_matmul_quant", "gemv_q8_0_128256x2048", "1B model: tied lm_head GEMV")

    def gemm_case(dt, M, K, N, tag, cfg):
        def make():
            W = qblocks(N * K // 32, 34 if dt == T.Q8_0 else 18, 17)
            X = f32((M, K), 18)
            Y = torch.empty((M, N), device=dev)
            return (lambda i, s: T.load().tb_matmul_quant(dt, T.ptr(X), M, K, T.ptr(W), N, T.ptr(Y), s)), (W, X, Y)
        wb = N * K // 32 * (34 if dt == T.Q8_0 else 18)
        cases.append(Case(tag, cfg, make, wb + M * K * 4 + M * N * 4, flops=2 * M * N * K))

    def packed_case(dt, M, K, N, tag, cfg):
        # W packed once outside the timed region (tb_pack_quant_weights), as
        # the host layer keeps it for a model's prefill
        def make():
            W = qblocks(N * K // 32, 34 if dt == T.Q8_0 else 18, 17)
            X = f32((M, K), 18)
            Y = torch.empty((M, N), device=dev)
            nbytes = ctypes.c_size_t(0)
            T.call("tb_packed_quant_weights_bytes", dt, N, K, ctypes.byref(nbytes))
            P = torch.empty(nbytes.value, dtype=torch.uint8, device=dev)
            T.call("tb_pack_quant_weights", dt, T.ptr(W), N, K, T.ptr(P), nbytes.value, None)
            torch.cuda.synchronize()
            return (lambda i, s: T.load().tb_matmul_quant_packed(dt, T.ptr(X), M, K, T.ptr(P), N, T.ptr(Y), s)), (
                W, X, Y, P)
        wb = N * K // 32 * (34 if dt == T.Q8_0 else 18)
        cases.append(Case(tag, cfg, make, wb + M * K * 4 + M * N * 4, flops=2 * M * N * K))

    gemm_case(T.Q4_0, 512, 8192, 2048, "gemm_q4_0_512x8192x2048", "prefill: Q4_0 down GEMM")
    gemm_case(T.Q8_0, 512, 2048, 8192, "gemm_q8_0_512x2048x8192", "prefill: Q8_0 gate/up GEMM")
    packed_case(T.Q4_0, 512, 8192, 2048, "gemm_packed_q4_0_512x8192x2048", "prefill: Q4_0 down GEMM, W packed once")
    packed_case(T.Q8_0, 512, 2048, 8192, "gemm_packed_q8_0_512x2048x8192", "prefill: Q8_0 gate/up GEMM, W packed once")
    return cases


def run(only=None, min_ms=20.0, out=None):
    import torch

    import turbo_b200 as T
    T.call("tb_init", 0)
    peak, kind = _peak()
    stream = torch.cuda.Stream()
    results = []
    for case in _cases(T, torch):
        if only and not any(o in case.name for o in only):
            continue
        launch, keep = case.make()
        sh = ctypes.c_void_p(stream.cuda_stream)
        with torch.cuda.stream(stream):
            for i in range(3):
                T.check(launch(i, sh), case.name)
        stream.synchronize()
        # size the graph for >= min_ms of GPU time
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        with torch.cuda.stream(stream):
            for i in range(3):
                T.check(launch(i, sh), case.name)
        t1.record(stream)
        stream.synchronize()
        est = max(t0.elapsed_time(t1) / 3, 1e-3)
        n = int(max(8, min(2000, min_ms / est)))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            cs = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
            for i in range(n):
                T.check(launch(i, cs), case.name)
        with torch.cuda.stream(stream):
            g.replay()
        stream.synchronize()
        t0.record(stream)
        with torch.cuda.stream(stream):
            g.replay()
        t1.record(stream)
        stream.synchronize()
        us = t0.elapsed_time(t1) * 1e3 / n
        gbs = case.algo_bytes / (us * 1e-6) / 1e9
        line = {"op": case.name, "config": case.config, "us_per_call": round(us, 3), "calls": n,
                "algo_bytes": case.algo_bytes, "GB_s": round(gbs, 1), "hbm_frac": round(gbs / peak, 4),
                "peak_GB_s": peak, "peak_source": kind}
        if case.flops:
            line["TFLOP_s"] = round(case.flops / (us * 1e-6) / 1e12, 3)
        results.append(line)
        print(json.dumps(line), flush=True)
        del g, keep, launch
        torch.cuda.empty_cache()
    if out:
        with open(out, "w") as f:
            for r in results:
                f.write(json.dumps(r) + "\n")
    return results


def _rand_q8(torch, rows, K, seed):
    """rows x K/32 random Q8_0 blocks on the device, every scale the finite
    half 0x1419 (about 1e-3)."""
    g = torch.Generator("cuda").manual_seed(seed)
    w = torch.randint(0, 256, (rows * (K // 32), 34), dtype=torch.uint8, device="cuda", generator=g)
    w[:, 0] = 0x19
    w[:, 1] = 0x14
    return w.reshape(-1)


def run_sharded(reps=20, sizes=None, only=None):
    """The sharded sweep on every rank of a torch.distributed job (one GPU per
    rank, NCCL).  Row-sharded ops (add, row-vector mul, RMSNorm, SwiGLU,
    contiguous() of a transposed slab) on [R, 4096] tensors of 1 MiB, 64 MiB,
    1 GiB and 16 GiB in fp32 and bf16, the rows of each tensor split over the
    ranks (no collective); then the vocab-sharded softmax and argmax of logits
    [64, 128256] split over the ranks (two float all-reduces / one int64
    all-reduce per call).  Time per call = max over ranks of the CUDA-event
    time; GB/s = bytes moved by all ranks / that time.  Rank 0 prints one JSON
    line per op and size.  `only`: section names to run (sweep, tp, peer,
    lm_head, vocab)."""
    import torch
    import torch.distributed as dist

    import turbo_b200 as T
    from .sharded import VocabShardGroup, shard_range

    def want(section):
        return not only or section in only

    ws, rank = dist.get_world_size(), dist.get_rank()
    peak, kind = _peak()
    dev = "cuda"
    T.call("tb_init", torch.cuda.current_device())
    stream = torch.cuda.current_stream()
    sh = ctypes.c_void_p(stream.cuda_stream)
    L = T.load()

    def timed(fn, n):
        fn()
        torch.cuda.synchronize()
        dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(n):
            fn()
        b.record()
        torch.cuda.synchronize()
        t = torch.tensor([a.elapsed_time(b) / n], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def report(op, ms, nbytes_total, cfg):
        if rank == 0:
            gbs = nbytes_total / (ms * 1e-3) / 1e9
            print(json.dumps({"suite": "sharded", "op": op, "n_gpus": ws, "config": cfg, "ms_per_call": round(ms, 4),
                              "GB_s": round(gbs, 1), "hbm_frac_per_gpu": round(gbs / ws / peak, 4),
                              "peak_GB_s": peak, "peak_source": kind, "timing": "max over ranks"}), flush=True)

    C = 4096
    sizes = sizes or [1 << 20, 1 << 26, 1 << 30, 1 << 34]  # bytes per tensor, whole job
    for tdt, code, es, tag in (() if not want("sweep") else
                               ((torch.float32, T.F32, 4, "f32"), (torch.bfloat16, T.BF16, 2, "bf16"))):
        for total in sizes:
            R_total = total // (C * es)
            _, R = shard_range(R_total, ws, rank)
            n_all = R_total * C
            n = R * C
            cfg = "[%d,%d] %s (%d MiB per tensor), rows split over %d ranks" % (R_total, C, tag, total >> 20, ws)
            it = 200 if total <= (1 << 26) else (20 if total <= (1 << 30) else 5)
            g = torch.Generator(dev).manual_seed(rank)
            a = torch.randn((R, C), device=dev, generator=g).to(tdt)
            b = torch.randn((R, C), device=dev, generator=g).to(tdt)
            o = torch.empty_like(a)
            va, vb, vo = T.view(a), T.view(b), T.view(o)
            ms = timed(lambda: T.check(L.tb_binary(0, T.byref(va), T.byref(vb), T.byref(vo), sh)), it)
            report("add_" + tag, ms, 3 * es * n_all, cfg)
            row = torch.randn((C,), device=dev, generator=g).to(tdt)
            vr = T.view(row)
            ms = timed(lambda: T.check(L.tb_binary(1, T.byref(va), T.byref(vr), T.byref(vo), sh)), it)
            report("mul_rowvec_" + tag, ms, 2 * es * n_all + es * C * ws, cfg)
            gam = torch.rand((C,), device=dev, generator=g) + 0.5
            ms = timed(lambda: T.check(L.tb_rmsnorm(code, T.ptr(a), T.ptr(gam), T.ptr(o), R, C, 1e-5, sh)), it)
            report("rmsnorm_" + tag, ms, 2 * es * n_all + 4 * C * ws, cfg)
            ms = timed(lambda: T.check(L.tb_swiglu(code, T.ptr(a), T.ptr(b), T.ptr(o), n, sh)), it)
            report("swiglu_" + tag, ms, 3 * es * n_all, cfg)
            vt = T.view(b, 0, (C, R), (1, C))  # contiguous() of a transposed [R, C] slab
            o2 = torch.empty((C, R), device=dev, dtype=tdt)
            vo2 = T.view(o2)
            ms = timed(lambda: T.check(L.tb_copy(T.byref(vo2), T.byref(vt), sh)), it)
            report("contiguous_transpose_" + tag, ms, 2 * es * n_all, cfg)
            del a, b, o, o2, row, gam
            torch.cuda.empty_cache()

    # tensor-parallel Q8_0 GEMV (row split + all-gather of y) and the
    # vocab-split LM head feeding the sharded argmax (no gather)
    from .sharded import RowShardedGemv
    for N, K in (((8192, 2048), (2048, 8192)) if want("tp") else ()):
        tp = RowShardedGemv(N, K)
        rb = K // 32 * 34
        w_local = _rand_q8(torch, tp.rows, K, seed=40 + rank)
        x = torch.randn(K, device=dev, generator=torch.Generator(dev).manual_seed(41))
        y = torch.empty(N, dtype=torch.float32, device=dev)
        ms = timed(lambda: tp(x, w_local, y), 200)
        report("tp_gemv_q8_0_%dx%d" % (N, K), ms, N * rb + K * 4 * ws + N * 4,
               "W[%d,%d] Q8_0 rows split over %d ranks, NCCL all-gather of y" % (N, K, ws))
        del w_local
    # the same GEMVs (and the LM head) through the C entry with the rows
    # exchanged by NVLink peer stores (tb_shard_group_enable_peer), timed as
    # replays of a CUDA graph of `n` calls: at one GPU the group of one is a
    # plain tb_matmul_quant, so the two counts compare like for like
    def timed_graph(fn_s, n):
        s2 = torch.cuda.Stream()
        s2.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s2):
            fn_s(ctypes.c_void_p(s2.cuda_stream))
        s2.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s2):
            cs = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
            for _ in range(n):
                fn_s(cs)
        with torch.cuda.stream(s2):
            g.replay()
        s2.synchronize()
        dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(s2):
            a.record()
            g.replay()
            b.record()
        s2.synchronize()
        t = torch.tensor([a.elapsed_time(b) / n], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        del g
        return float(t.item())

    uid = ctypes.create_string_buffer(128)
    if rank == 0:
        T.call("tb_shard_group_unique_id", uid)
    obj = [uid.raw if want("peer") else None]
    dist.broadcast_object_list(obj, src=0)
    cgrp = ctypes.c_void_p()
    if want("peer"):
        uid = ctypes.create_string_buffer(obj[0], 128)
        T.call("tb_shard_group_create", ws, rank, uid, 64, 60.0, ctypes.byref(cgrp))
        T.call("tb_shard_group_enable_peer", cgrp, 128256)
    for N, K in (((8192, 2048), (2048, 8192), (128256, 2048)) if want("peer") else ()):
        n_local = N // ws
        rb = K // 32 * 34
        w_local = _rand_q8(torch, n_local, K, seed=60 + rank)
        x = torch.randn(K, device=dev, generator=torch.Generator(dev).manual_seed(61))
        y = torch.empty(N, dtype=torch.float32, device=dev)

        def call(sh_):
            T.check(L.tb_gemv_q8_0_row_sharded(cgrp, T.ptr(x), K, T.ptr(w_local), n_local, T.ptr(y), sh_),
                    "tb_gemv_q8_0_row_sharded")
        ms = timed_graph(call, 100)
        report("tp_gemv_peer_q8_0_%dx%d" % (N, K), ms, N * rb + K * 4 * ws + N * 4,
               "W[%d,%d] Q8_0 rows split over %d ranks, rows exchanged by NVLink peer stores, CUDA graph of "
               "100 calls" % (N, K, ws))
        del w_local
    if want("peer"):
        # the vocab-sharded softmax and argmax through the C entries, (m, s)
        # pairs and argmax keys exchanged over NVLink peer memory
        V, rows = 128256, 64
        base, cols = rank * V // ws, (rank + 1) * V // ws - rank * V // ws
        full = torch.randn((rows, V), device=dev, generator=torch.Generator(dev).manual_seed(7)) * 2.0
        local = full[:, base:base + cols].contiguous()
        out = torch.empty_like(local)
        idx = torch.empty(rows, dtype=torch.int64, device=dev)
        ms = timed_graph(lambda sh_: T.check(L.tb_softmax_vocab_sharded(cgrp, T.ptr(local), rows, cols, cols,
                                                                        T.ptr(out), cols, sh_)), 50)
        report("vocab_sharded_softmax_peer", ms, 2 * 4 * rows * V,
               "logits [%d,%d] split over %d ranks, (m, s) pairs over NVLink peer memory, CUDA graph of 50 calls"
               % (rows, V, ws))
        ms = timed_graph(lambda sh_: T.check(L.tb_argmax_vocab_sharded(cgrp, T.ptr(local), rows, cols, cols, base,
                                                                       T.ptr(idx), sh_)), 50)
        report("vocab_sharded_argmax_peer", ms, 4 * rows * V,
               "logits [%d,%d] split over %d ranks, keys over NVLink peer memory, CUDA graph of 50 calls"
               % (rows, V, ws))
        del full, local, out
        # a decode step's pick at the tied LM head: each rank's vocabulary
        # rows (tensor-core GEMV), then the argmax over the ranks' logits
        K = 2048
        w_local = _rand_q8(torch, cols, K, seed=70 + rank)
        x = torch.randn(K, device=dev, generator=torch.Generator(dev).manual_seed(71))
        logits = torch.empty((1, cols), dtype=torch.float32, device=dev)
        idx1 = torch.empty(1, dtype=torch.int64, device=dev)

        def pick(sh_):
            T.check(L.tb_matmul_quant(T.Q8_0, T.ptr(x), 1, K, T.ptr(w_local), cols, T.ptr(logits), sh_),
                    "tb_matmul_quant")
            T.check(L.tb_argmax_vocab_sharded(cgrp, T.ptr(logits), 1, cols, cols, base, T.ptr(idx1), sh_),
                    "tb_argmax_vocab_sharded")
        ms = timed_graph(pick, 50)
        report("tp_lm_head_argmax_peer_%dx%d" % (V, K), ms, V * (K // 32 * 34) + K * 4 * ws + V * 4,
               "LM head W[%d,%d] Q8_0 vocab rows split over %d ranks -> argmax keys over NVLink peer memory, "
               "CUDA graph of 50 calls" % (V, K, ws))
        del w_local
    torch.cuda.synchronize()
    dist.barrier()
    if cgrp:
        T.call("tb_shard_group_destroy", cgrp)

    if want("lm_head"):
        V, K = 128256, 2048
        grp = VocabShardGroup(V)
        w_local = _rand_q8(torch, grp.cols, K, seed=50 + rank)
        x = torch.randn(K, device=dev, generator=torch.Generator(dev).manual_seed(51))
        logits = torch.empty((1, grp.cols), dtype=torch.float32, device=dev)

        def lm_head_argmax():
            T.check(L.tb_matmul_quant(T.Q8_0, T.ptr(x), 1, K, T.ptr(w_local), grp.cols, T.ptr(logits), sh),
                    "tb_matmul_quant")
            return grp.argmax(logits)
        ms = timed(lm_head_argmax, 100)
        report("tp_lm_head_argmax_%dx%d" % (V, K), ms, V * (K // 32 * 34) + K * 4 * ws + V * 4,
               "LM head W[%d,%d] Q8_0 vocab rows split over %d ranks -> sharded argmax" % (V, K, ws))
        del w_local
        torch.cuda.empty_cache()

    if want("vocab"):
        V, rows = 128256, 64
        grp = VocabShardGroup(V)
        full = torch.randn((rows, V), device=dev, generator=torch.Generator(dev).manual_seed(7)) * 2.0
        local = full[:, grp.col_base:grp.col_base + grp.cols].contiguous()
        out = torch.empty_like(local)
        ms = timed(lambda: grp.softmax(local, out), reps)
        report("vocab_sharded_softmax", ms, 2 * 4 * rows * V, "logits [%d,%d] split over %d ranks, NCCL" % (rows, V, ws))
        ms = timed(lambda: grp.argmax(local), reps)
        report("vocab_sharded_argmax", ms, 4 * rows * V, "logits [%d,%d] split over %d ranks, NCCL" % (rows, V, ws))

#!/usr/bin/env python3
"""Headline benchmark: the Q8_0 decode GEMV y = W.x, W[8192, 2048] (GGUF logical
{2048, 8192}), x fp32[1, 2048] -- Tensor::matmul's Q8_0 branch
(src/tensor/tensor.cpp:328-382) on one token, the hot loop of the 1B decode.

Metric: HBM GB/s of algorithmic bytes (Q8_0 weight blocks + x + y per GEMV,
17,866,752 B).  A step is one GEMV over one weight matrix.  32 weight copies
(571 MB, more than 4x the 126 MB L2) rotate, so every step reads its weights
from HBM.

  value  -- device-resident x and W, K steps replayed from a CUDA graph,
            timed with CUDA events on the launching stream (max over ranks).
  e2e    -- the same GEMV through the C ABI with x copied from pinned host
            memory and y copied back to pinned host memory every step (weights
            resident, uploaded once as the Storage layer does); the step's
            three C-ABI calls are captured once through the library's graph
            entry points and replayed per step (the call-by-call rate is in
            the note).
  roofline -- the GEMV kernel alone: bytes per launch / average launch time.
  cpu_baseline -- the reference's own CPU GEMV (oracle/_ref, built from the
            reference sources) on this host's cores, rank 0 only.

--impl reference runs the reference CPU implementation on the same config
(rank 0; other ranks exit 0).  Multi-GPU (torchrun): each rank runs its own row
shard of a [8192*N, 2048] matrix (weak scaling, no collective on the path).
"""
import argparse
import ctypes
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "turbo.cpp_b200", "python"))

N_ROWS, K_COLS = 8192, 2048
ROW_BYTES = K_COLS // 32 * 34
W_BYTES = N_ROWS * ROW_BYTES                      # 17,825,792
ALGO_BYTES = W_BYTES + K_COLS * 4 + N_ROWS * 4    # 17,866,752 per GEMV
N_COPIES = 32
REF_SAMPLE_S = 10.0             # seconds of reference CPU GEMVs per measurement
GRAPH_MAX = 256                 # GEMV launches per captured graph
L2_FLUSH_BYTES = 256 << 20      # read before a short timed region: twice the 126 MB L2
L2_ROTATION_MIN = 15            # steps whose distinct weight copies (267 MB) exceed twice the L2
SLEEP_CYCLES_BASE = 2000000     # ~1 ms of device sleep ahead of the start event
SLEEP_CYCLES_PER_REPLAY = 40000  # + ~20 us per graph replay the host must enqueue
METRIC = "Q8_0 decode GEMV HBM GB/s (W[8192,2048] Q8_0, x fp32[1,2048])"
WORKLOAD = "q8_0_gemv_8192x2048"


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def load_traffic():
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f).get(WORKLOAD)
    return None


class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), "--query-gpu=" + q,
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.reader = threading.Thread(target=self._read, daemon=True)
            self.reader.start()
            time.sleep(0.3)
        except FileNotFoundError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0}
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def cpu_reference_rate(seconds=10.0, max_steps=None):
    """Times the reference's own Q8_0 GEMV (oracle/_ref) on all host cores.
    Returns (GB/s, steps, cores, seconds)."""
    cores = os.cpu_count() or 1
    os.environ["OMP_NUM_THREADS"] = str(cores)
    import numpy as np
    from oracle import refbind as R
    from turbo_b200 import synth
    wq = synth.quantize_q8_0(synth.normal((N_ROWS, K_COLS), 0.02, seed=0))
    x = synth.normal((1, K_COLS), 1.0, seed=1)
    y = np.zeros((1, N_ROWS), np.float32)
    L = R.lib()
    L.ref_matmul_quant_repeat(R.ptr(x), 1, K_COLS, R.ptr(wq), R.DT_Q8_0, N_ROWS, R.ptr(y), 3)
    t0 = time.perf_counter()
    L.ref_matmul_quant_repeat(R.ptr(x), 1, K_COLS, R.ptr(wq), R.DT_Q8_0, N_ROWS, R.ptr(y), 10)
    per = (time.perf_counter() - t0) / 10
    steps = max(1, int(seconds / per))
    if max_steps:
        steps = min(steps, max_steps)
    t0 = time.perf_counter()
    L.ref_matmul_quant_repeat(R.ptr(x), 1, K_COLS, R.ptr(wq), R.DT_Q8_0, N_ROWS, R.ptr(y), steps)
    dt = time.perf_counter() - t0
    return ALGO_BYTES * steps / dt / 1e9, steps, cores, dt


def bench_config(n_gpus):
    """The workload both arms run (the same dict in both JSON lines)."""
    return {"workload": WORKLOAD, "N": N_ROWS, "K": K_COLS, "M": 1, "parallelism": "row-shard x%d" % n_gpus,
            "l2": "inputs larger than L2: %d rotating weight copies (%.0f MB), a step's copy was last read "
                  ">= 14 copies (250 MB) earlier; a 256 MB read flushes L2 before regions under %d steps"
                  % (N_COPIES, N_COPIES * W_BYTES / 1e6, L2_ROTATION_MIN)}


def run_reference(args):
    ws, rank, _ = dist_env()
    if rank != 0:
        return 0
    from oracle import refbind as R
    if not R.available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libturbo_ref.so was not built"}))
        return 0
    # a bounded sample of about REF_SAMPLE_S seconds of full GEMVs, the same
    # sample the cpu_baseline leg of our own arm takes (a step of K = 20 GEMVs
    # is ~25 ms of CPU work: too short to time the reference's OpenMP loop)
    gbs, steps, cores, dt = cpu_reference_rate(seconds=REF_SAMPLE_S)
    ms = dt / steps * 1e3
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic", "config": bench_config(args.gpus),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "reference",
                         "sample": "%d full GEMVs in %.1f s (Tensor::matmul Q8_0, OpenMP over %d threads)" % (
                             steps, dt, cores)},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


def run_ours(args):
    import numpy as np
    import torch
    import turbo_b200 as T
    from turbo_b200 import synth

    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    if ws > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    T.call("tb_init", local)
    stream = torch.cuda.Stream()
    sh = T.stream_handle(stream)

    # Inputs: this rank's row shard, quantized once on the host and uploaded.
    w_host = synth.quantize_q8_0(synth.normal((N_ROWS, K_COLS), 0.02, seed=100 + rank))
    x_host = synth.normal((1, K_COLS), 1.0, seed=1)
    w0 = torch.from_numpy(w_host.ravel()).cuda()
    wcopies = [w0] + [w0.clone() for _ in range(N_COPIES - 1)]
    x = torch.from_numpy(x_host).cuda()
    y = torch.empty((1, N_ROWS), dtype=torch.float32, device="cuda")

    entry = "tb_matmul_quant_exact" if args.exact else "tb_matmul_quant"
    fn = getattr(T.load(), entry)

    def gemv(i, s=sh, xx=x, yy=y):
        T.check(fn(T.Q8_0, T.ptr(xx), 1, K_COLS, T.ptr(wcopies[i % N_COPIES]), N_ROWS, T.ptr(yy), s), entry)

    # correctness gate before timing, rank 0, against the oracle: bit-exact for
    # the exact entry, else |y - y_ref| <= 1e-5 * sum|w x| per output
    with torch.cuda.stream(stream):
        gemv(0)
    stream.synchronize()
    if rank == 0:
        from oracle import orbind as O
        ref = O.matmul_q8_0(x_host, w_host, N_ROWS)
        got = y.cpu().numpy()
        if args.exact:
            ok = np.array_equal(got.view(np.uint32), ref.view(np.uint32))
        else:
            scale = np.abs(synth.dequantize_q8_0(w_host, K_COLS)).astype(np.float64) @ np.abs(x_host[0]).astype(np.float64)
            ok = bool(np.max(np.abs(got[0].astype(np.float64) - ref[0]) / scale) <= 1e-5)
        if not ok:
            raise SystemExit("GEMV result differs from the oracle beyond tolerance; not timing")

    # warmup
    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            gemv(i)
    stream.synchronize()

    # --- value: K steps replayed from CUDA graphs --------------------------------
    # One graph of G = min(K, GRAPH_MAX) GEMVs (weight copy i % 32 at step i),
    # replayed K // G times, plus a graph of the K % G remaining ones.  Every
    # graph is replayed once before the timed region (upload and first-launch
    # costs stay outside it).  A device-side sleep is queued ahead of the timed
    # replays, so that the host has enqueued every replay before the first
    # timed GEMV starts: the region measures the GPU.  With K <= GRAPH_MAX the
    # start and end events are recorded inside the graph, around its K GEMVs
    # (the graph's own launch stays outside the region); longer runs put them
    # around the replays.
    # L2: the K GEMVs of the region read K distinct weight copies, so from
    # K >= L2_ROTATION_MIN on every copy's lines have been evicted by the other
    # copies' reads before the region reaches it again (inputs larger than L2,
    # no flush).  Shorter runs read a 256 MB buffer before the region (a read:
    # it leaves clean lines, so the region does not write back a previous
    # write's dirty lines).
    G = min(args.steps, GRAPH_MAX)
    in_graph = args.steps <= GRAPH_MAX
    start = torch.cuda.Event(enable_timing=True, external=in_graph)
    end = torch.cuda.Event(enable_timing=True, external=in_graph)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        cur = torch.cuda.current_stream()
        if in_graph:
            start.record(cur)
        for i in range(G):
            gemv(i, s=T.stream_handle(cur))
        if in_graph:
            end.record(cur)
    tail = args.steps % G
    graph_tail = None
    if tail:
        graph_tail = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph_tail, stream=stream):
            for i in range(tail):
                gemv(G + i, s=T.stream_handle(torch.cuda.current_stream()))
    flush = None
    if args.steps < L2_ROTATION_MIN:
        # written before the warm replays, which evict (and write back) its lines
        flush = torch.ones(L2_FLUSH_BYTES // 4, dtype=torch.int32, device="cuda")
    warm_replays = 0
    with torch.cuda.stream(stream):
        for g in (graph, graph_tail):
            if g is not None:
                g.replay()
                warm_replays += 1
    stream.synchronize()

    if ws > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    n_replays = args.steps // G
    with ClockSampler(local) as clocks:
        with torch.cuda.stream(stream):
            flush_sum = flush.sum() if flush is not None else None
            torch.cuda._sleep(SLEEP_CYCLES_BASE + SLEEP_CYCLES_PER_REPLAY * (n_replays + 1))
            if not in_graph:
                start.record(stream)
            for _ in range(n_replays):
                graph.replay()
            if graph_tail is not None:
                graph_tail.replay()
            if not in_graph:
                end.record(stream)
        stream.synchronize()
    torch.cuda.synchronize()
    total_ms = start.elapsed_time(end)
    if flush is not None:
        assert int(flush_sum.item()) == L2_FLUSH_BYTES // 4
        del flush
    if ws > 1:
        t = torch.tensor([total_ms], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        total_ms = float(t.item())
        torch.distributed.barrier()

    # --- e2e: x from pinned host, y back to pinned host, through the C ABI -----
    e2e_steps = min(args.steps, 2000)
    xh = torch.from_numpy(x_host.copy()).pin_memory()
    yh = torch.empty((1, N_ROWS), dtype=torch.float32).pin_memory()
    L = T.load()

    def e2e_step(i):
        T.check(L.tb_upload(T.ptr(x), ctypes.c_void_p(xh.data_ptr()), K_COLS * 4, sh))
        gemv(i)
        T.check(L.tb_download(ctypes.c_void_p(yh.data_ptr()), T.ptr(y), N_ROWS * 4, sh))

    def timed_e2e(step):
        for i in range(3):
            step(i)
        stream.synchronize()
        if ws > 1:
            torch.distributed.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(e2e_steps):
            step(i)
        e1.record(stream)
        stream.synchronize()
        ms = e0.elapsed_time(e1)
        if ws > 1:
            t = torch.tensor([ms], device="cuda")
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    # (a) the three C-ABI calls per step; (b) the same three calls captured once
    # per weight copy through the C ABI (tb_capture_begin/end) and launched per
    # step with tb_graph_launch, as a caller that repeats a fixed step does
    e2e_calls_ms = timed_e2e(e2e_step)
    e2e_graphs = []
    for i in range(N_COPIES):
        T.check(L.tb_capture_begin(sh))
        e2e_step(i)
        g = ctypes.c_void_p()
        T.check(L.tb_capture_end(sh, ctypes.byref(g)))
        e2e_graphs.append(g)
    e2e_graph_ms = timed_e2e(lambda i: T.check(L.tb_graph_launch(e2e_graphs[i % N_COPIES], sh)))
    for g in e2e_graphs:
        T.check(L.tb_graph_destroy(g))
    e2e_ms = e2e_graph_ms

    del graph, graph_tail
    if ws > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if rank != 0:
        return 0

    peak, peak_kind = load_peaks()
    value = ALGO_BYTES * args.steps * ws / (total_ms * 1e-3) / 1e9
    # the timed region holds only GEMV launches, back to back in the graph:
    # the average launch duration is the region's time per launch (this rank)
    kernel_ms = total_ms / args.steps
    achieved = ALGO_BYTES / (kernel_ms * 1e-3) / 1e9
    e2e_gbs = ALGO_BYTES * e2e_steps * ws / (e2e_ms * 1e-3) / 1e9
    cpu = None
    if not args.no_cpu_baseline and ws == 1:
        from oracle import refbind as R
        if R.available():
            gbs, steps, cores, dt = cpu_reference_rate(seconds=REF_SAMPLE_S)
            cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "reference",
                   "sample": "%d full GEMVs on the reference library (%.1f s, OpenMP %d threads)" % (steps, dt, cores)}
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 6), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic (N(0,0.02) weights quantized Q8_0, x N(0,1), seeded)",
        "config": bench_config(ws),
        "method": {"entry": entry, "tolerance": "bit-exact" if args.exact else "1e-5 * sum|w x| per output",
                   "launch": "CUDA graph of %d GEMVs replayed %d times%s; every graph replayed once before "
                             "timing (%d warm replays); replays queued behind a device sleep; %s%s"
                             % (G, n_replays, " + a %d-GEMV tail graph" % tail if tail else "", warm_replays,
                                "start/end events recorded inside the graph around its GEMVs" if in_graph
                                else "start/end events around the replays",
                                "; L2 flushed by a 256 MB read" if args.steps < L2_ROTATION_MIN else "")},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": load_traffic(),
                     "peak_source": peak_kind, "kernel_us": round(kernel_ms * 1e3, 3),
                     "timing": "CUDA events on the launching stream, recorded inside the graph around its GEMVs"
                               if in_graph else "CUDA events on the launching stream around the graph replays"},
        "e2e": {"value": round(e2e_gbs, 2), "unit": "GB/s", "h2d_bytes_per_step": K_COLS * 4,
                "d2h_bytes_per_step": N_ROWS * 4, "steps": e2e_steps,
                "note": "tb_upload(x) + tb_matmul_quant + tb_download(y) per step from pinned host buffers, "
                        "weights resident; the step captured once per weight copy through the C ABI "
                        "(tb_capture_begin/end) and replayed with tb_graph_launch; the same three calls issued "
                        "one by one: %.1f GB/s" % (ALGO_BYTES * e2e_steps * ws / (e2e_calls_ms * 1e-3) / 1e9)},
        "gpu_launches": args.steps,
        "clocks": clocks.summary(),
        "cpu_baseline": cpu,
    }
    if ws == 1 and not args.no_decode:
        line["decode_1b"] = decode_1b_leg(args)
    print(json.dumps(line))
    return 0


DECODE_WEIGHT_BYTES = 1312980992  # Q8_0 layer blocks + the tied 128256 x 2048 LM head, per token
REF_DECODE_PROMPT, REF_DECODE_STEPS = 16, 8


def decode_1b_leg(args):
    """The second half of the headline metric: the Llama-3.2-1B-shaped Q8_0
    greedy decode (prompt of 512 seeded ids, then 128 steps) through the C++
    host layer's public model API (libturbo_b200_host.so: one CUDA graph per
    token), its token ids against the reference's run of the same model
    (tests/golden/decode_1b.npz), and the reference's own CPU decode timed on
    this host in the same run on a bounded sample."""
    import ctypes as C
    import numpy as np
    from turbo_b200 import gguf_synth
    from turbo_b200.model import Model
    golden = np.load(os.path.join(ROOT, "tests", "golden", "decode_1b.npz"))
    t0 = time.perf_counter()
    path = gguf_synth.ensure_model()
    synth_s = time.perf_counter() - t0
    steps, max_seq = int(golden["steps"]), int(golden["max_seq"])
    prompt = golden["prompt"]
    t0 = time.perf_counter()
    m = Model(path, exact=False)
    load_s = time.perf_counter() - t0
    m.generate(prompt, 4, max_seq=max_seq, want_margins=False)  # warm-up (graph capture, first launches)
    runs = [m.generate(prompt, steps, max_seq=max_seq, want_margins=False) for _ in range(2)]
    best = min(runs, key=lambda r: r["decode_ms"])
    same = all(bool(np.array_equal(r["ids"], golden["ids"])) for r in runs)
    short = m.generate(prompt[:REF_DECODE_PROMPT], REF_DECODE_STEPS, max_seq=max_seq, want_margins=False)
    m.close()
    tok_s = steps / (best["decode_ms"] / 1e3)
    kv_bytes = 16 * 2 * 512 * 4 * (prompt.size + steps / 2)  # K and V rows read per token, mean context
    per_tok = DECODE_WEIGHT_BYTES + kv_bytes
    peak, peak_kind = load_peaks()
    out = {"metric": "Q8_0 1B-shape greedy decode tokens/sec", "value": round(tok_s, 1), "unit": "tok/s",
           "steps": steps, "prompt": int(prompt.size), "runs": len(runs),
           "decode_ms": round(best["decode_ms"], 2), "prefill_ms": round(best["prefill_ms"], 1),
           "ids_identical_to_reference": same,
           "path": "tbm_model_generate: one CUDA graph per token of the fused layer kernels (5 per layer)",
           "roofline": {"bound": "hbm", "bytes_per_token": int(per_tok), "achieved": round(per_tok * tok_s / 1e9, 1),
                        "peak": peak, "unit": "GB/s", "frac": round(per_tok * tok_s / 1e9 / peak, 4),
                        "peak_source": peak_kind},
           "model": {"path_kind": "synthetic GGUF, seed 0 (turbo_b200.gguf_synth)", "write_s": round(synth_s, 1),
                     "load_upload_s": round(load_s, 2)}}
    from oracle import refbind as R
    if args.no_cpu_baseline or not R.available():
        out["reference_cpu"] = None
        return out
    cores = os.cpu_count() or 1
    os.environ["OMP_NUM_THREADS"] = str(cores)
    L = R.lib()
    h = L.ref_model_load(path.encode())
    if not h:
        out["reference_cpu"] = {"unavailable": "the reference failed to load the model"}
        return out
    sp = np.ascontiguousarray(prompt[:REF_DECODE_PROMPT], np.int32)
    ids = np.zeros(REF_DECODE_STEPS + 1, np.int32)
    pre, dec = C.c_double(), C.c_double()
    R.check(L.ref_model_generate(h, R.ptr(sp), sp.size, REF_DECODE_STEPS, max_seq, R.ptr(ids), None, None,
                                 C.byref(pre), C.byref(dec)), "ref_model_generate")
    L.ref_model_free(h)
    ref_tok_s = REF_DECODE_STEPS / (dec.value / 1e3)
    out["reference_cpu"] = {
        "value": round(ref_tok_s, 3), "unit": "tok/s", "cores": cores, "kind": "reference",
        "sample": "reference MiniGPT (its sources compiled under oracle/_ref), prompt of %d ids then %d greedy "
                  "steps (context %d-%d), OpenMP %d threads; prefill %.1f s" % (
                      REF_DECODE_PROMPT, REF_DECODE_STEPS, REF_DECODE_PROMPT, REF_DECODE_PROMPT + REF_DECODE_STEPS,
                      cores, pre.value / 1e3),
        "ids_identical_on_sample": bool(np.array_equal(ids, short["ids"]))}
    return out


def ops_cpu_reference():
    """The reference's own CPU ops (oracle/_ref) at the benchmark-config sizes,
    all host cores; one JSON line each."""
    cores = os.cpu_count() or 1
    os.environ["OMP_NUM_THREADS"] = str(cores)
    from oracle import refbind as R
    from turbo_b200 import synth
    if not R.available():
        print(json.dumps({"cpu_reference": "unavailable: oracle/_ref/libturbo_ref.so was not built"}))
        return
    x = synth.normal((1, 128, 2048), 1.0, seed=0)
    a = synth.normal((1, 128, 2048), 1.0, seed=1)
    g = synth.uniform((2048,), 0.5, 1.5, seed=1)
    gg = synth.normal((1, 128, 8192), 1.0, seed=2)
    uu = synth.normal((1, 128, 8192), 1.0, seed=3)
    lg = synth.normal((1, 128256), 2.0, seed=4)
    wq = synth.quantize_q8_0(synth.normal((8192, 2048), 0.02, seed=5))
    xv = synth.normal((1, 2048), 1.0, seed=6)
    cases = [("add_f32_1x128x2048", lambda: R.add(x, a), 3 * x.nbytes),
             ("rmsnorm_128x2048", lambda: R.rmsnorm(x.reshape(128, 2048), g), 2 * x.nbytes),
             ("swiglu_1x128x8192", lambda: R.swiglu(gg, uu), 3 * gg.nbytes),
             ("softmax_1x128256", lambda: R.softmax(lg), 2 * lg.nbytes),
             ("argmax_1x128256", lambda: R.greedy_sample(lg), lg.nbytes),
             ("gemv_q8_0_8192x2048", lambda: R.matmul_quant(xv, wq, R.DT_Q8_0, 8192), ALGO_BYTES)]
    for name, fn, nbytes in cases:
        fn()
        reps, t0 = 0, time.perf_counter()
        while True:
            fn()
            reps += 1
            dt = time.perf_counter() - t0
            if dt > 1.0 or reps >= 200:
                break
        us = dt / reps * 1e6
        print(json.dumps({"op": name, "impl": "reference_cpu", "us_per_call": round(us, 2),
                          "GB_s": round(nbytes / (us * 1e-6) / 1e9, 2), "cores": cores, "calls": reps}),
              flush=True)


def run_ops_suite(args):
    """Every hot-path op through the C ABI at the benchmark-config sizes and at
    large sweep sizes: one JSON line per op (us per call, GB/s of algorithmic
    bytes, fraction of the HBM roofline), then the reference CPU ops."""
    ws, rank, _ = dist_env()
    if rank != 0:
        return 0
    from turbo_b200 import opbench
    opbench.run(only=args.only.split(",") if args.only else None)
    if not args.no_cpu_baseline:
        ops_cpu_reference()
    return 0


def run_decode_suite(args):
    """The 1B-shaped Q8_0 greedy decode (prefill 512 ids, then 128 steps) through
    the C++ host layer, both paths; token ids checked against the reference's
    run (tests/golden/decode_1b.npz, made by tests/golden/make_decode_golden.py
    on the reference library)."""
    import numpy as np
    ws, rank, _ = dist_env()
    if rank != 0:
        return 0
    from turbo_b200 import gguf_synth
    from turbo_b200.model import Model
    golden = np.load(os.path.join(ROOT, "tests", "golden", "decode_1b.npz"))
    model_path = gguf_synth.ensure_model()
    steps = int(golden["steps"])
    paths = [("fused", False, False), ("persistent", False, True)] + ([("exact", True, False)] if args.only == "both" else [])
    for name, exact, persistent in paths:
        m = Model(model_path, exact=exact, persistent=persistent)
        m.generate(golden["prompt"], 4, max_seq=int(golden["max_seq"]), want_margins=False)  # warm-up
        runs = [m.generate(golden["prompt"], steps, max_seq=int(golden["max_seq"]), want_margins=False)
                for _ in range(max(1, args.reps))]
        m.close()
        best = min(runs, key=lambda r: r["decode_ms"])
        same = all(bool(np.array_equal(r["ids"], golden["ids"])) for r in runs)
        line = {"suite": "decode", "metric": "Q8_0 1B-shape greedy decode tokens/sec",
                "value": round(steps / (best["decode_ms"] / 1e3), 1), "unit": "tok/s",
                "path": {"exact": "exact op-by-op", "fused": "CUDA graph per token, fused layer kernels",
                         "persistent": "CUDA graph per token: one persistent kernel for the step + pick"}[name],
                "prefill_ms": round(best["prefill_ms"], 1), "decode_ms": round(best["decode_ms"], 1),
                "steps": steps, "prompt": int(golden["prompt"].size), "runs": len(runs),
                "ids_identical_to_reference": same,
                "reference_cpu": {"decode_tok_s": round(steps / (float(golden["decode_ms"]) / 1e3), 2),
                                  "prefill_ms": round(float(golden["prefill_ms"]), 1),
                                  "threads": int(golden["threads"]),
                                  "note": "the reference library on this repository's build host (golden file)"}}
        print(json.dumps(line), flush=True)
    return 0


def run_sharded_suite(args):
    """Row-sharded sweep ops and the NCCL vocab-sharded softmax/argmax on every
    rank (launch under torchrun for N > 1; N = 1 runs a one-rank group)."""
    import datetime
    import torch
    import torch.distributed as dist
    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29533")
    os.environ.setdefault("RANK", "0")
    os.environ.setdefault("WORLD_SIZE", "1")
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    try:
        from turbo_b200 import opbench
        opbench.run_sharded(only=args.only.split(",") if args.only else None)
    finally:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-decode", action="store_true",
                    help="skip the 1B-shaped decode leg of the N=1 line (it writes a 1.3 GB synthetic model once)")
    ap.add_argument("--exact", action="store_true",
                    help="time tb_matmul_quant_exact (bit-identical to the reference) instead")
    ap.add_argument("--suite", default="headline", choices=["headline", "ops", "decode", "sharded"],
                    help="ops: per-op throughput of every hot-path kernel (one JSON line per op); "
                         "decode: the 1B-shaped greedy decode in tokens/sec")
    ap.add_argument("--reps", type=int, default=3, help="with --suite decode: timed generate calls")
    ap.add_argument("--only", default="", help="with --suite ops: comma-separated op name filters; with --suite "
                    "sharded: sections (sweep, tp, peer, lm_head, vocab)")
    args = ap.parse_args()
    if args.suite == "ops":
        return run_ops_suite(args)
    if args.suite == "decode":
        return run_decode_suite(args)
    if args.suite == "sharded":
        return run_sharded_suite(args)
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())

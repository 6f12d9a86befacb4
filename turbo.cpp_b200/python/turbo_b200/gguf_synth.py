"""Writes seeded synthetic Llama-shaped models as GGUF (v3) files.

The tensors and metadata keys are the ones the Turbo.cpp loader and MiniGPT
read (token_embd, blk.N.{attn_norm,attn_q,attn_k,attn_v,attn_output,ffn_norm,
ffn_gate,ffn_up,ffn_down}, output_norm; llama.* hyper-parameters).  Weights are
N(0, std) quantized per GGUF Q8_0 (or Q4_0), norm weights are 1, and there is no
output.weight, so the LM head is tied to token_embd.  The same seed gives the
same bytes on every machine with the same numpy.
"""
import struct

import numpy as np

from . import synth

GGUF_MAGIC = 0x46554747
T_UINT32, T_FLOAT32, T_STRING = 4, 6, 8
GGML_F32, GGML_Q4_0, GGML_Q8_0 = 0, 2, 8

LLAMA_1B = dict(n_layers=16, hidden=2048, n_heads=32, n_kv_heads=8, ffn=8192, vocab=128256,
                rope_theta=500000.0, context=1024)


def _str(s):
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _kv_u32(k, v):
    return _str(k) + struct.pack("<II", T_UINT32, v)


def _kv_f32(k, v):
    return _str(k) + struct.pack("<If", T_FLOAT32, v)


def tensor_specs(cfg):
    """(name, ggml dims [ne0=K, ne1=N], kind) in file order."""
    H, F, V = cfg["hidden"], cfg["ffn"], cfg["vocab"]
    kv = H // cfg["n_heads"] * cfg["n_kv_heads"]
    specs = [("token_embd.weight", [H, V], "w")]
    for i in range(cfg["n_layers"]):
        p = "blk.%d." % i
        specs += [(p + "attn_norm.weight", [H], "norm"), (p + "attn_q.weight", [H, H], "w"),
                  (p + "attn_k.weight", [H, kv], "w"), (p + "attn_v.weight", [H, kv], "w"),
                  (p + "attn_output.weight", [H, H], "w"), (p + "ffn_norm.weight", [H], "norm"),
                  (p + "ffn_gate.weight", [H, F], "w"), (p + "ffn_up.weight", [H, F], "w"),
                  (p + "ffn_down.weight", [F, H], "w")]
    specs.append(("output_norm.weight", [H], "norm"))
    return specs


def tensor_chunks(dims, kind, qtype, rng, std, chunk_values=1 << 22):
    """The tensor's bytes in row chunks of about `chunk_values` weights (the
    generator's stream is the same however the rows are split, so the bytes
    equal one draw of the whole [N, K] matrix)."""
    if kind == "norm":
        yield np.ones(dims[0], np.float32).tobytes()
        return
    K, N = dims
    rows = max(1, chunk_values // K)
    quant = synth.quantize_q8_0 if qtype == GGML_Q8_0 else synth.quantize_q4_0
    for r0 in range(0, N, rows):
        n = min(rows, N - r0)
        w = (rng.standard_normal((n, K), dtype=np.float32) * np.float32(std)).astype(np.float32)
        yield quant(w).tobytes()


def default_model_path():
    """Where the tests and the bench keep the synthetic 1B-shaped model: the
    TURBO_B200_MODEL environment variable, else a file in the system's
    temporary directory."""
    import os
    import tempfile
    return os.environ.get("TURBO_B200_MODEL") or os.path.join(tempfile.gettempdir(),
                                                              "turbo_b200_llama1b_q8_0_seed0.gguf")


def ensure_model(path=None):
    """Writes the seed-0 1B-shaped Q8_0 model at `path` unless it is there."""
    import os
    path = path or default_model_path()
    if not os.path.exists(path):
        write_model(path + ".part")
        os.replace(path + ".part", path)
    return path


def write_model(path, cfg=LLAMA_1B, seed=0, std=0.02, qtype=GGML_Q8_0, alignment=32):
    specs = tensor_specs(cfg)
    rng = np.random.default_rng(seed)
    kvs = [_kv_u32("general.alignment", alignment), _kv_u32("llama.block_count", cfg["n_layers"]),
           _kv_u32("llama.embedding_length", cfg["hidden"]), _kv_u32("llama.feed_forward_length", cfg["ffn"]),
           _kv_u32("llama.attention.head_count", cfg["n_heads"]),
           _kv_u32("llama.attention.head_count_kv", cfg["n_kv_heads"]),
           _kv_u32("llama.context_length", cfg["context"]), _kv_f32("llama.rope.freq_base", cfg["rope_theta"])]
    # sizes first (offsets), then stream the data
    sizes = []
    for name, dims, kind in specs:
        n = int(np.prod(dims))
        if kind == "norm":
            sizes.append(n * 4)
        else:
            sizes.append(n // 32 * (34 if qtype == GGML_Q8_0 else 18))
    infos = b""
    off = 0
    offsets = []
    for (name, dims, kind), sz in zip(specs, sizes):
        offsets.append(off)
        ty = GGML_F32 if kind == "norm" else qtype
        infos += _str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        infos += struct.pack("<IQ", ty, off)
        off += (sz + alignment - 1) // alignment * alignment
    head = struct.pack("<IIQQ", GGUF_MAGIC, 3, len(specs), len(kvs)) + b"".join(kvs) + infos
    pad = (alignment - len(head) % alignment) % alignment
    with open(path, "wb") as f:
        f.write(head + b"\0" * pad)
        for (name, dims, kind), sz in zip(specs, sizes):
            n = 0
            for data in tensor_chunks(dims, kind, qtype, rng, std):
                f.write(data)
                n += len(data)
            assert n == sz
            f.write(b"\0" * ((alignment - sz % alignment) % alignment))
    return path


def prompt_ids(n=512, vocab=LLAMA_1B["vocab"], seed=0):
    return np.random.default_rng(seed).integers(0, vocab, size=n).astype(np.int32)

"""The C ABI library loads without a GPU and exports every entry point that
include/*.h declares (no compute calls: this suite runs on CPU)."""
import glob
import os
import re
import ctypes
import subprocess

import pytest

import turbo_b200 as T

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DECL = re.compile(r"^\s*(?:tb_status|const\s+char\s*\*|void|int)\s*\*?\s*(tb_\w+)\s*\(", re.M)


def declared():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        names |= set(DECL.findall(open(h).read()))
    return sorted(names)


def test_header_declares_entry_points():
    names = declared()
    assert "tb_matmul_quant" in names and "tb_softmax" in names and len(names) >= 25


def test_library_exports_every_declared_symbol():
    if not os.path.exists(T.LIB_PATH):
        pytest.skip("library not built")
    out = subprocess.run(["nm", "-D", "--defined-only", T.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(line.split()[-1] for line in out.splitlines() if " T " in line)
    missing = [n for n in declared() if n not in exported]
    assert not missing, missing
    # nothing but the C ABI is exported (hidden visibility)
    extra = [n for n in exported if not n.startswith("tb_")]
    assert not extra, extra[:10]


def test_library_loads_and_binding_matches_header():
    if not os.path.exists(T.LIB_PATH):
        pytest.skip("library not built")
    L = T.load()
    assert L.tb_version().startswith(b"turbo_b200 sm_100a")
    assert L.tb_status_name(T.ERANGE) == b"TB_ERANGE"
    assert set(T.SIGNATURES) == set(declared())


def test_no_cuda_device_fails_loudly():
    # Without a GPU every compute entry point must fail (TB_ECUDA), never run on the CPU.
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    if not os.path.exists(T.LIB_PATH):
        pytest.skip("library not built")
    L = T.load()
    st = L.tb_softmax(None, None, 1, 1, None)
    assert st in (T.EINVAL, T.ECUDA)
    st = L.tb_init(0)
    assert st == T.ECUDA


def test_host_library_exports_model_interface():
    host = os.path.join(os.path.dirname(T.LIB_PATH), "libturbo_b200_host.so")
    if not os.path.exists(host):
        pytest.skip("host library not built")
    out = subprocess.run(["nm", "-D", "--defined-only", host], capture_output=True, text=True).stdout
    for sym in ("tbm_model_load", "tbm_model_generate", "tbm_model_free", "tbm_last_error"):
        assert sym in out


def test_packed_weight_size_needs_no_device():
    """The packed-weight size is host arithmetic: both fp16 planes of every
    128-row tile (4 bytes per weight), then one scale per row and 256 K, each
    part rounded up to 1 KiB."""
    n = ctypes.c_size_t(0)
    T.call("tb_packed_quant_weights_bytes", T.Q4_0, 300, 512, ctypes.byref(n))
    assert n.value == 384 * 512 * 4 + 3072
    T.call("tb_packed_quant_weights_bytes", T.Q8_0, 128, 256, ctypes.byref(n))
    assert n.value == 128 * 256 * 4 + 1024
    for dt, N, K in [(T.Q4_0, 300, 480), (T.Q4_0, 0, 512), (T.F32, 128, 256), (T.Q8_0, 128, 0)]:
        with pytest.raises(T.TbError) as e:
            T.call("tb_packed_quant_weights_bytes", dt, N, K, ctypes.byref(n))
        assert e.value.status == T.EINVAL

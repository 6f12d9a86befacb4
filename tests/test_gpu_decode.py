"""The Llama-3.2-1B-shaped Q8_0 greedy decode through the C++ host layer
(MiniGPT over the device Tensor) against the reference MiniGPT's token ids.

tests/golden/decode_1b.npz holds the reference run (tests/golden/
make_decode_golden.py): prefill of 512 seeded ids, then 128 greedy steps.  The
same synthetic GGUF is regenerated here from its seed.
"""
import os

import numpy as np
import pytest

from turbo_b200 import gguf_synth

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "decode_1b.npz")
MODEL = "/tmp/turbo_b200_llama1b_q8_0_seed0.gguf"


@pytest.fixture(scope="module")
def model_path():
    if not os.path.exists(MODEL):
        gguf_synth.write_model(MODEL + ".part")
        os.replace(MODEL + ".part", MODEL)
    return MODEL


@pytest.fixture(scope="module")
def golden():
    if not os.path.exists(GOLDEN):
        pytest.skip("decode golden fixture not generated")
    return np.load(GOLDEN)


@pytest.mark.parametrize("exact", [True, False])
def test_decode_token_ids_match_reference(model_path, golden, exact):
    from turbo_b200.model import Model
    m = Model(model_path, exact=exact)
    steps = int(golden["steps"])
    out = m.generate(golden["prompt"], steps, max_seq=int(golden["max_seq"]))
    m.close()
    ref_ids = golden["ids"]
    ref_margin = golden["margins"]
    first_bad = np.nonzero(out["ids"] != ref_ids)[0]
    info = "prefill %.1f ms, decode %.1f ms (%.1f tok/s); min ref margin %.3g" % (
        out["prefill_ms"], out["decode_ms"], steps / (out["decode_ms"] / 1e3), ref_margin.min())
    print(info)
    assert first_bad.size == 0, "first differing step %d (ref margin there %.3g, ours %.3g); %s" % (
        first_bad[0], ref_margin[first_bad[0]], out["margins"][first_bad[0]], info)
    # the chosen logits' margins agree closely too
    assert np.max(np.abs(out["margins"] - ref_margin)) < 1e-3

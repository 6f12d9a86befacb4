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


@pytest.fixture(scope="module")
def model_path():
    return gguf_synth.ensure_model()


@pytest.fixture(scope="module")
def golden():
    if not os.path.exists(GOLDEN):
        pytest.skip("decode golden fixture not generated")
    return np.load(GOLDEN)


# exact: the bit-identical kernels, one per reference op; fused: one CUDA graph
# per token of fused per-op kernels; persistent: one kernel per token
@pytest.mark.parametrize("path", ["exact", "fused", "persistent"])
def test_decode_token_ids_match_reference(model_path, golden, path):
    from turbo_b200.model import Model
    m = Model(model_path, exact=path == "exact", persistent=path == "persistent")
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


# ---- sampled decode (generate_text with temperature > 0) -----------------------
# The graph samples each token on the device with the uniform number of its
# position.  With u = 0 the draw is the most probable token and with a tiny
# top_p the nucleus is that token alone, so both runs reproduce the reference's
# greedy ids; a run with random uniform numbers is reproducible from them.

STEPS_SAMPLED = 32


@pytest.mark.parametrize("exact", [False, True])
def test_sampled_decode_u0_is_greedy(model_path, golden, exact):
    from turbo_b200.model import Model
    m = Model(model_path, exact=exact)
    n = STEPS_SAMPLED
    out = m.generate(golden["prompt"], n, max_seq=int(golden["max_seq"]), temperature=0.8, top_p=0.9,
                     uniforms=np.zeros(n + 1))
    tiny = m.generate(golden["prompt"], n, max_seq=int(golden["max_seq"]), temperature=0.8, top_p=1e-6,
                      uniforms=np.random.default_rng(1).random(n + 1))
    m.close()
    assert np.array_equal(out["ids"], golden["ids"][:n + 1])
    assert np.array_equal(tiny["ids"], golden["ids"][:n + 1])


def test_sampled_decode_reproducible(model_path, golden):
    from turbo_b200.model import Model
    m = Model(model_path, exact=False)
    n = STEPS_SAMPLED
    us = np.random.default_rng(7).random(n + 1)
    a = m.generate(golden["prompt"], n, max_seq=int(golden["max_seq"]), temperature=0.8, top_p=0.9, uniforms=us)
    b = m.generate(golden["prompt"], n, max_seq=int(golden["max_seq"]), temperature=0.8, top_p=0.9, uniforms=us)
    m.close()
    assert np.array_equal(a["ids"], b["ids"])
    assert ((a["ids"] >= 0) & (a["ids"] < 128256)).all()
    print("sampled ids", a["ids"][:12], "decode %.1f ms" % a["decode_ms"])


@pytest.mark.parametrize("exact", [False, True])
def test_sampled_decode_reads_each_positions_uniform(model_path, golden, exact):
    # u = 0 draws the greedy id at every step but one, s_star, whose u just
    # below 1 draws the last id of the 0.9 nucleus (never the top id: the
    # nucleus of this model's flat logits holds many ids).  The first step that
    # differs from the greedy ids must be s_star itself: a step that read its
    # neighbour's uniform number would move the deviation or miss it.
    from turbo_b200.model import Model
    m = Model(model_path, exact=exact)
    n = 10
    ref = golden["ids"]
    try:
        for s_star in ((0, 1, 2, 7, 10) if not exact else (1, 6)):
            us = np.zeros(n + 1)
            us[s_star] = 1.0 - 1e-9
            out = m.generate(golden["prompt"], n, max_seq=int(golden["max_seq"]), temperature=0.8, top_p=0.9,
                             uniforms=us, want_margins=False)
            ids = out["ids"]
            assert np.array_equal(ids[:s_star], ref[:s_star]), (s_star, ids[:s_star + 1], ref[:s_star + 1])
            assert ids[s_star] != ref[s_star], (s_star, ids[s_star])
    finally:
        m.close()

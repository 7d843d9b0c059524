"""The oracle pinned against the golden fixtures (tests/golden/make_golden.py):
gguf's codec for the block formats, a float64 matmul over gguf-dequantized
weights for mul_mat_id, and the reference ExpertCache for remap traces.
Also checks the host streamer against the recorded reference trace (works
without oracle/_ref)."""
import os

import numpy as np

from oracle import oracle as O

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return np.load(os.path.join(GOLD, name))


def test_mxfp4_quantize_matches_gguf():
    g = load("mxfp4_gguf.npz")
    assert np.array_equal(O.quantize("mxfp4", g["x"]).reshape(g["q"].shape), g["q"])


def test_mxfp4_dequantize_matches_gguf():
    g = load("mxfp4_gguf.npz")
    assert np.array_equal(O.dequantize("mxfp4", g["q"], g["x"].shape[1]), g["dq"])


def test_iq4nl_dequantize_matches_gguf():
    g = load("iq4nl_gguf.npz")
    got = O.dequantize("iq4_nl", g["q"], g["dq"].shape[1])
    assert np.array_equal(got, g["dq"])


def test_iq4nl_quantizer_round_trip_is_close():
    """This library's IQ4_NL quantizer (no gguf counterpart): dequantized
    error within half a codebook step of the block scale."""
    rng = np.random.default_rng(0)
    x = rng.normal(0, 0.02, size=(64, 256)).astype(np.float32)
    q = O.quantize("iq4_nl", x)
    d = O.dequantize("iq4_nl", q, 256)
    rel = np.sqrt(np.mean((d - x) ** 2) / np.mean(x ** 2))
    assert rel < 0.12
    # zero blocks stay exactly zero
    z = O.dequantize("iq4_nl", O.quantize("iq4_nl", np.zeros((1, 32), np.float32)), 32)
    assert np.all(z == 0)


def test_mul_mat_id_exact_matches_golden():
    g = load("mmid_exact.npz")
    got = O.mul_mat_id("mxfp4", g["slab"], int(g["K"]), int(g["N"]), g["b"], g["ids"],
                       mode="exact")
    assert O.max_abs_normalized(got, g["res"]) < 1e-6
    q8 = O.mul_mat_id("mxfp4", g["slab"], int(g["K"]), int(g["N"]), g["b"], g["ids"], mode="q8")
    assert O.max_abs_normalized(q8, g["res"]) < 1e-2


def test_q8_quantization_form():
    """ggml q8_0: d = amax/127 stored as fp16, codes from the unrounded d."""
    x = np.linspace(-1.0, 1.0, 32, dtype=np.float32)
    q, d = O.quantize_q8(x)
    assert q.max() == 127 and q.min() == -127
    assert d[0] == np.float32(np.float16(1.0 / 127))


def _replay(fn):
    g = load("remap_ref_trace.npz")
    top_k = int(g["top_k"])
    i = j = 0
    for c, n in enumerate(g["sizes"]):
        ids = g["ids"][i:i + n * top_k].reshape(n, top_k)
        out, pend = fn(ids)
        assert np.array_equal(out.reshape(-1), g["out"][i:i + n * top_k]), c
        npend = int(g["npend"][c])
        assert [tuple(p) for p in g["pend"][j:j + npend].tolist()] == [tuple(p) for p in pend], c
        i += n * top_k
        j += npend
    return g


def test_streamer_matches_recorded_reference_trace():
    from moestream_b200 import SlotStreamer
    g = load("remap_ref_trace.npz")
    st = SlotStreamer(1, int(g["n_expert"]), int(g["n_slot"]), 1000)
    _replay(lambda ids: st.remap(0, ids)[:2])
    s = st.stats()
    want = g["stats"].tolist()
    assert [s[k] for k in O.STATS_FIELDS] + [s["exhausted"]] == want


def test_reference_remap_matches_recorded_trace():
    if not O.ref_available():
        import pytest
        pytest.skip("oracle/_ref not built")
    g = load("remap_ref_trace.npz")
    r = O.RefRemap(int(g["n_expert"]), int(g["n_slot"]), 1000)
    _replay(r)


def test_oracle_gpt_oss_activation_follows_the_formula():
    """The oracle's gpt-oss activation (moe_ffn act=(alpha, limit)) equals
    the formula evaluated in numpy on the oracle's own gate and up
    projections: x = min(g, limit), y = clamp(u, -limit, limit),
    h = x * sigmoid(alpha * x) * (y + 1). Activations are scaled so that both
    clamps are active for some elements."""
    from tests.helpers import experts
    K, n_ff, E, T, top_k = 256, 64, 4, 3, 2
    gate = experts("mxfp4", E, K, n_ff, seed=1)
    up = experts("mxfp4", E, K, n_ff, seed=2)
    down = experts("mxfp4", E, n_ff, K, seed=3)
    rng = np.random.default_rng(4)
    x = (40 * rng.normal(0, 1, size=(T, K))).astype(np.float32)
    ids = np.array([[0, 1], [2, 3], [1, 2]], dtype=np.int32)
    w = np.full((T, top_k), 0.5, dtype=np.float32)
    g = O.mul_mat_id("mxfp4", gate, K, n_ff, x[:, None, :], ids, mode="exact")
    u = O.mul_mat_id("mxfp4", up, K, n_ff, x[:, None, :], ids, mode="exact")
    alpha, limit = 1.702, 7.0
    xg = np.minimum(g, limit).astype(np.float64)
    yu = np.clip(u, -limit, limit).astype(np.float64)
    want = xg / (1 + np.exp(-alpha * xg)) * (yu + 1)
    assert (g > limit).any() and (u < -limit).any() and (u > limit).any()
    _, h = O.moe_ffn("mxfp4", gate, up, down, K, n_ff, x, ids, w, mode="exact",
                     act=(alpha, limit))
    assert np.abs(h - want).max() <= 1e-5 * np.abs(want).max()

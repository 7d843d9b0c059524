"""Generates the golden fixtures in this directory.

Sources (never this project's own code, so the fixtures pin the oracle):
  - gguf 0.19.0, ggml's Python codec (quants.py: MXFP4 quantize/dequantize,
    IQ4_NL dequantize), for the block formats;
  - numpy float64 matmul over gguf-dequantized weights, for mul_mat_id's
    exact result;
  - the reference's own ExpertCache compiled from its source
    (oracle/_ref/libref_cache.so, built by oracle/Makefile) driven through the
    restated ms_remap_fn loop, for remap traces.

Run from the repository root: python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)


def mxfp4():
    import gguf
    from gguf import quants
    rng = np.random.default_rng(2024)
    x = rng.normal(0.0, 0.02, size=(24, 128)).astype(np.float32)
    x[0, :32] = 0.0                      # all-zero block -> e = 0
    x[1, :32] = np.linspace(-0.1, 0.1, 32)
    x[2, 32:64] *= 1000.0                # large scale
    x[3, 64:96] = 0.015                  # constant block
    x[4, :32] = [0.5 * k for k in range(-16, 16)]  # ties between codes
    q = quants.quantize(x, gguf.GGMLQuantizationType.MXFP4)
    d = quants.dequantize(q, gguf.GGMLQuantizationType.MXFP4)
    return dict(x=x, q=q.reshape(x.shape[0], -1), dq=d.reshape(x.shape))


def iq4nl():
    import gguf
    from gguf import quants
    rng = np.random.default_rng(7)
    n_rows, K = 16, 128
    nb = K // 32
    blocks = rng.integers(0, 256, size=(n_rows * nb, 18), dtype=np.uint8)
    d = rng.normal(0, 1e-4, size=n_rows * nb).astype(np.float16)
    d[0] = np.float16(0.0)
    d[1] = np.float16(6.1e-5)  # near the fp16 normal boundary
    d[2] = np.float16(-3.0e-7)  # subnormal
    blocks[:, :2] = d.view(np.uint8).reshape(-1, 2)
    q = blocks.reshape(n_rows, -1)
    dq = quants.dequantize(q, gguf.GGMLQuantizationType.IQ4_NL)
    return dict(q=q, dq=dq.reshape(n_rows, K))


def mmid():
    """Exact mul_mat_id over gguf-dequantized MXFP4 weights: res[t, k, n]."""
    import gguf
    from gguf import quants
    rng = np.random.default_rng(11)
    K, N, n_slots, T, top_k = 256, 48, 5, 3, 2
    w = rng.normal(0, 0.02, size=(n_slots * N, K)).astype(np.float32)
    q = quants.quantize(w, gguf.GGMLQuantizationType.MXFP4)
    wd = quants.dequantize(q, gguf.GGMLQuantizationType.MXFP4).reshape(n_slots, N, K)
    b = rng.normal(0, 1, size=(T, 1, K)).astype(np.float32)
    ids = rng.integers(0, n_slots, size=(T, top_k)).astype(np.int32)
    res = np.einsum("tkni,ti->tkn", wd[ids].astype(np.float64), b[:, 0].astype(np.float64))
    return dict(slab=q.reshape(n_slots, -1), b=b, ids=ids, res=res, K=K, N=N)


def remap():
    from oracle import oracle as O
    assert O.ref_available(), "build oracle/_ref first (make -C oracle)"
    rng = np.random.default_rng(5)
    n_expert, n_slot, top_k = 128, 32, 4
    r = O.RefRemap(n_expert, n_slot, 1000)
    sizes = [1, 4, 16, 1, 1, 4, 16, 2, 8, 1] * 3
    ids_all, out_all, pend_all, ncalls = [], [], [], []
    for n in sizes:
        ids = np.stack([rng.permutation(n_expert)[:top_k] for _ in range(n)]).astype(np.int32)
        out, pend = r(ids)
        ids_all.append(ids.reshape(-1))
        out_all.append(out.reshape(-1))
        pend_all.append(np.array(pend, dtype=np.int32).reshape(-1, 2))
        ncalls.append(len(pend))
    st = r.stats()
    return dict(sizes=np.array(sizes, np.int32), ids=np.concatenate(ids_all),
                out=np.concatenate(out_all), pend=np.concatenate(pend_all),
                npend=np.array(ncalls, np.int32), n_expert=n_expert, n_slot=n_slot,
                top_k=top_k, stats=np.array([st[k] for k in O.STATS_FIELDS] +
                                            [st["exhausted"]], dtype=np.uint64))


def main():
    np.savez_compressed(os.path.join(HERE, "mxfp4_gguf.npz"), **mxfp4())
    np.savez_compressed(os.path.join(HERE, "iq4nl_gguf.npz"), **iq4nl())
    np.savez_compressed(os.path.join(HERE, "mmid_exact.npz"), **mmid())
    np.savez_compressed(os.path.join(HERE, "remap_ref_trace.npz"), **remap())
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()

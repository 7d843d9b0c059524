"""Seeded synthetic inputs shared by the tests (weights N(0, 0.02) quantized by
the oracle, activations N(0, 1), router logits N(0, 1))."""
import numpy as np

from oracle import oracle as O


def experts(wtype, n, K, N, seed):
    """n experts of shape [N rows, K] -> uint8 [n, expert_bytes] (ggml layout)."""
    rng = np.random.default_rng(seed)
    w = rng.normal(0.0, 0.02, size=(n * N, K)).astype(np.float32)
    return O.quantize(wtype, w).reshape(n, -1)


def topk_ids(rng, n_tok, n_expert, top_k, bias=None):
    logits = rng.normal(0.0, 1.0, size=(n_tok, n_expert))
    if bias is not None:
        logits = logits + bias
    ids = np.argsort(-logits, axis=1, kind="stable")[:, :top_k].astype(np.int32)
    sel = np.take_along_axis(logits, ids, axis=1)
    w = np.exp(sel - sel.max(axis=1, keepdims=True))
    w = (w / w.sum(axis=1, keepdims=True)).astype(np.float32)
    return ids, w


def zipf_bias(rng, n_expert, s=1.1):
    """log p_e with p_e proportional to rank^-s over a seeded permutation."""
    ranks = rng.permutation(n_expert) + 1
    p = ranks.astype(np.float64) ** (-s)
    return np.log(p / p.sum())


def write_gguf(path, tensors, kvs=(), arch="gpt-oss", split_max_tensors=0, alignment=None):
    """Writes a GGUF with the gguf package's writer (an implementation
    independent of the library's parser). tensors: [(name, array, ggml type
    or None)]; quantized arrays are uint8 [..., row bytes]. kvs: [(method of
    GGUFWriter, args...)]. Returns the paths written, shard order."""
    import os

    from gguf import GGUFWriter
    w = GGUFWriter(str(path), arch, split_max_tensors=split_max_tensors)
    if alignment is not None:
        w.add_custom_alignment(alignment)
    for method, *args in kvs:
        getattr(w, method)(*args)
    for name, arr, raw in tensors:
        w.add_tensor(name, arr, raw_dtype=raw)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    d, base = os.path.split(str(path))
    stem = base[:-5] if base.endswith(".gguf") else base
    if split_max_tensors:
        return sorted(os.path.join(d, f) for f in os.listdir(d)
                      if f.startswith(stem + "-") and f.endswith(".gguf"))
    return [str(path)]

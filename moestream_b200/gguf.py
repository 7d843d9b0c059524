"""GGUF expert source over the C ABI (msb_gguf_*).

Opens a GGUF model file (every shard of a split one), exposes the tensor
table and the integer metadata the slot sizing needs, and reads expert byte
ranges either into caller memory or, through pinned staging owned by the
handle, straight into slots of a SlotPool. Mirrors the reference's own
reads (src/llama-moestream.cpp:571-598 shard naming, :610-693 metadata by
key suffix, :1230-1263 per-expert pread spread over threads).
"""
import ctypes

import numpy as np
import torch

from ._lib import GgufTensor, MsbError, c_vp, check, lib

ROLES = {"gate": 0, "up": 1, "down": 2}


def _stream(stream):
    if stream is None:
        return c_vp(torch.cuda.current_stream().cuda_stream)
    return c_vp(stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream))


class GGUFFile:
    """An open GGUF; close() (or the context manager) releases the files and
    the pinned staging memory."""

    def __init__(self, path):
        h = c_vp()
        check(lib().msb_gguf_open(str(path).encode(), ctypes.byref(h)))
        self.handle = h
        self.n_shard = int(lib().msb_gguf_shard_count(h))
        self.tensors = []
        for i in range(int(lib().msb_gguf_tensor_count(h))):
            t = GgufTensor()
            check(lib().msb_gguf_tensor_info(h, i, ctypes.byref(t)))
            self.tensors.append({"name": t.name.decode(), "type": t.type, "n_dims": t.n_dims,
                                 "ne": tuple(t.ne[:t.n_dims]), "shard": t.shard,
                                 "offset": t.offset, "nbytes": t.nbytes})
        self._by_name = {t["name"]: i for i, t in enumerate(self.tensors)}

    def close(self):
        if self.handle:
            check(lib().msb_gguf_close(self.handle))
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def kv_int(self, key_suffix):
        """First integer metadata value whose key ends in key_suffix, or None."""
        v = ctypes.c_int64()
        if lib().msb_gguf_kv_int(self.handle, key_suffix.encode(), ctypes.byref(v)) != 0:
            return None
        return v.value

    def bytes_per_slot(self):
        return int(lib().msb_gguf_bytes_per_slot(self.handle))

    def index(self, name):
        return self._by_name.get(name, -1)

    def expert_tensor(self, layer, role):
        """Index of blk.<layer>.ffn_<role>_exps.weight, -1 if absent."""
        return int(lib().msb_gguf_expert_tensor(self.handle, layer, ROLES.get(role, role)))

    def expert_bytes(self, tensor):
        t = self.tensors[tensor]
        return t["nbytes"] // t["ne"][2]

    def read_experts(self, tensor, experts, n_threads=4):
        """Expert byte ranges of a 3-D tensor as numpy uint8 arrays."""
        experts = [int(e) for e in experts]
        n = len(experts)
        eb = self.expert_bytes(tensor)
        out = np.empty((n, eb), dtype=np.uint8)
        ids = (ctypes.c_int32 * max(n, 1))(*experts)
        dst = (c_vp * max(n, 1))(*[out[i].ctypes.data for i in range(n)])
        check(lib().msb_gguf_read_experts(self.handle, tensor, n, ids, dst, n_threads))
        return out

    def fill_slots(self, tensor, pool, experts, slots, n_threads=4, stream=None):
        """Reads the experts and fills the pool's slots with them
        (stream-ordered; the reads themselves finish before this returns)."""
        experts = [int(e) for e in experts]
        slots = [int(s) for s in slots]
        if len(experts) != len(slots):
            raise MsbError("fill_slots: one slot per expert")
        n = len(experts)
        ids = (ctypes.c_int32 * max(n, 1))(*experts)
        sl = (ctypes.c_int32 * max(n, 1))(*slots)
        check(lib().msb_gguf_fill_slots_async(self.handle, tensor, pool.handle, n, ids, sl,
                                              n_threads, _stream(stream)))


class ExpertArena:
    """Per-layer device arenas holding every expert of a layer, loaded from a
    GGUF (msb_arena_*): the prefill path for micro-batches whose expert union
    exceeds the slots. Route a batch with ops.remap_group(ids, n_expert)
    (no table: slot e is expert e) and run the FFN over the pools of
    ready(). One thread drives it; the background load is the library's."""

    def __init__(self, path, n_buf=2, n_threads=4):
        h = c_vp()
        check(lib().msb_arena_create(str(path).encode(), n_buf, n_threads, ctypes.byref(h)))
        self.handle = h
        nl, ne, nb = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
        check(lib().msb_arena_info(h, ctypes.byref(nl), ctypes.byref(ne), ctypes.byref(nb)))
        self.n_layer, self.n_expert, self.n_buf = nl.value, ne.value, nb.value

    def close(self):
        if self.handle:
            check(lib().msb_arena_destroy(self.handle))
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _mask(self, need):
        """uint8 mask over experts from expert ids or a boolean mask; None stays None."""
        if need is None:
            return None, None
        need = np.asarray(need)
        if need.dtype == bool:
            m = need.astype(np.uint8)
            assert m.shape == (self.n_expert,)
        else:
            m = np.zeros(self.n_expert, dtype=np.uint8)
            m[need.astype(np.int64).ravel()] = 1
        return m, c_vp(m.ctypes.data)

    def load(self, layer, need=None, stream=None):
        """need: experts to hold (ids or a boolean mask over experts); None = all."""
        m, p = self._mask(need)
        check(lib().msb_arena_load(self.handle, layer, p, _stream(stream)))

    def prefetch(self, layer, hint=None, stream=None):
        m, p = self._mask(hint)
        check(lib().msb_arena_prefetch(self.handle, layer, p, _stream(stream)))

    def wait(self):
        check(lib().msb_arena_wait(self.handle))

    def ready(self, layer, stream=None):
        """(gate, up, down) pools of the layer, the stream made to wait for them."""
        from .ops import SlotPool
        g, u, d = c_vp(), c_vp(), c_vp()
        check(lib().msb_arena_ready(self.handle, layer, _stream(stream), ctypes.byref(g),
                                    ctypes.byref(u), ctypes.byref(d)))
        return SlotPool.borrowed(g), SlotPool.borrowed(u), SlotPool.borrowed(d)

    def release(self, layer, stream=None):
        check(lib().msb_arena_release(self.handle, layer, _stream(stream)))

    def stats(self):
        from ._lib import ArenaStats
        st = ArenaStats()
        check(lib().msb_arena_stats(self.handle, ctypes.byref(st)))
        return st.as_dict()

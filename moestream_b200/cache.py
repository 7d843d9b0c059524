"""Host expert cache and slot streamer over the C ABI.

ExpertCache mirrors the reference class moestream::ExpertCache
(src/expert_cache.hpp:61-147): same constructor config, same acquire /
mark_resident / release / end_step / build_pinned methods and the same
decisions. SlotStreamer is the host half of the reference's ms_remap_fn
(src/llama-moestream.cpp:1799-2105): per-layer caches, reference release on
the next call, misses in first-seen order, zero slot on exhaustion.
"""
import ctypes

import numpy as np

from ._lib import (CacheConfig, CacheStats, NO_SLOT, ORIGIN_DEMAND, c_i32p, c_u32p, c_vp,
                   check, lib)


class ExpertCache:
    def __init__(self, n_layer=40, n_expert=256, n_slot=0, **kw):
        cfg = CacheConfig()
        lib().msb_cache_config_default(ctypes.byref(cfg))
        cfg.n_layer, cfg.n_expert, cfg.n_slot = n_layer, n_expert, n_slot
        for k, v in kw.items():
            setattr(cfg, k, int(v) if k == "layer_quota_adapt" else v)
        h = c_vp()
        check(lib().msb_cache_create(ctypes.byref(cfg), ctypes.byref(h)))
        self.h = h
        self.n_layer = n_layer

    def __del__(self):
        if getattr(self, "h", None):
            lib().msb_cache_destroy(self.h)
            self.h = None

    def acquire(self, layer, expert, origin=ORIGIN_DEMAND):
        """Returns (hit, slot); slot is NO_SLOT when none was reserved."""
        s = ctypes.c_uint32(0)
        hit = lib().msb_cache_acquire(self.h, layer, expert, origin, ctypes.byref(s))
        return bool(hit), int(s.value)

    def mark_resident(self, layer, expert, nbytes):
        lib().msb_cache_mark_resident(self.h, layer, expert, nbytes)

    def release(self, layer, expert):
        lib().msb_cache_release(self.h, layer, expert)

    def end_step(self):
        lib().msb_cache_end_step(self.h)

    def build_pinned(self, freq):
        a = np.ascontiguousarray(freq, dtype=np.uint32)
        lib().msb_cache_build_pinned(self.h, a.ctypes.data_as(c_u32p), a.size)

    def stats(self):
        st = CacheStats()
        lib().msb_cache_get_stats(self.h, ctypes.byref(st))
        return st.as_dict()

    @property
    def n_slot(self):
        return int(lib().msb_cache_n_slot(self.h))

    def slot_of(self, layer, expert):
        return int(lib().msb_cache_slot_of(self.h, layer, expert))

    def layer_quota(self):
        out = np.zeros(self.n_layer, dtype=np.uint32)
        lib().msb_cache_layer_quota(self.h, out.ctypes.data_as(c_u32p))
        return out


class SlotStreamer:
    def __init__(self, n_layer, n_expert, n_slot, expert_bytes_total=0):
        h = c_vp()
        check(lib().msb_streamer_create(n_layer, n_expert, n_slot, expert_bytes_total,
                                        ctypes.byref(h)))
        self.h = h
        self.n_expert, self.n_slot = n_expert, n_slot

    def __del__(self):
        if getattr(self, "h", None):
            lib().msb_streamer_destroy(self.h)
            self.h = None

    def remap(self, layer, ids, want_table=False):
        """ids: int32 array [n_tok, top_k] (any strides). Returns
        (slots [n_tok, top_k], misses [(expert, slot)], table or None)."""
        ids = np.asarray(ids)
        assert ids.dtype == np.int32 and ids.ndim == 2
        n_tok, top_k = ids.shape
        nb0, nb1 = ids.strides[1], ids.strides[0]
        out = np.empty((n_tok, top_k), dtype=np.int32)
        me = np.empty(max(n_tok * top_k, 1), dtype=np.int32)
        ms = np.empty_like(me)
        nm = ctypes.c_int32(0)
        table = np.empty(self.n_expert, dtype=np.int32) if want_table else None
        base = ids.__array_interface__["data"][0]
        check(lib().msb_streamer_remap(
            self.h, layer, ctypes.cast(base, c_i32p), nb0, nb1, top_k, n_tok,
            out.ctypes.data_as(c_i32p), ctypes.byref(nm), me.ctypes.data_as(c_i32p),
            ms.ctypes.data_as(c_i32p),
            table.ctypes.data_as(c_i32p) if table is not None else None))
        misses = list(zip(me[:nm.value].tolist(), ms[:nm.value].tolist()))
        return out, misses, table

    def stats(self):
        st = CacheStats()
        ex = ctypes.c_uint64(0)
        check(lib().msb_streamer_stats(self.h, ctypes.byref(st), ctypes.byref(ex)))
        d = st.as_dict()
        d["exhausted"] = int(ex.value)
        return d


class DeviceSlotStreamer:
    """The SlotStreamer's decisions made on the device (msb_dstreamer_*):
    cache state in device memory, the miss queue in mapped pinned memory,
    and a fill kernel that copies missed experts from pinned host memory, so
    a decode step needs no host round trip. on_host=True runs the same
    decision code on the host (numpy ids and slots; no fills)."""

    def __init__(self, n_layer, n_expert, n_slot, max_pairs, expert_bytes_total=0,
                 on_host=False):
        h = c_vp()
        check(lib().msb_dstreamer_create(n_layer, n_expert, n_slot, max_pairs,
                                         expert_bytes_total, 1 if on_host else 0,
                                         ctypes.byref(h)))
        self.h = h
        self.n_layer, self.n_expert, self.n_slot = n_layer, n_expert, n_slot
        self.max_pairs, self.on_host = max_pairs, on_host

    def close(self):
        if getattr(self, "h", None):
            check(lib().msb_dstreamer_destroy(self.h))
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def remap(self, layer, ids, out=None, stream=None):
        """ids: int32 [n_tok, top_k] (numpy on a host streamer, a device tensor
        otherwise; any strides). Returns the slots [n_tok, top_k]."""
        if self.on_host:
            ids = np.asarray(ids)
            assert ids.dtype == np.int32 and ids.ndim == 2
            n_tok, top_k = ids.shape
            if out is None:
                out = np.empty((n_tok, top_k), dtype=np.int32)
            nb0, nb1 = ids.strides[1], ids.strides[0]
            base, dst, st = ids.__array_interface__["data"][0], out.ctypes.data, None
        else:
            import torch
            assert ids.dtype == torch.int32 and ids.is_cuda and ids.dim() == 2
            n_tok, top_k = ids.shape
            if out is None:
                out = torch.empty(n_tok, top_k, dtype=torch.int32, device=ids.device)
            nb0, nb1 = ids.stride(1) * 4, ids.stride(0) * 4
            base, dst = ids.data_ptr(), out.data_ptr()
            st = stream if stream is not None else torch.cuda.current_stream()
            st = st.cuda_stream
        check(lib().msb_dstreamer_remap(self.h, layer, c_vp(base), nb0, nb1, top_k, n_tok,
                                        c_vp(dst), c_vp(st)))
        return out

    def fill(self, layer, pool, src, stream=None):
        """src: uint8 [n_expert, stride] tensor of ggml-layout experts, pinned
        host memory or device memory."""
        import torch
        assert src.dtype == torch.uint8 and src.dim() == 2 and src.stride(1) == 1
        assert src.shape[0] >= self.n_expert and src.shape[1] >= pool.expert_bytes
        assert src.is_cuda or src.is_pinned()
        st = stream if stream is not None else torch.cuda.current_stream()
        check(lib().msb_dstreamer_fill(self.h, layer, pool.handle, c_vp(src.data_ptr()),
                                       src.stride(0), c_vp(st.cuda_stream)))

    def fill_roles(self, layer, pools, srcs, stream=None):
        """fill() of several roles (pools[i] from srcs[i]) in one launch."""
        import torch
        n = len(pools)
        assert n == len(srcs) and 1 <= n <= 3
        for p, src in zip(pools, srcs):
            assert src.dtype == torch.uint8 and src.dim() == 2 and src.stride(1) == 1
            assert src.shape[0] >= self.n_expert and src.shape[1] >= p.expert_bytes
            assert src.is_cuda or src.is_pinned()
        st = stream if stream is not None else torch.cuda.current_stream()
        hp = (c_vp * n)(*[p.handle.value for p in pools])
        sp = (c_vp * n)(*[src.data_ptr() for src in srcs])
        strides = (ctypes.c_int64 * n)(*[src.stride(0) for src in srcs])
        check(lib().msb_dstreamer_fill_roles(self.h, layer, n, hp, sp, strides,
                                             c_vp(st.cuda_stream)))

    def misses(self, layer):
        """[(expert, slot)] of the layer's last remap (after it completed)."""
        me = np.empty(self.max_pairs, dtype=np.int32)
        ms = np.empty(self.max_pairs, dtype=np.int32)
        n = ctypes.c_int32(0)
        check(lib().msb_dstreamer_misses(self.h, layer, ctypes.byref(n),
                                         me.ctypes.data_as(c_i32p), ms.ctypes.data_as(c_i32p)))
        return list(zip(me[:n.value].tolist(), ms[:n.value].tolist()))

    def table(self, layer):
        t = np.empty(self.n_expert, dtype=np.int32)
        check(lib().msb_dstreamer_table(self.h, layer, t.ctypes.data_as(c_i32p)))
        return t

    def stats(self):
        st = CacheStats()
        ex = ctypes.c_uint64(0)
        check(lib().msb_dstreamer_stats(self.h, ctypes.byref(st), ctypes.byref(ex)))
        d = st.as_dict()
        d["exhausted"] = int(ex.value)
        return d


__all__ = ["ExpertCache", "SlotStreamer", "DeviceSlotStreamer", "NO_SLOT"]

"""ctypes binding of libmsb.so (declarations in include/msb.h).

The library is built in-tree by moestream_b200/csrc/build.py. Loading fails
loudly when it is missing: there is no fallback implementation.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmsb.so")

TYPE_F32 = 0
TYPE_F16 = 1
TYPE_IQ4_NL = 20
TYPE_BF16 = 30
TYPE_MXFP4 = 39

ORIGIN_DEMAND, ORIGIN_PREFETCH_HIGH, ORIGIN_PREFETCH_LOW, ORIGIN_SWEEP = 0, 1, 2, 3
NO_SLOT = 0xFFFFFFFF
OPT_MXFP4_PATH = 1
OPT_WAIT_LIMIT_US = 2
OPT_WIDE_PASSES = 3
OPT_IQ4NL_PATH = 4
ROUTER_SOFTMAX_TOPK, ROUTER_SOFTMAX_ALL = 0, 1

c_i32p = ctypes.POINTER(ctypes.c_int32)
c_u32p = ctypes.POINTER(ctypes.c_uint32)
c_u64p = ctypes.POINTER(ctypes.c_uint64)
c_vp = ctypes.c_void_p


class MsbError(RuntimeError):
    pass


class PoolInfo(ctypes.Structure):
    _fields_ = [("wtype", ctypes.c_int), ("K", ctypes.c_int64), ("N", ctypes.c_int64),
                ("n_slot", ctypes.c_int32), ("device", ctypes.c_int32),
                ("expert_bytes", ctypes.c_int64), ("slot_stride", ctypes.c_int64),
                ("data", c_vp)]


EP_MAX_RANKS = 8
EP_HANDLE_BYTES = 64


class EpPeers(ctypes.Structure):
    _fields_ = [("n_rank", ctypes.c_int32), ("rank", ctypes.c_int32), ("cap", ctypes.c_int32),
                ("K", ctypes.c_int64), ("peer", c_vp * EP_MAX_RANKS)]


class GgufTensor(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("type", ctypes.c_int), ("n_dims", ctypes.c_int),
                ("ne", ctypes.c_int64 * 4), ("shard", ctypes.c_int32), ("offset", ctypes.c_uint64),
                ("nbytes", ctypes.c_int64)]


class ArenaStats(ctypes.Structure):
    _fields_ = [(f, ctypes.c_uint64) for f in ("loads", "hits", "experts_asked", "experts_read",
                                                "bytes_read")]

    def as_dict(self):
        return {f: int(getattr(self, f)) for f, _ in self._fields_}


ACT_SILU, ACT_SWIGLU_OAI = 0, 1


class FfnActCfg(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int), ("alpha", ctypes.c_float), ("limit", ctypes.c_float)]


class FfnBiasCfg(ctypes.Structure):
    _fields_ = [("gate_b", c_vp), ("up_b", c_vp), ("down_b", c_vp), ("gate_ld", ctypes.c_int64),
                ("up_ld", ctypes.c_int64), ("down_ld", ctypes.c_int64), ("ids", c_vp),
                ("ids_nb0", ctypes.c_int64), ("ids_nb1", ctypes.c_int64),
                ("n_expert", ctypes.c_int32)]


class Route(ctypes.Structure):
    _fields_ = [("slot_ids", c_vp), ("counts", c_vp), ("offsets", c_vp),
                ("rows", c_vp), ("active", c_vp)]


class CacheConfig(ctypes.Structure):
    _fields_ = [("n_layer", ctypes.c_uint32), ("n_expert", ctypes.c_uint32),
                ("n_slot", ctypes.c_uint32), ("cache_frac", ctypes.c_double),
                ("pin_ratio", ctypes.c_double), ("small_ratio", ctypes.c_double),
                ("ghost_mult", ctypes.c_uint32), ("layer_quota_adapt", ctypes.c_int32),
                ("quota_period", ctypes.c_uint32), ("quota_eta", ctypes.c_double),
                ("quota_min", ctypes.c_uint32)]


STATS_FIELDS = ("hit", "miss", "hit_pinned", "hit_small", "hit_main", "ghost_hit",
                "admit", "evict", "bypass", "promote", "bytes_fetched")


class CacheStats(ctypes.Structure):
    _fields_ = [(f, ctypes.c_uint64) for f in STATS_FIELDS]

    def as_dict(self):
        return {f: int(getattr(self, f)) for f in STATS_FIELDS}


# name -> (restype, argtypes); every symbol declared in include/msb.h.
SIGNATURES = {
    "msb_version": (ctypes.c_int, []),
    "msb_last_error": (ctypes.c_char_p, []),
    "msb_expert_bytes": (ctypes.c_int64, [ctypes.c_int, ctypes.c_int64, ctypes.c_int64]),
    "msb_slab_slots": (ctypes.c_uint32, [ctypes.c_int64, ctypes.c_double, ctypes.c_int, ctypes.c_int]),
    "msb_arena_threshold": (ctypes.c_int, [ctypes.c_int64, ctypes.c_int, ctypes.c_uint32]),
    "msb_pool_create": (ctypes.c_int, [ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_int32,
                                       ctypes.c_int32, ctypes.POINTER(c_vp)]),
    "msb_pool_destroy": (ctypes.c_int, [c_vp]),
    "msb_pool_get_info": (ctypes.c_int, [c_vp, ctypes.POINTER(PoolInfo)]),
    "msb_fill_slots_async": (ctypes.c_int, [c_vp, ctypes.c_int32, c_i32p, ctypes.POINTER(c_vp), c_vp]),
    "msb_fill_slots_from_device_async": (ctypes.c_int, [c_vp, ctypes.c_int32, c_i32p,
                                                        ctypes.POINTER(c_vp), c_vp]),
    "msb_read_slot_async": (ctypes.c_int, [c_vp, ctypes.c_int32, c_vp, c_vp]),
    "msb_remap_group": (ctypes.c_int, [c_vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int32,
                                       ctypes.c_int32, c_vp, ctypes.c_int32, ctypes.c_int32,
                                       ctypes.POINTER(Route), c_vp]),
    "msb_workspace_bytes": (ctypes.c_int64, [ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                             ctypes.c_int32]),
    "msb_mul_mat_id": (ctypes.c_int, [c_vp, c_vp, ctypes.c_int, ctypes.c_int64, ctypes.c_int64,
                                      ctypes.c_int64, ctypes.POINTER(Route), ctypes.c_int32,
                                      ctypes.c_int32, c_vp, c_vp, ctypes.c_int64, c_vp]),
    "msb_mul_mat_id_noalloc": (ctypes.c_int, [c_vp, c_vp, ctypes.c_int, ctypes.c_int64,
                                              ctypes.c_int64, ctypes.c_int64,
                                              ctypes.POINTER(Route), ctypes.c_int32,
                                              ctypes.c_int32, c_vp, c_vp]),
    "msb_device_status": (ctypes.c_int, [c_i32p, ctypes.c_int32]),
    "msb_stream_check": (ctypes.c_int, [c_vp, ctypes.c_int32]),
    "msb_moe_ffn": (ctypes.c_int, [c_vp, c_vp, ctypes.c_int64, c_vp, c_vp, ctypes.c_int,
                                   ctypes.c_int64, ctypes.POINTER(Route), c_vp, ctypes.c_int32,
                                   ctypes.c_int32, c_vp, c_vp, c_vp, ctypes.c_int64, c_vp]),
    "msb_moe_ffn_act": (ctypes.c_int, [c_vp, c_vp, ctypes.c_int64, c_vp, c_vp, ctypes.c_int,
                                       ctypes.c_int64, ctypes.POINTER(Route), c_vp,
                                       ctypes.c_int32, ctypes.c_int32, c_vp, c_vp,
                                       ctypes.POINTER(FfnActCfg), c_vp, ctypes.c_int64, c_vp]),
    "msb_moe_ffn_ex": (ctypes.c_int, [c_vp, c_vp, ctypes.c_int64, c_vp, c_vp, ctypes.c_int,
                                      ctypes.c_int64, ctypes.POINTER(Route), c_vp,
                                      ctypes.c_int32, ctypes.c_int32, c_vp, c_vp,
                                      ctypes.POINTER(FfnActCfg), ctypes.POINTER(FfnBiasCfg),
                                      ctypes.c_int32, c_vp, ctypes.c_int64, c_vp]),
    "msb_ep_dispatch": (ctypes.c_int, [c_vp, c_vp, ctypes.c_int, ctypes.c_int64, ctypes.c_int32,
                                       ctypes.c_int32, ctypes.c_int64, ctypes.c_int32,
                                       ctypes.c_int32, ctypes.c_int32, c_vp, ctypes.c_int64,
                                       c_vp, ctypes.c_int64, c_vp, c_vp]),
    "msb_ep_buffer_bytes": (ctypes.c_int64, [ctypes.c_int32, ctypes.c_int32, ctypes.c_int64]),
    "msb_ep_row_bytes": (ctypes.c_int64, [ctypes.c_int64]),
    "msb_ep_yback_offset": (ctypes.c_int64, [ctypes.c_int32, ctypes.c_int32, ctypes.c_int64]),
    "msb_ep_buffer_create": (ctypes.c_int, [ctypes.c_int64, ctypes.POINTER(c_vp), c_vp]),
    "msb_ep_buffer_open": (ctypes.c_int, [c_vp, ctypes.POINTER(c_vp)]),
    "msb_ep_buffer_close": (ctypes.c_int, [c_vp]),
    "msb_ep_buffer_destroy": (ctypes.c_int, [c_vp]),
    "msb_ep_dispatch_peers": (ctypes.c_int, [ctypes.POINTER(EpPeers), c_vp, c_vp, ctypes.c_int,
                                             ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                             ctypes.c_int32, c_vp, c_vp]),
    "msb_ep_return_peers": (ctypes.c_int, [ctypes.POINTER(EpPeers), c_vp, c_vp]),
    "msb_ep_wait": (ctypes.c_int, [ctypes.POINTER(EpPeers), ctypes.c_int32, c_vp]),
    "msb_ep_remap_group": (ctypes.c_int, [ctypes.POINTER(EpPeers), ctypes.c_int32,
                                          ctypes.POINTER(Route), c_vp]),
    "msb_ep_moe_ffn_peers": (ctypes.c_int, [ctypes.POINTER(EpPeers), c_vp, c_vp, ctypes.c_int64,
                                            c_vp, ctypes.POINTER(Route), c_vp, ctypes.c_int64,
                                            c_vp]),
    "msb_ep_combine_peers": (ctypes.c_int, [ctypes.POINTER(EpPeers), c_vp, c_vp, ctypes.c_int32,
                                            ctypes.c_int32, c_vp, c_vp]),
    "msb_ep_combine": (ctypes.c_int, [c_vp, c_vp, c_vp, ctypes.c_int32, ctypes.c_int32,
                                      ctypes.c_int64, c_vp, c_vp]),
    "msb_kernel_launches": (ctypes.c_uint64, []),
    "msb_set_option": (ctypes.c_int, [ctypes.c_int, ctypes.c_int]),
    "msb_time_next_gate_up": (None, [c_vp, c_vp]),
    "msb_quantize_rows": (ctypes.c_int, [ctypes.c_int, c_vp, ctypes.c_int64, ctypes.c_int64,
                                         c_vp, c_vp]),
    "msb_cache_config_default": (None, [ctypes.POINTER(CacheConfig)]),
    "msb_cache_create": (ctypes.c_int, [ctypes.POINTER(CacheConfig), ctypes.POINTER(c_vp)]),
    "msb_cache_destroy": (None, [c_vp]),
    "msb_cache_acquire": (ctypes.c_int, [c_vp, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_int, c_u32p]),
    "msb_cache_mark_resident": (None, [c_vp, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint64]),
    "msb_cache_release": (None, [c_vp, ctypes.c_uint32, ctypes.c_uint32]),
    "msb_cache_end_step": (None, [c_vp]),
    "msb_cache_build_pinned": (None, [c_vp, c_u32p, ctypes.c_size_t]),
    "msb_cache_get_stats": (None, [c_vp, ctypes.POINTER(CacheStats)]),
    "msb_cache_n_slot": (ctypes.c_uint32, [c_vp]),
    "msb_cache_slot_of": (ctypes.c_uint32, [c_vp, ctypes.c_uint32, ctypes.c_uint32]),
    "msb_cache_layer_quota": (None, [c_vp, c_u32p]),
    "msb_streamer_create": (ctypes.c_int, [ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                                           ctypes.c_uint64, ctypes.POINTER(c_vp)]),
    "msb_streamer_destroy": (None, [c_vp]),
    "msb_streamer_remap": (ctypes.c_int, [c_vp, ctypes.c_uint32, c_i32p, ctypes.c_int64,
                                          ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, c_i32p,
                                          c_i32p, c_i32p, c_i32p, c_i32p]),
    "msb_streamer_stats": (ctypes.c_int, [c_vp, ctypes.POINTER(CacheStats), c_u64p]),
    "msb_gguf_open": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(c_vp)]),
    "msb_gguf_close": (ctypes.c_int, [c_vp]),
    "msb_gguf_shard_count": (ctypes.c_int32, [c_vp]),
    "msb_gguf_tensor_count": (ctypes.c_int64, [c_vp]),
    "msb_gguf_tensor_info": (ctypes.c_int, [c_vp, ctypes.c_int64, ctypes.POINTER(GgufTensor)]),
    "msb_gguf_find_tensor": (ctypes.c_int64, [c_vp, ctypes.c_char_p]),
    "msb_gguf_expert_tensor": (ctypes.c_int64, [c_vp, ctypes.c_int32, ctypes.c_int]),
    "msb_gguf_kv_int": (ctypes.c_int, [c_vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int64)]),
    "msb_gguf_bytes_per_slot": (ctypes.c_uint64, [c_vp]),
    "msb_gguf_read_experts": (ctypes.c_int, [c_vp, ctypes.c_int64, ctypes.c_int32, c_i32p,
                                             ctypes.POINTER(c_vp), ctypes.c_int32]),
    "msb_gguf_fill_slots_async": (ctypes.c_int, [c_vp, ctypes.c_int64, c_vp, ctypes.c_int32,
                                                 c_i32p, c_i32p, ctypes.c_int32, c_vp]),
    "msb_router_topk": (ctypes.c_int, [c_vp, ctypes.c_int, ctypes.c_int64, ctypes.c_int32,
                                       ctypes.c_int32, ctypes.c_int32, ctypes.c_int, c_vp, c_vp,
                                       c_vp]),
    "msb_dstreamer_create": (ctypes.c_int, [ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                                            ctypes.c_int32, ctypes.c_uint64, ctypes.c_int,
                                            ctypes.POINTER(c_vp)]),
    "msb_dstreamer_destroy": (ctypes.c_int, [c_vp]),
    "msb_dstreamer_remap": (ctypes.c_int, [c_vp, ctypes.c_uint32, c_vp, ctypes.c_int64,
                                           ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, c_vp,
                                           c_vp]),
    "msb_dstreamer_fill": (ctypes.c_int, [c_vp, ctypes.c_uint32, c_vp, c_vp, ctypes.c_int64,
                                          c_vp]),
    "msb_dstreamer_fill_roles": (ctypes.c_int, [c_vp, ctypes.c_uint32, ctypes.c_int32,
                                                ctypes.POINTER(c_vp), ctypes.POINTER(c_vp),
                                                ctypes.POINTER(ctypes.c_int64), c_vp]),
    "msb_dstreamer_misses": (ctypes.c_int, [c_vp, ctypes.c_uint32, c_i32p, c_i32p, c_i32p]),
    "msb_dstreamer_table": (ctypes.c_int, [c_vp, ctypes.c_uint32, c_i32p]),
    "msb_dstreamer_stats": (ctypes.c_int, [c_vp, ctypes.POINTER(CacheStats), c_u64p]),
    "msb_arena_create": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_int32, ctypes.c_int32,
                                        ctypes.POINTER(c_vp)]),
    "msb_arena_destroy": (ctypes.c_int, [c_vp]),
    "msb_arena_info": (ctypes.c_int, [c_vp, c_i32p, c_i32p, c_i32p]),
    "msb_arena_load": (ctypes.c_int, [c_vp, ctypes.c_int32, c_vp, c_vp]),
    "msb_arena_prefetch": (ctypes.c_int, [c_vp, ctypes.c_int32, c_vp, c_vp]),
    "msb_arena_wait": (ctypes.c_int, [c_vp]),
    "msb_arena_ready": (ctypes.c_int, [c_vp, ctypes.c_int32, c_vp, ctypes.POINTER(c_vp),
                                       ctypes.POINTER(c_vp), ctypes.POINTER(c_vp)]),
    "msb_arena_release": (ctypes.c_int, [c_vp, ctypes.c_int32, c_vp]),
    "msb_arena_stats": (ctypes.c_int, [c_vp, ctypes.POINTER(ArenaStats)]),
}

_lib = None


def lib():
    """Returns the loaded libmsb.so, raising if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise MsbError(f"{LIB_PATH} is missing: build it with "
                           "`python moestream_b200/csrc/build.py` (there is no fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc):
    if rc != 0:
        msg = lib().msb_last_error()
        raise MsbError(f"msb error {rc}: {msg.decode() if msg else ''}")
    return rc

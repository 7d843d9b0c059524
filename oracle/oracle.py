"""CPU oracle bindings (TEST INFRASTRUCTURE ONLY).

Loads oracle/liboracle.so (this project's C restatement, msb_oracle.c) and,
when built, oracle/_ref/libref_cache.so (the reference's own ExpertCache with
the ms_remap_fn loop restated over it, ref_shim.cpp). Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg import this module,
as the checker or the timed CPU baseline.

The per-slot grouping oracle is restated here in numpy: the pairs of each
slot in increasing pair order (a stable sort by slot), slots ascending; this
is the row order ggml's mul_mat_id groups by expert.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIBORACLE = os.path.join(HERE, "liboracle.so")
LIBREF = os.path.join(HERE, "_ref", "libref_cache.so")

IQ4_NL = 20
MXFP4 = 39
TYPES = {"iq4_nl": IQ4_NL, "mxfp4": MXFP4}
BLOCK_BYTES = {IQ4_NL: 18, MXFP4: 17}

_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int32)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_u32p = ctypes.POINTER(ctypes.c_uint32)
_u64p = ctypes.POINTER(ctypes.c_uint64)
_vp = ctypes.c_void_p

_orc = None
_ref = None


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def _p(a, t):
    return a.ctypes.data_as(t)


def orc():
    global _orc
    if _orc is None:
        if not os.path.exists(LIBORACLE):
            build()
        L = ctypes.CDLL(LIBORACLE)
        L.orc_dequant_row.argtypes = [ctypes.c_int, _u8p, _f32p, ctypes.c_int64]
        L.orc_quantize_rows.argtypes = [ctypes.c_int, _f32p, ctypes.c_int64, ctypes.c_int64, _u8p]
        L.orc_mul_mat_id.argtypes = [ctypes.c_int, _u8p, ctypes.c_int64, ctypes.c_int64,
                                     ctypes.c_int64, _f32p, ctypes.c_int64, _i32p, ctypes.c_int,
                                     ctypes.c_int, ctypes.c_int, _f32p, ctypes.c_int]
        L.orc_moe_ffn.argtypes = [ctypes.c_int, _u8p, ctypes.c_int64, _u8p, ctypes.c_int64,
                                  ctypes.c_int64, _u8p, ctypes.c_int64, ctypes.c_int64,
                                  ctypes.c_int64, _f32p, _i32p, _f32p, ctypes.c_int, ctypes.c_int,
                                  ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_float,
                                  _f32p, _f32p, ctypes.c_int]
        L.orc_moe_ffn_bias.argtypes = L.orc_moe_ffn.argtypes + [
            _f32p, _f32p, _f32p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _i32p,
            ctypes.c_int]
        L.orc_e2m1_split.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int, _f32p, _u8p, _u8p]
        L.orc_quantize_q8.argtypes = [_f32p, ctypes.c_int64, ctypes.POINTER(ctypes.c_int8), _f32p]
        L.orc_f32_to_f16.argtypes = [ctypes.c_float]
        L.orc_f32_to_f16.restype = ctypes.c_uint16
        L.orc_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.orc_f16_to_f32.restype = ctypes.c_float
        L.orc_moe_ffn_fast.argtypes = [ctypes.c_int, _u8p, ctypes.c_int64, _u8p, ctypes.c_int64,
                                       ctypes.c_int64, _u8p, ctypes.c_int64, ctypes.c_int64,
                                       ctypes.c_int64, _f32p, _i32p, _f32p, ctypes.c_int,
                                       ctypes.c_int, ctypes.c_int, ctypes.c_float,
                                       ctypes.c_float, _f32p, ctypes.c_int]
        L.orc_fast_isa.restype = ctypes.c_int
        L.orc_fast_set_isa.argtypes = [ctypes.c_int]
        _orc = L
    return _orc


def ref_available():
    return os.path.exists(LIBREF)


def ref():
    global _ref
    if _ref is None:
        L = ctypes.CDLL(LIBREF)
        L.orc_cache_new_cfg.restype = _vp
        L.orc_cache_new_cfg.argtypes = [ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                                        ctypes.c_double, ctypes.c_double, ctypes.c_double,
                                        ctypes.c_uint32, ctypes.c_int, ctypes.c_uint32,
                                        ctypes.c_double, ctypes.c_uint32]
        L.orc_cache_free.argtypes = [_vp]
        L.orc_cache_acquire.argtypes = [_vp, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_int, _u32p]
        L.orc_cache_mark_resident.argtypes = [_vp, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint64]
        L.orc_cache_release.argtypes = [_vp, ctypes.c_uint32, ctypes.c_uint32]
        L.orc_cache_end_step.argtypes = [_vp]
        L.orc_cache_slot_of.argtypes = [_vp, ctypes.c_uint32, ctypes.c_uint32]
        L.orc_cache_slot_of.restype = ctypes.c_uint32
        L.orc_cache_build_pinned.argtypes = [_vp, _u32p, ctypes.c_size_t]
        L.orc_cache_quota.argtypes = [_vp, _u32p]
        L.orc_cache_stats.argtypes = [_vp, _u64p]
        L.orc_remap_new.restype = _vp
        L.orc_remap_new.argtypes = [ctypes.c_uint32, ctypes.c_uint32]
        L.orc_remap_free.argtypes = [_vp]
        L.orc_remap_call.argtypes = [_vp, _i32p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int,
                                     ctypes.c_int, ctypes.c_uint64, _i32p, _i32p, _i32p, _i32p]
        L.orc_remap_stats.argtypes = [_vp, _u64p, _u64p]
        _ref = L
    return _ref


STATS_FIELDS = ("hit", "miss", "hit_pinned", "hit_small", "hit_main", "ghost_hit", "admit",
                "evict", "bypass", "promote", "bytes_fetched")


class RefCache:
    """The reference ExpertCache, compiled from its own source."""

    def __init__(self, n_layer=40, n_expert=256, n_slot=0, cache_frac=0.25, pin_ratio=0.05,
                 small_ratio=0.10, ghost_mult=2, layer_quota_adapt=True, quota_period=512,
                 quota_eta=0.10, quota_min=8):
        self.n_layer = n_layer
        self.h = ref().orc_cache_new_cfg(n_layer, n_expert, n_slot, cache_frac, pin_ratio,
                                         small_ratio, ghost_mult, int(layer_quota_adapt),
                                         quota_period, quota_eta, quota_min)

    def __del__(self):
        if getattr(self, "h", None):
            ref().orc_cache_free(self.h)
            self.h = None

    def acquire(self, layer, expert, origin=0):
        s = ctypes.c_uint32(0)
        hit = ref().orc_cache_acquire(self.h, layer, expert, origin, ctypes.byref(s))
        return bool(hit), int(s.value)

    def mark_resident(self, layer, expert, nbytes):
        ref().orc_cache_mark_resident(self.h, layer, expert, nbytes)

    def release(self, layer, expert):
        ref().orc_cache_release(self.h, layer, expert)

    def end_step(self):
        ref().orc_cache_end_step(self.h)

    def slot_of(self, layer, expert):
        return int(ref().orc_cache_slot_of(self.h, layer, expert))

    def build_pinned(self, freq):
        a = np.ascontiguousarray(freq, dtype=np.uint32)
        ref().orc_cache_build_pinned(self.h, _p(a, _u32p), a.size)

    def layer_quota(self):
        out = np.zeros(self.n_layer, dtype=np.uint32)
        ref().orc_cache_quota(self.h, _p(out, _u32p))
        return out

    def stats(self):
        out = np.zeros(11, dtype=np.uint64)
        ref().orc_cache_stats(self.h, _p(out, _u64p))
        return {f: int(v) for f, v in zip(STATS_FIELDS, out)}


class RefRemap:
    """ms_remap_fn's loop over the reference ExpertCache, one layer."""

    def __init__(self, n_expert, n_slot, expert_bytes=0):
        self.h = ref().orc_remap_new(n_expert, n_slot)
        self.expert_bytes = expert_bytes

    def __del__(self):
        if getattr(self, "h", None):
            ref().orc_remap_free(self.h)
            self.h = None

    def __call__(self, ids):
        ids = np.asarray(ids)
        n_tok, top_k = ids.shape
        out = np.empty((n_tok, top_k), dtype=np.int32)
        pe = np.empty(max(n_tok * top_k, 1), dtype=np.int32)
        ps = np.empty_like(pe)
        n = ctypes.c_int32(0)
        base = ids.__array_interface__["data"][0]
        ref().orc_remap_call(self.h, ctypes.cast(base, _i32p), ids.strides[1], ids.strides[0],
                             top_k, n_tok, self.expert_bytes, _p(out, _i32p), _p(pe, _i32p),
                             _p(ps, _i32p), ctypes.byref(n))
        return out, list(zip(pe[:n.value].tolist(), ps[:n.value].tolist()))

    def stats(self):
        out = np.zeros(11, dtype=np.uint64)
        ex = ctypes.c_uint64(0)
        ref().orc_remap_stats(self.h, _p(out, _u64p), ctypes.byref(ex))
        d = {f: int(v) for f, v in zip(STATS_FIELDS, out)}
        d["exhausted"] = int(ex.value)
        return d


# ---------------------------------------------------------------------------
# Block formats and matmul
# ---------------------------------------------------------------------------
def expert_bytes(wtype, K, N):
    return (K // 32) * BLOCK_BYTES[TYPES.get(wtype, wtype)] * N


def quantize(wtype, x):
    """f32 [n_rows, K] -> ggml block bytes (uint8, flat)."""
    t = TYPES.get(wtype, wtype)
    x = np.ascontiguousarray(x, dtype=np.float32)
    n_rows, K = x.shape
    out = np.empty(n_rows * (K // 32) * BLOCK_BYTES[t], dtype=np.uint8)
    assert orc().orc_quantize_rows(t, _p(x, _f32p), n_rows, K, _p(out, _u8p)) == 0
    return out


def dequantize(wtype, data, K):
    """ggml block bytes -> f32 [n_rows, K]."""
    t = TYPES.get(wtype, wtype)
    data = np.ascontiguousarray(data, dtype=np.uint8).reshape(-1)
    rb = (K // 32) * BLOCK_BYTES[t]
    n_rows = data.size // rb
    out = np.empty((n_rows, K), dtype=np.float32)
    for r in range(n_rows):
        row = data[r * rb:(r + 1) * rb]
        assert orc().orc_dequant_row(t, _p(row, _u8p), _p(out[r], _f32p), K) == 0
    return out


def quantize_q8(x):
    """ggml q8_0 of one f32 row -> (int8 codes, fp16-rounded scales)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    q = np.empty(x.size, dtype=np.int8)
    d = np.empty(x.size // 32, dtype=np.float32)
    orc().orc_quantize_q8(_p(x, _f32p), x.size, q.ctypes.data_as(ctypes.POINTER(ctypes.c_int8)),
                          _p(d, _f32p))
    return q, d


MODES = {"exact": 0, "q8": 1, "e2m1x4": 2, "f16": 3}


def e2m1_split(x, terms=4):
    """Tensor-core activation form: (sum of terms, codes [terms, nb, 32],
    scale bytes [terms, nb]) for a 1-D f32 vector."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    nb = x.size // 32
    approx = np.empty_like(x)
    codes = np.empty((terms, nb, 32), dtype=np.uint8)
    exps = np.empty((terms, nb), dtype=np.uint8)
    orc().orc_e2m1_split(_p(x, _f32p), x.size, terms, _p(approx, _f32p), _p(codes, _u8p),
                         _p(exps, _u8p))
    return approx, codes, exps


def mul_mat_id(wtype, slab, K, N, b, ids, mode="exact", nthreads=None):
    """slab: uint8 [n_slots, expert_bytes] (ggml layout); b: f32 [T, b_ne1, K];
    ids: int32 slot ids [T, top_k]. Returns f32 [T, top_k, N]."""
    t = TYPES.get(wtype, wtype)
    slab = np.ascontiguousarray(slab, dtype=np.uint8)
    b = np.ascontiguousarray(b, dtype=np.float32)
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    T, top_k = ids.shape
    out = np.empty((T, top_k, N), dtype=np.float32)
    rc = orc().orc_mul_mat_id(t, _p(slab, _u8p), K, N, slab.shape[0], _p(b, _f32p), b.shape[1],
                              _p(ids, _i32p), top_k, T, MODES[mode],
                              _p(out, _f32p), nthreads or os.cpu_count() or 1)
    assert rc == 0, rc
    return out


def moe_ffn(wtype, gate, up, down, K, n_ff, x, ids, w, mode="exact", up_row0=0, up_rows=None,
            nthreads=None, act=None, bias=None):
    """gate/up/down: uint8 [n_slots, bytes]; x: f32 [T, K]; ids: [T, top_k] slot
    ids; w: f32 [T, top_k]. The gate is rows [0, n_ff) and the up projection
    rows [up_row0, up_row0 + n_ff) of their slots (the same array for a fused
    gate_up tensor). act: None for silu(gate) * up, or (alpha, limit) for the
    gpt-oss form min(g, limit) * sigmoid(alpha * min(g, limit)) *
    (clamp(u, -limit, limit) + 1). bias: None, or (gate_b, up_b, down_b,
    expert_ids, n_expert) with f32 rows [n_expert, >= rows] (None to skip one)
    looked up by the pairs' expert ids [T, top_k] and added to the matmul
    results of pairs not in the zero slot (the last slab row). Returns
    (y [T, K], h [T, top_k, n_ff])."""
    t = TYPES.get(wtype, wtype)
    gate, up, down = (np.ascontiguousarray(a, dtype=np.uint8) for a in (gate, up, down))
    row_bytes = (K // 32) * BLOCK_BYTES[t]
    gate_rows = gate.shape[1] // row_bytes
    up_rows = up.shape[1] // row_bytes
    x = np.ascontiguousarray(x, dtype=np.float32)
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    T, top_k = ids.shape
    y = np.empty((T, K), dtype=np.float32)
    h = np.empty((T, top_k, n_ff), dtype=np.float32)
    args = (t, _p(gate, _u8p), gate_rows, _p(up, _u8p), up_rows, up_row0,
            _p(down, _u8p), K, n_ff, gate.shape[0], _p(x, _f32p), _p(ids, _i32p),
            _p(w, _f32p), top_k, T, MODES[mode], 1 if act else 0,
            act[0] if act else 1.0, act[1] if act else 0.0, _p(y, _f32p),
            _p(h, _f32p), nthreads or os.cpu_count() or 1)
    if bias is None:
        rc = orc().orc_moe_ffn(*args)
    else:
        gb, ub, db, eids, n_expert = bias
        keep = [np.ascontiguousarray(b, dtype=np.float32) if b is not None else None
                for b in (gb, ub, db)]
        eids = np.ascontiguousarray(eids, dtype=np.int32)
        assert eids.shape == ids.shape
        ptr = lambda b: _p(b, _f32p) if b is not None else None
        ld = lambda b: b.shape[1] if b is not None else 0
        rc = orc().orc_moe_ffn_bias(*args, ptr(keep[0]), ptr(keep[1]), ptr(keep[2]),
                                    ld(keep[0]), ld(keep[1]), ld(keep[2]), _p(eids, _i32p),
                                    n_expert)
    assert rc == 0, rc
    return y, h


FAST_ISA = {0: "scalar", 1: "avx2", 2: "avx512-vnni"}


def fast_isa(force=None):
    """Instruction set of the vectorized CPU baseline ("avx512-vnni", "avx2"
    or "scalar"); force an index to compare them (-1 restores detection)."""
    if force is not None:
        orc().orc_fast_set_isa(force)
    return FAST_ISA[orc().orc_fast_isa()]


def moe_ffn_fast(wtype, gate, up, down, K, n_ff, x, ids, w, up_row0=0, nthreads=None, act=None):
    """The FFN in ggml's q8 form, vectorized and threaded (msb_cpu_fast.c):
    the timed CPU baseline. Arguments as moe_ffn; returns y [T, K]. Works on
    views of the slabs without copying them (each a C-contiguous uint8 array
    [n_slots, bytes])."""
    t = TYPES.get(wtype, wtype)
    for a in (gate, up, down):
        assert a.dtype == np.uint8 and a.flags["C_CONTIGUOUS"]
    row_bytes = (K // 32) * BLOCK_BYTES[t]
    x = np.ascontiguousarray(x, dtype=np.float32)
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    T, top_k = ids.shape
    y = np.empty((T, K), dtype=np.float32)
    rc = orc().orc_moe_ffn_fast(t, _p(gate, _u8p), gate.shape[1] // row_bytes, _p(up, _u8p),
                                up.shape[1] // row_bytes, up_row0, _p(down, _u8p), K, n_ff,
                                gate.shape[0], _p(x, _f32p), _p(ids, _i32p), _p(w, _f32p), top_k,
                                T, 1 if act else 0, act[0] if act else 1.0,
                                act[1] if act else 0.0, _p(y, _f32p),
                                nthreads or os.cpu_count() or 1)
    assert rc == 0, rc
    return y


def group(slot_ids, n_slot):
    """Grouping oracle: (counts[S], offsets[S+1], rows, active) for S = n_slot+1."""
    s = np.asarray(slot_ids, dtype=np.int64).reshape(-1)
    S = n_slot + 1
    counts = np.bincount(s, minlength=S).astype(np.int32)
    offsets = np.zeros(S + 1, dtype=np.int32)
    offsets[1:] = np.cumsum(counts)
    rows = np.argsort(s, kind="stable").astype(np.int32)
    active = np.nonzero(counts)[0].astype(np.int32)
    return counts, offsets, rows, active


def remap_table(ids, table, n_slot):
    """Slot of each id through an expert -> slot table (zero slot otherwise)."""
    ids = np.asarray(ids, dtype=np.int64)
    table = np.asarray(table, dtype=np.int64)
    out = np.full(ids.shape, n_slot, dtype=np.int32)
    ok = (ids >= 0) & (ids < table.size)
    s = np.where(ok, table[np.clip(ids, 0, table.size - 1)], -1)
    good = ok & (s >= 0) & (s < n_slot)
    out[good] = s[good]
    return out


def max_abs_normalized(got, want):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    den = np.max(np.abs(want))
    return float(np.max(np.abs(got - want)) / (den if den > 0 else 1.0))


# --------------------------------------------------------------------------
# Expert-parallel packing (no counterpart in the reference, which is
# single-process): restates the meaning of msb_ep_dispatch / msb_ep_combine
# on CPU torch tensors, with the same signatures as moestream_b200.ops, so
# the host-side exchange logic can run with gloo ranks on CPU.
# --------------------------------------------------------------------------
def ep_dispatch(ids, x, n_local, n_rank, cap, send_x, send_e, pos):
    """Row of pair p = t*top_k + k goes to block ids[p] // n_local at its rank
    among earlier pairs with that destination; unused rows get id -1."""
    import torch
    n_tok, top_k = ids.shape
    flat = ids.reshape(-1).tolist()
    send_e.fill_(-1)
    used = [0] * n_rank
    for p, e in enumerate(flat):
        dest = e // n_local if 0 <= e < n_local * n_rank else -1
        if dest < 0 or used[dest] >= cap:
            if dest >= 0:
                used[dest] += 1
            pos[p] = -1
            continue
        row = dest * cap + used[dest]
        used[dest] += 1
        pos[p] = row
        send_e[row] = e - dest * n_local
        send_x[row] = x[p // top_k].to(torch.bfloat16)


def ep_combine(back, pos, w, y):
    """y[t] = sum_k w[t, k] * back[pos[t, k]] in k order, each step one f32
    fused multiply-add (pos -1 adds nothing)."""
    import torch
    n_tok, top_k = w.shape
    p = pos.reshape(n_tok, top_k)
    acc = torch.zeros(n_tok, back.shape[1], dtype=torch.float32)
    for k in range(top_k):
        r = p[:, k].long()
        ok = (r >= 0).unsqueeze(1)
        rows = back[r.clamp(min=0)].to(torch.float32)
        fused = (w[:, k:k + 1].double() * rows.double() + acc.double()).to(torch.float32)
        acc = torch.where(ok, fused, acc)
    y.copy_(acc)
    return y


# --------------------------------------------------------------------------
# Prefill arena bookkeeping: which experts each load reads.
# --------------------------------------------------------------------------
class ArenaPlan:
    """Restates load_layer_arena's choice of reads
    (src/llama-moestream.cpp:2167-2283): arena il % n_buf; when it switches
    layers it forgets what it held (:2235-2239); it reads the experts that
    `need` marks (all when need is None, :2249) and it does not hold
    (:2250); a load with nothing to read is a hit (:2269-2276)."""

    def __init__(self, n_expert, n_buf):
        self.n_expert, self.n_buf = n_expert, n_buf
        self.layer = [-1] * n_buf
        self.have = [set() for _ in range(n_buf)]
        self.loads = self.hits = self.asked = self.read = 0

    def load(self, layer, need=None):
        b = layer % self.n_buf
        if self.layer[b] != layer:
            self.have[b] = set()
            self.layer[b] = layer
        want = set(range(self.n_expert)) if need is None else {int(e) for e in need}
        todo = sorted(want - self.have[b])
        self.asked += self.n_expert
        if not todo:
            self.hits += 1
        else:
            self.loads += 1
            self.read += len(todo)
            self.have[b] |= set(todo)
        return todo

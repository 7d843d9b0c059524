"""Device operations over the C ABI, taking and returning torch CUDA tensors.

torch provides device memory and streams here; every computation runs in
libmsb.so's kernels.
"""
import ctypes

import torch

from ._lib import (OPT_MXFP4_PATH, OPT_WIDE_PASSES, TYPE_BF16, TYPE_F32, TYPE_IQ4_NL, TYPE_MXFP4, FfnActCfg,
                   FfnBiasCfg, PoolInfo, Route, c_vp, check, lib)

WEIGHT_TYPES = {"iq4_nl": TYPE_IQ4_NL, "mxfp4": TYPE_MXFP4}
_ACT_TYPES = {torch.float32: TYPE_F32, torch.bfloat16: TYPE_BF16}


def _stream(stream=None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return c_vp(s.cuda_stream)


def _ptr(t):
    return c_vp(t.data_ptr()) if t is not None else c_vp(0)


def set_mxfp4_path(path):
    """'tc' (tensor cores where shapes allow, passes of 8 or 24 pairs by batch
    size: the default), 'tc_wide' (tensor cores, always 24-pair passes where
    K is not split) or 'q8' (CUDA cores, int8 activations)."""
    check(lib().msb_set_option(OPT_MXFP4_PATH, {"tc": 0, "tc_wide": 0, "q8": 1}[path]))
    check(lib().msb_set_option(OPT_WIDE_PASSES, 2 if path == "tc_wide" else 0))


def tc_eligible(wtype, K):
    """Whether an MXFP4 projection with K inputs runs on the tensor cores."""
    return WEIGHT_TYPES.get(wtype, wtype) == TYPE_MXFP4 and K % 64 == 0


def f16_eligible(K, N):
    """Whether an IQ4_NL projection with K inputs and N rows can run on the
    tensor cores (fp16 dequantization)."""
    return K % 64 == 0 and N % 8 == 0


def device_status(clear=False):
    """Status bits of the tensor-core kernels on the current device (0 when
    every bounded wait completed). Synchronize the streams first."""
    v = ctypes.c_int32(0)
    check(lib().msb_device_status(ctypes.byref(v), 1 if clear else 0))
    return v.value


def expert_bytes(wtype, K, N):
    return int(lib().msb_expert_bytes(WEIGHT_TYPES.get(wtype, wtype), K, N))


class SlotPool:
    """Device slab of n_slot + 1 expert slots; slot n_slot is the zero slot."""

    def __init__(self, wtype, K, N, n_slot, max_fill_batch=4):
        self.wtype = WEIGHT_TYPES.get(wtype, wtype)
        h = c_vp()
        check(lib().msb_pool_create(self.wtype, K, N, n_slot, max_fill_batch, ctypes.byref(h)))
        self.handle = h
        info = PoolInfo()
        check(lib().msb_pool_get_info(h, ctypes.byref(info)))
        self.K, self.N, self.n_slot = info.K, info.N, info.n_slot
        self.expert_bytes = info.expert_bytes
        self.slot_stride = info.slot_stride
        self.zero_slot = n_slot

    @classmethod
    def borrowed(cls, handle):
        """A view of a pool the library owns (an arena's): not destroyed here."""
        self = cls.__new__(cls)
        self.handle = handle if isinstance(handle, c_vp) else c_vp(handle)
        self._owned = False
        info = PoolInfo()
        check(lib().msb_pool_get_info(handle, ctypes.byref(info)))
        self.wtype, self.K, self.N, self.n_slot = info.wtype, info.K, info.N, info.n_slot
        self.expert_bytes = info.expert_bytes
        self.slot_stride = info.slot_stride
        self.zero_slot = info.n_slot
        return self

    def close(self):
        if self.handle and getattr(self, "_owned", True):
            check(lib().msb_pool_destroy(self.handle))
        self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def fill(self, slots, srcs, stream=None):
        """Fills slots from ggml-layout expert bytes: host uint8 tensors
        (pinned for asynchrony) or device uint8 tensors."""
        slots = [int(s) for s in slots]
        n = len(slots)
        if n == 0:
            return
        sl = (ctypes.c_int32 * n)(*slots)
        ptrs = (c_vp * n)(*[s.data_ptr() for s in srcs])
        for s in srcs:
            assert s.dtype == torch.uint8 and s.numel() >= self.expert_bytes
        if srcs[0].is_cuda:
            check(lib().msb_fill_slots_from_device_async(self.handle, n, sl, ptrs, _stream(stream)))
        else:
            check(lib().msb_fill_slots_async(self.handle, n, sl, ptrs, _stream(stream)))

    def read_slot(self, slot, stream=None):
        out = torch.empty(self.expert_bytes, dtype=torch.uint8, device="cuda")
        check(lib().msb_read_slot_async(self.handle, slot, _ptr(out), _stream(stream)))
        return out


class RouteBuffers:
    """Device arrays of one grouped route (msb_route_t)."""

    def __init__(self, n_pairs, n_slot, device="cuda"):
        z = lambda n: torch.empty(max(n, 1), dtype=torch.int32, device=device)
        self.slot_ids = z(n_pairs)
        self.counts = z(n_slot + 1)
        self.offsets = z(n_slot + 2)
        self.rows = z(n_pairs)
        self.active = z(n_slot + 2)
        self.n_slot = n_slot
        self.c = Route(self.slot_ids.data_ptr(), self.counts.data_ptr(), self.offsets.data_ptr(),
                       self.rows.data_ptr(), self.active.data_ptr())


def remap_group(ids, n_slot, table=None, n_expert=None, route=None, stream=None):
    """ids: int32 [n_tok, top_k] device tensor (any strides). Returns RouteBuffers."""
    assert ids.dtype == torch.int32 and ids.is_cuda and ids.dim() == 2
    n_tok, top_k = ids.shape
    if route is None:
        route = RouteBuffers(n_tok * top_k, n_slot, ids.device)
    nb0, nb1 = ids.stride(1) * 4, ids.stride(0) * 4
    ne = int(n_expert if n_expert is not None else (table.numel() if table is not None else 0))
    check(lib().msb_remap_group(_ptr(ids), nb0, nb1, top_k, n_tok, _ptr(table), ne, n_slot,
                                ctypes.byref(route.c), _stream(stream)))
    return route


def router_topk(logits, top_k, mode="topk", ids=None, w=None, stream=None):
    """logits: [n_tok, n_expert] f32/f16/bf16 device tensor (row stride free).
    Returns (ids int32 [n_tok, top_k], w f32 [n_tok, top_k]); mode "topk":
    softmax over the selected logits, "all": softmax over all experts."""
    n_tok, n_expert = logits.shape
    assert logits.stride(1) == 1
    if ids is None:
        ids = torch.empty(n_tok, top_k, dtype=torch.int32, device=logits.device)
    if w is None:
        w = torch.empty(n_tok, top_k, dtype=torch.float32, device=logits.device)
    types = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 30}
    check(lib().msb_router_topk(_ptr(logits), types[logits.dtype],
                                logits.stride(0) * logits.element_size(), n_tok, n_expert, top_k,
                                {"topk": 0, "all": 1}[mode], _ptr(ids), _ptr(w), _stream(stream)))
    return ids, w


def workspace(K_max, n_tok, top_k, n_slot, device="cuda"):
    nbytes = int(lib().msb_workspace_bytes(K_max, n_tok, top_k, n_slot))
    return torch.empty(nbytes, dtype=torch.uint8, device=device)


def mul_mat_id(pool, b, route, top_k, ws=None, out=None, stream=None):
    """b: [n_tok, b_ne1, K] f32/bf16 (ggml b [K, b_ne1, n_tok]); returns res
    [n_tok, top_k, N] f32 (ggml res [N, top_k, n_tok])."""
    n_tok, b_ne1, K = b.shape
    assert K == pool.K and b.stride(2) == 1
    if ws is None:
        ws = workspace(pool.K, n_tok, top_k, pool.n_slot, b.device)
    if out is None:
        out = torch.empty(n_tok, top_k, pool.N, dtype=torch.float32, device=b.device)
    es = b.element_size()
    check(lib().msb_mul_mat_id(pool.handle, _ptr(b), _ACT_TYPES[b.dtype], b_ne1, b.stride(1) * es,
                               b.stride(0) * es, ctypes.byref(route.c), top_k, n_tok, _ptr(out),
                               _ptr(ws), ws.numel(), _stream(stream)))
    return out


def moe_ffn(gate, up, down, x, route, w, top_k, up_row0=0, ws=None, out=None, act=None,
            stream=None, activation=None, bias=None, accumulate=False):
    """x: [n_tok, K] f32/bf16; w: [n_tok, top_k] f32, or None with top_k 1 (y is
    the expert output itself). activation: None for silu(g) * u, or
    ("swiglu_oai", alpha, limit) for gpt-oss's clamped form. bias: None, or
    (gate_b, up_b, down_b, ids) -- f32 device tensors [n_expert, >= rows]
    (row stride free; None skips one) looked up by the router's expert ids
    (int32 [n_tok, top_k]) of every pair not in the zero slot. accumulate:
    out += the weighted sum (out must be given). Returns y [n_tok, K] f32."""
    n_tok, K = x.shape
    assert x.stride(1) == 1
    assert (w is None and top_k == 1) or (w.dtype == torch.float32 and w.is_contiguous())
    kmax = max(K, down.K)
    if ws is None:
        ws = workspace(kmax, n_tok, top_k, gate.n_slot, x.device)
    if out is None:
        out = torch.empty(n_tok, K, dtype=torch.float32, device=x.device)
    assert not accumulate or (out is not None and w is not None)
    if bias is not None or accumulate:
        gb, ub, db, ids = bias if bias is not None else (None, None, None, None)
        bc = None
        if bias is not None:
            n_expert = next(b.shape[0] for b in (gb, ub, db) if b is not None)
            for b in (gb, ub, db):
                assert b is None or (b.dtype == torch.float32 and b.stride(1) == 1 and b.is_cuda)
            assert ids.dtype == torch.int32 and ids.shape == (n_tok, top_k)
            bc = FfnBiasCfg(*[b.data_ptr() if b is not None else None for b in (gb, ub, db)],
                            *[b.stride(0) if b is not None else 0 for b in (gb, ub, db)],
                            ids.data_ptr(), ids.stride(1) * 4, ids.stride(0) * 4, n_expert)
        kind, alpha, limit = activation if activation is not None else ("silu", 1.0, 0.0)
        cfg = FfnActCfg({"silu": 0, "swiglu_oai": 1}[kind], alpha, limit)
        check(lib().msb_moe_ffn_ex(gate.handle, up.handle, up_row0, down.handle, _ptr(x),
                                   _ACT_TYPES[x.dtype], x.stride(0) * x.element_size(),
                                   ctypes.byref(route.c), _ptr(w), top_k, n_tok, _ptr(out),
                                   _ptr(act), ctypes.byref(cfg),
                                   ctypes.byref(bc) if bc is not None else None,
                                   1 if accumulate else 0, _ptr(ws), ws.numel(), _stream(stream)))
        return out
    if activation is None:
        check(lib().msb_moe_ffn(gate.handle, up.handle, up_row0, down.handle, _ptr(x),
                                _ACT_TYPES[x.dtype], x.stride(0) * x.element_size(),
                                ctypes.byref(route.c), _ptr(w), top_k, n_tok, _ptr(out),
                                _ptr(act), _ptr(ws), ws.numel(), _stream(stream)))
        return out
    kind, alpha, limit = activation
    cfg = FfnActCfg({"silu": 0, "swiglu_oai": 1}[kind], alpha, limit)
    check(lib().msb_moe_ffn_act(gate.handle, up.handle, up_row0, down.handle, _ptr(x),
                                _ACT_TYPES[x.dtype], x.stride(0) * x.element_size(),
                                ctypes.byref(route.c), _ptr(w), top_k, n_tok, _ptr(out),
                                _ptr(act), ctypes.byref(cfg), _ptr(ws), ws.numel(),
                                _stream(stream)))
    return out


def quantize_rows(wtype, src, stream=None):
    """src: f32 [n_rows, K] device tensor -> ggml block bytes (uint8)."""
    wt = WEIGHT_TYPES.get(wtype, wtype)
    n_rows, K = src.shape
    nbytes = int(lib().msb_expert_bytes(wt, K, n_rows))
    out = torch.empty(nbytes, dtype=torch.uint8, device=src.device)
    check(lib().msb_quantize_rows(wt, _ptr(src.contiguous()), n_rows, K, _ptr(out),
                                  _stream(stream)))
    return out


def ep_dispatch(ids, x, n_local, n_rank, cap, send_x, send_e, pos, stream=None):
    """Packs this rank's (token, k) rows for an equal-split all-to-all.
    send_x: bf16 [n_rank * cap, >= K] (row stride free); send_e: int32
    [n_rank * cap] view with any row stride (it may alias a column of the
    send_x rows, so that one exchange carries both)."""
    n_tok, top_k = ids.shape
    assert ids.is_contiguous() and x.stride(1) == 1 and send_x.dtype == torch.bfloat16
    assert send_x.stride(1) == 1 and send_e.dtype == torch.int32
    check(lib().msb_ep_dispatch(_ptr(ids), _ptr(x), _ACT_TYPES[x.dtype],
                                x.stride(0) * x.element_size(), top_k, n_tok, x.shape[1],
                                n_local, n_rank, cap, _ptr(send_x), send_x.stride(0) * 2,
                                _ptr(send_e), send_e.stride(0) * 4, _ptr(pos), _stream(stream)))


def ep_dispatch_peers(peers, ids, x, n_local, pos, stream=None):
    """Stores this rank's (token, k) rows into the owning ranks' exchange
    buffers (peers: an EpPeers)."""
    n_tok, top_k = ids.shape
    assert ids.is_contiguous() and x.stride(1) == 1
    check(lib().msb_ep_dispatch_peers(ctypes.byref(peers), _ptr(ids), _ptr(x), _ACT_TYPES[x.dtype],
                                      x.stride(0) * x.element_size(), top_k, n_tok, n_local,
                                      _ptr(pos), _stream(stream)))


def ep_return_peers(peers, y_loc, stream=None):
    """Stores the local results of received rows back into their source
    ranks' exchange buffers."""
    assert y_loc.dtype == torch.float32 and y_loc.is_contiguous()
    check(lib().msb_ep_return_peers(ctypes.byref(peers), _ptr(y_loc), _stream(stream)))


def ep_wait(peers, phase, stream=None):
    """Waits (on the device, bounded) for every rank's rows (phase 0) or
    results (phase 1) to arrive in this rank's exchange buffer."""
    check(lib().msb_ep_wait(ctypes.byref(peers), phase, _stream(stream)))


def ep_remap_group(peers, n_slot, route, stream=None):
    """Waits (on the device, bounded) for every rank's rows, then groups the
    received rows by local slot into `route` (RouteBuffers)."""
    check(lib().msb_ep_remap_group(ctypes.byref(peers), n_slot, ctypes.byref(route.c),
                                   _stream(stream)))
    return route


ERR_UNSUPPORTED = 4


def ep_moe_ffn_peers(peers, gate, up, down, route, ws, up_row0=0, stream=None):
    """The local FFN over the received rows with the results stored straight
    into their source ranks' buffers by the down projection. Returns False
    (nothing launched) when the pools are not tensor-core shapes."""
    rc = lib().msb_ep_moe_ffn_peers(ctypes.byref(peers), gate.handle, up.handle, up_row0,
                                    down.handle, ctypes.byref(route.c), _ptr(ws), ws.numel(),
                                    _stream(stream))
    if rc == ERR_UNSUPPORTED:
        return False
    check(rc)
    return True


def ep_combine_peers(peers, pos, w, y, stream=None):
    """Waits (on the device, bounded) for every result, then
    y[t] = sum_k w[t, k] * (returned row of pair (t, k))."""
    n_tok, top_k = w.shape
    check(lib().msb_ep_combine_peers(ctypes.byref(peers), _ptr(pos), _ptr(w), top_k, n_tok,
                                     _ptr(y), _stream(stream)))
    return y


def ep_combine(back, pos, w, y, stream=None):
    """y[t] = sum_k w[t, k] * back[pos[t, k]]."""
    n_tok, top_k = w.shape
    check(lib().msb_ep_combine(_ptr(back), _ptr(pos), _ptr(w), top_k, n_tok, back.shape[1],
                               _ptr(y), _stream(stream)))
    return y

"""Prefill arena on the device (msb_arena_*), loaded from a GGUF.

Three MoE layers in a GGUF, two arena buffers, two passes over the layers in
the reference's order (load_layer_arena for the batch's union, then the next
layer's load started in the background with that layer's union from the
previous pass as the hint: src/llama-moestream.cpp:2167-2317). Each layer's
FFN over the arena pools matches the oracle's FFN over all experts (the
tensor-core tolerance of the single-GPU layer), and the experts read by each
load are the oracle's restatement of the reference's choice (ArenaPlan).
"""
import numpy as np
import pytest
import torch
from gguf import GGMLQuantizationType as T

from oracle import oracle as O
from tests.helpers import experts, topk_ids, write_gguf, zipf_bias

pytestmark = pytest.mark.gpu

N_LAYER, E, K, N_FF, TOP_K, N_TOK = 3, 16, 512, 256, 4, 24


def _model(tmp_path):
    mats, tensors = {}, []
    for il in range(N_LAYER):
        for r, (kk, nn) in (("gate", (K, N_FF)), ("up", (K, N_FF)), ("down", (N_FF, K))):
            ex = experts("mxfp4", E, kk, nn, seed=100 * il + len(r))
            mats[il, r] = ex
            tensors.append((f"blk.{il}.ffn_{r}_exps.weight", ex.reshape(E, nn, -1), T.MXFP4))
    path = write_gguf(tmp_path / "moe.gguf", tensors, [("add_block_count", N_LAYER),
                                                       ("add_expert_count", E)])[0]
    return path, mats


def _slab(m):
    return np.concatenate([m, np.zeros((1, m.shape[1]), np.uint8)])


def test_arena_prefill_two_passes_match_oracle(tmp_path):
    from moestream_b200 import ops
    from moestream_b200.gguf import ExpertArena
    path, mats = _model(tmp_path)
    rng = np.random.default_rng(5)
    bias = zipf_bias(rng, E)
    compute = torch.cuda.current_stream()
    copy = torch.cuda.Stream()
    plan = O.ArenaPlan(E, 2)
    prev_union = [None] * N_LAYER
    with ExpertArena(path, n_buf=2, n_threads=3) as arena:
        assert (arena.n_layer, arena.n_expert, arena.n_buf) == (N_LAYER, E, 2)
        for p in range(2):
            for il in range(N_LAYER):
                ids, w = topk_ids(rng, N_TOK, E, TOP_K, bias=bias)
                x = torch.from_numpy(rng.normal(0, 1, size=(N_TOK, K)).astype(np.float32))
                x = x.to(torch.bfloat16)
                union = np.unique(ids)
                ids_d = torch.from_numpy(ids).cuda()
                route = ops.remap_group(ids_d, E)              # slot e is expert e
                arena.load(il, union, stream=copy)             # what the hint missed
                plan.load(il, union)
                gate, up, down = arena.ready(il, stream=compute)
                y = ops.moe_ffn(gate, up, down, x.cuda(), route,
                                torch.from_numpy(w).cuda(), TOP_K)
                arena.release(il, stream=compute)
                nxt = (il + 1) % N_LAYER
                if p == 0 or il + 1 < N_LAYER:                 # the next layer, background
                    arena.prefetch(nxt, prev_union[nxt], stream=copy)
                    plan.load(nxt, prev_union[nxt])
                prev_union[il] = union
                want, _ = O.moe_ffn("mxfp4", _slab(mats[il, "gate"]), _slab(mats[il, "up"]),
                                    _slab(mats[il, "down"]), K, N_FF, x.float().numpy(), ids,
                                    w, mode="e2m1x4")
                err = O.max_abs_normalized(y.cpu().numpy(), want)
                assert err < 1e-3, (p, il, err)
        st = arena.stats()
    assert st["experts_read"] == plan.read and st["loads"] == plan.loads
    assert st["hits"] == plan.hits and st["experts_asked"] == plan.asked
    assert plan.read < 2 * N_LAYER * E                          # unions and hints saved reads
    eb = sum(mats[0, r].shape[1] for r in ("gate", "up", "down"))
    assert st["bytes_read"] == plan.read * eb
    assert ops.device_status() == 0


def test_arena_ready_refuses_a_layer_it_does_not_hold(tmp_path):
    from moestream_b200 import MsbError
    from moestream_b200.gguf import ExpertArena
    path, _ = _model(tmp_path)
    with ExpertArena(path, n_buf=2) as arena:
        arena.load(0, [1, 2])
        with pytest.raises(MsbError, match="holds layer 0, not 2"):
            arena.ready(2)
        arena.ready(0)
        with pytest.raises(MsbError, match="two arena buffers"):
            ExpertArena(path, n_buf=1).prefetch(1)


def test_arena_is_bit_identical_to_slot_pools(tmp_path):
    """The reference's arena spike checks mul_mat_id over the arena against
    the normal buffer bit for bit (research/spikes/s6_arena_mulmatid/
    main.c:206-243). Here: one layer's FFN over the arena loaded from the
    GGUF, against the same experts filled into ordinary pools from memory."""
    from moestream_b200 import ops
    from moestream_b200.gguf import ExpertArena
    path, mats = _model(tmp_path)
    rng = np.random.default_rng(8)
    ids, w = topk_ids(rng, N_TOK, E, TOP_K)
    x = torch.from_numpy(rng.normal(0, 1, size=(N_TOK, K)).astype(np.float32)).cuda()
    ids_d, w_d = torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda()
    pools = {}
    for r, (kk, nn) in (("gate", (K, N_FF)), ("up", (K, N_FF)), ("down", (N_FF, K))):
        pools[r] = ops.SlotPool("mxfp4", kk, nn, E)
        pools[r].fill(list(range(E)), [torch.from_numpy(mats[1, r][e]).pin_memory()
                                       for e in range(E)])
    route = ops.remap_group(ids_d, E)
    y_pool = ops.moe_ffn(pools["gate"], pools["up"], pools["down"], x, route, w_d, TOP_K)
    with ExpertArena(path, n_buf=2) as arena:
        arena.load(1, np.unique(ids))
        gate, up, down = arena.ready(1)
        y_arena = ops.moe_ffn(gate, up, down, x, route, w_d, TOP_K)
        arena.release(1)
        torch.cuda.synchronize()
    assert torch.equal(y_arena, y_pool)

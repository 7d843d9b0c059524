"""Device slot streamer on the GPU: the decode remap, the fills and the FFN
with no host round trip.

- The remap kernel's slots, miss queue (read from mapped memory), table and
  counters equal the host slot streamer's on random traces.
- The fill kernel copies the missed experts from pinned host memory (and
  from device memory) into their slots bit-exactly.
- A whole decode step (remap -> three fills -> grouping -> FFN) captured in
  one CUDA graph and replayed with new router ids written in place each
  time: every replay's output equals the oracle's FFN over the experts the
  ids name, and its slots equal the host streamer's.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import experts, topk_ids, zipf_bias

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n_expert,n_slot,top_k,max_tok,seed", [
    (128, 32, 4, 4, 0), (128, 32, 4, 64, 1), (256, 64, 8, 8, 2), (16, 8, 4, 6, 3)])
def test_device_remap_matches_host_streamer(n_expert, n_slot, top_k, max_tok, seed):
    from moestream_b200 import DeviceSlotStreamer, SlotStreamer
    rng = np.random.default_rng(seed)
    n_layer = 2
    ref = SlotStreamer(n_layer, n_expert, n_slot, 77)
    dev = DeviceSlotStreamer(n_layer, n_expert, n_slot, max_tok * top_k, 77)
    bias = zipf_bias(rng, n_expert)
    for step in range(25):
        for il in range(n_layer):
            n_tok = int(rng.integers(1, max_tok + 1))
            ids, _ = topk_ids(rng, n_tok, n_expert, top_k, bias=bias)
            if step % 6 == 2:
                ids[0, 0] = -1
            want, misses, table = ref.remap(il, ids, want_table=True)
            got = dev.remap(il, torch.from_numpy(ids).cuda())
            torch.cuda.synchronize()
            assert np.array_equal(got.cpu().numpy(), want), (step, il)
            assert dev.misses(il) == misses, (step, il)
            assert np.array_equal(dev.table(il), table), (step, il)
    assert dev.stats() == ref.stats()


@pytest.mark.parametrize("wtype,K,N", [("mxfp4", 2880, 256), ("iq4_nl", 2048, 128),
                                       ("mxfp4", 96, 40)])
@pytest.mark.parametrize("where", ["pinned", "device"])
def test_device_fill_from_host_memory(wtype, K, N, where):
    from moestream_b200 import DeviceSlotStreamer, ops
    n_expert, n_slot, top_k = 12, 5, 2
    ex = experts(wtype, n_expert, K, N, seed=K + N)
    src = torch.from_numpy(ex)
    src = src.pin_memory() if where == "pinned" else src.cuda()
    pool = ops.SlotPool(wtype, K, N, n_slot)
    dev = DeviceSlotStreamer(1, n_expert, n_slot, 16)
    rng = np.random.default_rng(9)
    for step in range(4):
        ids = np.stack([rng.permutation(n_expert)[:top_k] for _ in range(2)]).astype(np.int32)
        dev.remap(0, torch.from_numpy(ids).cuda())
        dev.fill(0, pool, src)
        torch.cuda.synchronize()
        table = dev.table(0)
        for e in np.unique(ids):
            assert np.array_equal(pool.read_slot(int(table[e])).cpu().numpy(), ex[e]), (step, e)
    assert int(pool.read_slot(n_slot).to(torch.int64).sum()) == 0


def test_fill_of_three_roles_in_one_launch():
    """fill_roles: pools of different shapes and types of block rows (gate
    and up [K -> N_ff], down [N_ff -> K]) filled by one launch, bit-exact."""
    from moestream_b200 import DeviceSlotStreamer, ops
    n_expert, n_slot, K, N_FF = 10, 4, 2880, 640
    shapes = {"gate": (K, N_FF), "up": (K, N_FF), "down": (N_FF, K)}
    mats = {r: experts("mxfp4", n_expert, kk, nn, seed=i) for i, (r, (kk, nn)) in
            enumerate(shapes.items())}
    src = {r: torch.from_numpy(m).pin_memory() for r, m in mats.items()}
    pools = {r: ops.SlotPool("mxfp4", kk, nn, n_slot) for r, (kk, nn) in shapes.items()}
    dev = DeviceSlotStreamer(1, n_expert, n_slot, 8)
    rng = np.random.default_rng(2)
    for step in range(4):
        ids = rng.permutation(n_expert)[:3].astype(np.int32).reshape(1, 3)
        dev.remap(0, torch.from_numpy(ids).cuda())
        dev.fill_roles(0, [pools[r] for r in shapes], [src[r] for r in shapes])
        torch.cuda.synchronize()
        table = dev.table(0)
        for r in shapes:
            for e in ids.ravel():
                got = pools[r].read_slot(int(table[e])).cpu().numpy()
                assert np.array_equal(got, mats[r][e]), (step, r, e)


def test_graph_captured_decode_step_matches_oracle():
    from moestream_b200 import DeviceSlotStreamer, SlotStreamer, ops
    wtype, K, N_FF, n_expert, n_slot, top_k, n_tok = "mxfp4", 512, 256, 32, 12, 4, 2
    mats = {r: experts(wtype, n_expert, kk, nn, seed=s)
            for r, kk, nn, s in (("gate", K, N_FF, 1), ("up", K, N_FF, 2), ("down", N_FF, K, 3))}
    src = {r: torch.from_numpy(m).pin_memory() for r, m in mats.items()}
    pools = {r: ops.SlotPool(wtype, kk, nn, n_slot)
             for r, kk, nn in (("gate", K, N_FF), ("up", K, N_FF), ("down", N_FF, K))}
    dev = DeviceSlotStreamer(1, n_expert, n_slot, n_tok * top_k)
    ref = SlotStreamer(1, n_expert, n_slot)
    ids_d = torch.zeros(n_tok, top_k, dtype=torch.int32, device="cuda")
    w_d = torch.zeros(n_tok, top_k, dtype=torch.float32, device="cuda")
    x_d = torch.zeros(n_tok, K, dtype=torch.bfloat16, device="cuda")
    slots = torch.empty(n_tok, top_k, dtype=torch.int32, device="cuda")
    route = ops.RouteBuffers(n_tok * top_k, n_slot)
    ws = ops.workspace(K, n_tok, top_k, n_slot)
    y = torch.empty(n_tok, K, dtype=torch.float32, device="cuda")

    def step():
        dev.remap(0, ids_d, out=slots)
        roles = ("gate", "up", "down")
        dev.fill_roles(0, [pools[r] for r in roles], [src[r] for r in roles])
        ops.remap_group(slots, n_slot, route=route)
        ops.moe_ffn(pools["gate"], pools["up"], pools["down"], x_d, route, w_d, top_k,
                    ws=ws, out=y)

    rng = np.random.default_rng(17)
    bias = zipf_bias(rng, n_expert)

    def new_inputs():
        ids, w = topk_ids(rng, n_tok, n_expert, top_k, bias=bias)
        x = rng.normal(0, 1, size=(n_tok, K)).astype(np.float32)
        ids_d.copy_(torch.from_numpy(ids))
        w_d.copy_(torch.from_numpy(w))
        x_d.copy_(torch.from_numpy(x).to(torch.bfloat16))
        return ids, w, torch.from_numpy(x).to(torch.bfloat16).float().numpy()

    def check(ids, w, x):
        want_slots, _, _ = ref.remap(0, ids)
        assert np.array_equal(slots.cpu().numpy(), want_slots)
        slab = {r: np.concatenate([m, np.zeros((1, m.shape[1]), np.uint8)])
                for r, m in mats.items()}
        want, _ = O.moe_ffn(wtype, slab["gate"], slab["up"], slab["down"], K, N_FF, x,
                            np.where(want_slots == n_slot, n_expert, ids), w, mode="e2m1x4")
        assert O.max_abs_normalized(y.cpu().numpy(), want) < 1e-3

    # Warm up eagerly (also creates the kernels' attributes), then capture.
    check_in = new_inputs()
    step()
    torch.cuda.synchronize()
    check(*check_in)
    g = torch.cuda.CUDAGraph()
    cap_in = new_inputs()
    with torch.cuda.graph(g):
        step()
    # Capture records without running: the streamer's state is untouched.
    for _ in range(6):
        inp = new_inputs() if _ else cap_in
        g.replay()
        torch.cuda.synchronize()
        check(*inp)
    assert ops.device_status() == 0
    assert dev.stats()["miss"] > 6


def test_streamed_ffn_is_bit_identical_to_resident():
    """The reference's streaming spike checks that the streamed MoE FFN is
    bit-identical to the fully resident one (research/spikes/
    s1_real_expert_stream/main.c:375-388). Here: experts streamed through
    the device streamer into 12 slots, against every expert resident in a
    pool of its own (slot e = expert e), step after step."""
    from moestream_b200 import DeviceSlotStreamer, ops
    wtype, K, N_FF, n_expert, n_slot, top_k, n_tok = "mxfp4", 512, 256, 32, 12, 4, 3
    shapes = {"gate": (K, N_FF), "up": (K, N_FF), "down": (N_FF, K)}
    mats = {r: experts(wtype, n_expert, kk, nn, seed=40 + i)
            for i, (r, (kk, nn)) in enumerate(shapes.items())}
    src = {r: torch.from_numpy(m).pin_memory() for r, m in mats.items()}
    stream_pools = {r: ops.SlotPool(wtype, kk, nn, n_slot) for r, (kk, nn) in shapes.items()}
    full = {r: ops.SlotPool(wtype, kk, nn, n_expert) for r, (kk, nn) in shapes.items()}
    for r in shapes:
        full[r].fill(list(range(n_expert)), [src[r][e] for e in range(n_expert)])
    dev = DeviceSlotStreamer(1, n_expert, n_slot, n_tok * top_k)
    rng = np.random.default_rng(23)
    bias = zipf_bias(rng, n_expert)
    roles = ("gate", "up", "down")
    for step in range(8):
        ids, w = topk_ids(rng, n_tok, n_expert, top_k, bias=bias)
        x = torch.from_numpy(rng.normal(0, 1, size=(n_tok, K)).astype(np.float32)).cuda()
        ids_d, w_d = torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda()
        slots = dev.remap(0, ids_d)
        dev.fill_roles(0, [stream_pools[r] for r in roles], [src[r] for r in roles])
        r_s = ops.remap_group(slots, n_slot)
        y_s = ops.moe_ffn(stream_pools["gate"], stream_pools["up"], stream_pools["down"], x,
                          r_s, w_d, top_k)
        r_f = ops.remap_group(ids_d, n_expert)
        y_f = ops.moe_ffn(full["gate"], full["up"], full["down"], x, r_f, w_d, top_k)
        torch.cuda.synchronize()
        assert int((slots == n_slot).sum()) == 0          # no exhaustion at these sizes
        assert torch.equal(y_s, y_f), step

"""Prompt processing while missing experts are filled (the 512-token Zipf
batch with ~30% of its experts not resident).

The batch runs in two FFN calls over two routes of the same router ids: the
first sends the experts that are still being filled to the zero slot and
computes the resident ones, while a side stream copies the missing experts
from pinned host memory into their slots (msb_fill_slots_async); the second
waits on the fill's event, sends every other expert to the zero slot, and
adds the filled experts' contributions into y (accumulate). Before the fill
the missing slots hold another expert's bytes, so reading them early would
show. The result is compared with the same batch computed in one call with
every expert resident (equal up to the rounding of the final addition,
1e-6 of the output's max) and with the oracle (the tensor-core form, 1e-3).
The reference loads a prompt batch's experts into the arena before running
it (src/llama-moestream.cpp:2167-2317); the overlap is this library's.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import zipf_bias

pytestmark = pytest.mark.gpu


def zipf_routing(n_tok, n_expert, top_k, seed):
    rng = np.random.default_rng(seed)
    logits = rng.normal(0, 1, size=(n_tok, n_expert)) + zipf_bias(rng, n_expert)
    ids = np.argsort(-logits, axis=1, kind="stable")[:, :top_k].astype(np.int32)
    sel = np.take_along_axis(logits, ids, 1)
    w = np.exp(sel - sel.max(1, keepdims=True))
    return ids, (w / w.sum(1, keepdims=True)).astype(np.float32)


def two_phase(pools, x, ids, w, pending, host_src, wrong_src, top_k):
    """Phase 1 over the resident experts while the side stream fills
    `pending`; phase 2 over the filled ones. Returns y (device)."""
    from moestream_b200 import ops
    ga, up, dn = pools
    E = ga.n_slot
    # The pending slots first hold the wrong bytes.
    for p, src in zip(pools, wrong_src):
        p.fill(pending, src)
    torch.cuda.synchronize()
    table_a = np.arange(E, dtype=np.int32)
    table_a[pending] = -1
    table_b = np.full(E, -1, dtype=np.int32)
    table_b[pending] = pending
    n_tok = x.shape[0]
    ws = ops.workspace(ga.K, n_tok, top_k, E)
    y = torch.empty(n_tok, ga.K, dtype=torch.float32, device="cuda")
    ids_t = torch.from_numpy(ids).cuda()
    w_t = torch.from_numpy(w).cuda()
    ta, tb = torch.from_numpy(table_a).cuda(), torch.from_numpy(table_b).cuda()
    side = torch.cuda.Stream()
    main = torch.cuda.current_stream()
    start = torch.cuda.Event()
    start.record(main)
    side.wait_event(start)
    ra = ops.remap_group(ids_t, E, table=ta, n_expert=E)
    ops.moe_ffn(ga, up, dn, x, ra, w_t, top_k, ws=ws, out=y)
    for p, src in zip(pools, host_src):
        p.fill(pending, src, stream=side)
    filled = torch.cuda.Event()
    filled.record(side)
    main.wait_event(filled)
    rb = ops.remap_group(ids_t, E, table=tb, n_expert=E)
    ops.moe_ffn(ga, up, dn, x, rb, w_t, top_k, ws=ws, out=y, accumulate=True)
    torch.cuda.synchronize()
    return y


@pytest.mark.parametrize("K,n_ff,n_tok", [(512, 256, 64), (2880, 2880, 512)])
def test_fill_overlapped_two_phase_ffn(K, n_ff, n_tok):
    import bench
    from moestream_b200 import ops
    torch.cuda.set_device(0)
    E, top_k = (16 if K == 512 else 128), 4
    (ga, up, dn), = bench.build_layers(1, 0, E, K, n_ff, seed=77)
    pools = (ga, up, dn)
    ids, w = zipf_routing(n_tok, E, top_k, seed=n_tok)
    referenced = np.unique(ids)
    rng = np.random.default_rng(5)
    pending = np.sort(rng.choice(referenced, max(1, int(0.3 * len(referenced))), replace=False))
    pending = pending.astype(np.int32)
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    x = torch.randn(n_tok, K, generator=g, device="cuda").to(torch.bfloat16)
    # Every expert resident: the one-call result.
    r = ops.remap_group(torch.from_numpy(ids).cuda(), E)
    want = ops.moe_ffn(ga, up, dn, x, r, torch.from_numpy(w).cuda(), top_k)
    slabs = []
    for p in pools:
        rows = [p.read_slot(s).cpu() for s in range(E)]
        slabs.append(np.stack([t.numpy() for t in rows] + [np.zeros(p.expert_bytes, np.uint8)]))
    torch.cuda.synchronize()
    host_src = [[torch.from_numpy(slabs[i][e]).pin_memory() for e in pending] for i in range(3)]
    wrong_src = [[torch.from_numpy(slabs[i][(e + 1) % E]).pin_memory() for e in pending]
                 for i in range(3)]
    got = two_phase(pools, x, ids, w, pending.tolist(), host_src, wrong_src, top_k)
    assert ops.device_status() == 0
    assert O.max_abs_normalized(got.cpu().numpy(), want.cpu().numpy()) < 1e-6
    sample = np.sort(np.random.default_rng(1).choice(n_tok, min(n_tok, 24), replace=False))
    x_np = x.float().cpu().numpy()[sample]
    y_o, _ = O.moe_ffn("mxfp4", slabs[0], slabs[1], slabs[2], K, n_ff, x_np, ids[sample],
                       w[sample], mode="e2m1x4")
    assert O.max_abs_normalized(got.cpu().numpy()[sample], y_o) < 1e-3
    # The fills wrote the right bytes.
    for p, sl in zip(pools, slabs):
        for e in pending[:3]:
            assert np.array_equal(p.read_slot(int(e)).cpu().numpy(), sl[e])

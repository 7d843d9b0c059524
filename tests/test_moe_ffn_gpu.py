"""MoE FFN layer (gate/up mul_mat_id + SwiGLU, down mul_mat_id, weighted
combine) against the CPU oracle, for separate gate/up tensors and for a
fused gate_up tensor whose first N_ff rows are the gate.

MXFP4 layers whose shapes allow it (K and N_ff multiples of 64, the up rows
starting on a 32-row boundary) run on the tensor cores with activations as
four e2m1 terms; the rest, and every layer with the q8 option, on the CUDA
cores with int8 activations (ggml's q8_0 form).
Tolerances (max |got - want| / max |want|):
  - against the oracle in the path's own form: 2e-3 (q8) or 1e-3 (e2m1x4)
    for y, 1e-5 (q8) or 1e-4 (e2m1x4) for the SwiGLU output (the
    re-quantized SwiGLU output can round a code differently where the f32
    sums differ in their last bits);
  - against the exact f64 oracle: 1e-2 for each projection's input h, and
    for y no further from exact than ggml's q8 form itself (plus 5e-4).
    Two chained projections with int8 activations are 1.1-1.3% from exact
    in ggml's own CPU arithmetic on these shapes, so 1e-2 applies per
    mul_mat_id (tests/test_mul_mat_id_gpu.py), not to the chain.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import experts, topk_ids

pytestmark = pytest.mark.gpu


@pytest.fixture(params=["tc", "tc_wide", "q8"])
def path(request):
    """"tc" / "tc_wide": MXFP4 on the tensor cores (passes by batch size, or
    always 24 pairs) and IQ4_NL on the tensor cores wherever the shapes
    allow; "q8": both on the CUDA cores."""
    from moestream_b200 import ops
    from moestream_b200._lib import OPT_IQ4NL_PATH
    ops.set_mxfp4_path(request.param)
    ops.check(ops.lib().msb_set_option(OPT_IQ4NL_PATH, 1 if request.param == "q8" else 2))
    yield request.param
    ops.set_mxfp4_path("tc")
    ops.check(ops.lib().msb_set_option(OPT_IQ4NL_PATH, 0))


@pytest.fixture(params=["q8", "f16"])
def iq4_form(request):
    """IQ4_NL arithmetic for tests that do not take `path`: the CUDA-core
    q8_0 form or the tensor-core f16 form."""
    from moestream_b200 import ops
    from moestream_b200._lib import OPT_IQ4NL_PATH
    ops.check(ops.lib().msb_set_option(OPT_IQ4NL_PATH, 1 if request.param == "q8" else 2))
    yield request.param
    ops.check(ops.lib().msb_set_option(OPT_IQ4NL_PATH, 0))


def build_layer(wtype, K, n_ff, n_expert, n_slot, fused, seed):
    from moestream_b200 import ops
    rng = np.random.default_rng(seed)
    resident = rng.permutation(n_expert)[:n_slot]
    slot_of = {int(e): int(s) for e, s in zip(resident, rng.permutation(n_slot))}
    if fused:
        gu = experts(wtype, n_expert, K, 2 * n_ff, seed)
        pools = {"gate": ops.SlotPool(wtype, K, 2 * n_ff, n_slot)}
        pools["up"] = pools["gate"]
        mats = {"gate": gu}
    else:
        mats = {"gate": experts(wtype, n_expert, K, n_ff, seed),
                "up": experts(wtype, n_expert, K, n_ff, seed + 1)}
        pools = {r: ops.SlotPool(wtype, K, n_ff, n_slot) for r in ("gate", "up")}
    mats["down"] = experts(wtype, n_expert, n_ff, K, seed + 2)
    pools["down"] = ops.SlotPool(wtype, n_ff, K, n_slot)
    for role, m in mats.items():
        srcs = [torch.from_numpy(m[e]).pin_memory() for e in slot_of]
        pools[role].fill(list(slot_of.values()), srcs)
    slabs = {}
    for role, m in mats.items():
        slab = np.zeros((n_slot + 1, m.shape[1]), dtype=np.uint8)
        for e, s in slot_of.items():
            slab[s] = m[e]
        slabs[role] = slab
    torch.cuda.synchronize()
    return pools, slabs, slot_of


CASES = [
    # wtype, K, n_ff, n_expert, n_slot, n_tok, top_k, fused
    ("mxfp4", 2880, 2880, 6, 4, 2, 4, True),     # gpt-oss widths, fused gate_up (up half off
                                                 # the 128-row tile grid)
    ("mxfp4", 2880, 2880, 6, 4, 3, 4, False),    # gpt-oss widths, separate gate and up
    ("mxfp4", 2880, 2880, 6, 4, 16, 4, True),    # the same fused layout with 64 pairs: wide
                                                 # passes (8-block stages, the up half's scale
                                                 # records from two tiles)
    ("iq4_nl", 2048, 512, 10, 8, 8, 8, False),   # 256-expert model widths
    ("mxfp4", 512, 256, 8, 8, 40, 4, True),      # several passes per slot
    ("iq4_nl", 256, 128, 6, 3, 5, 2, False),
]


@pytest.mark.parametrize("wtype,K,n_ff,n_expert,n_slot,n_tok,top_k,fused", CASES)
@pytest.mark.parametrize("xdtype", [torch.float32, torch.bfloat16])
def test_moe_ffn_matches_oracle(wtype, K, n_ff, n_expert, n_slot, n_tok, top_k, fused, xdtype,
                                path):
    from moestream_b200 import ops
    pools, slabs, slot_of = build_layer(wtype, K, n_ff, n_expert, n_slot, fused, seed=K + n_ff)
    rng = np.random.default_rng(n_tok)
    x = rng.normal(0, 1, size=(n_tok, K)).astype(np.float32)
    if xdtype == torch.bfloat16:
        x = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    ids_e, w = topk_ids(rng, n_tok, n_expert, top_k)
    table = np.full(n_expert, -1, dtype=np.int32)
    for e, s in slot_of.items():
        table[e] = s
    slots = O.remap_table(ids_e, table, n_slot)  # non-resident experts -> zero slot

    xt = torch.from_numpy(x).cuda().to(xdtype)
    r = ops.remap_group(torch.from_numpy(ids_e).cuda(), n_slot,
                        table=torch.from_numpy(table).cuda(), n_expert=n_expert)
    act = torch.empty(n_tok, top_k, n_ff, dtype=torch.float32, device="cuda")
    y = ops.moe_ffn(pools["gate"], pools["up"], pools["down"], xt, r,
                    torch.from_numpy(w).cuda(), top_k, up_row0=n_ff if fused else 0, act=act)
    torch.cuda.synchronize()
    y = y.cpu().numpy()

    up = slabs["gate"] if fused else slabs["up"]
    kw = dict(up_row0=n_ff if fused else 0)
    tc = (path.startswith("tc") and wtype == "mxfp4" and K % 64 == 0 and n_ff % 64 == 0 and
          (not fused or n_ff % 32 == 0))
    f16 = (path.startswith("tc") and wtype == "iq4_nl" and K % 64 == 0 and n_ff % 64 == 0 and
           (not fused or n_ff % 128 == 0))
    mode = "e2m1x4" if tc else ("f16" if f16 else "q8")
    tc = tc or f16
    y_f, h_f = O.moe_ffn(wtype, slabs["gate"], up, slabs["down"], K, n_ff, x, slots, w,
                         mode=mode, **kw)
    y_ex, h_ex = O.moe_ffn(wtype, slabs["gate"], up, slabs["down"], K, n_ff, x, slots, w,
                           mode="exact", **kw)
    a = act.cpu().numpy()
    assert O.max_abs_normalized(a, h_f) < (1e-4 if tc else 1e-5)
    assert O.max_abs_normalized(y, y_f) < (1e-3 if tc else 2e-3)
    assert O.max_abs_normalized(a, h_ex) < 1e-2
    form_err = O.max_abs_normalized(y_f, y_ex)
    assert O.max_abs_normalized(y, y_ex) < max(1e-2, form_err + 5e-4)


@pytest.mark.parametrize("n_tok", [1, 8])
def test_shared_expert_runs_with_the_routed_ones(n_tok, path):
    """The 256-expert model's layer shape (IQ4_NL, hidden 2048, expert FFN
    512) with an always-on shared expert: every token's ids are its top-k
    routed experts plus the shared expert (its own slot, weight 1.0), so the
    shared expert runs in the same grouped matmuls and combine. y matches
    the oracle, which sums the shared expert's output into every token."""
    from moestream_b200 import ops
    n_routed, top_k, K, n_ff = 8, 4, 2048, 512
    n_expert = n_routed + 1                      # expert n_routed is the shared one
    pools, slabs, slot_of = build_layer("iq4_nl", K, n_ff, n_expert, n_expert, False, seed=31)
    rng = np.random.default_rng(40 + n_tok)
    x = rng.normal(0, 1, size=(n_tok, K)).astype(np.float32)
    ids_r, w_r = topk_ids(rng, n_tok, n_routed, top_k)
    ids_e = np.concatenate([ids_r, np.full((n_tok, 1), n_routed, np.int32)], axis=1)
    w = np.concatenate([w_r, np.ones((n_tok, 1), np.float32)], axis=1)
    table = np.full(n_expert, -1, dtype=np.int32)
    for e, sl in slot_of.items():
        table[e] = sl
    slots = O.remap_table(ids_e, table, n_expert)
    r = ops.remap_group(torch.from_numpy(ids_e).cuda(), n_expert,
                        table=torch.from_numpy(table).cuda(), n_expert=n_expert)
    y = ops.moe_ffn(pools["gate"], pools["up"], pools["down"], torch.from_numpy(x).cuda(), r,
                    torch.from_numpy(w).cuda(), top_k + 1)
    torch.cuda.synchronize()
    y = y.cpu().numpy()
    f16 = path.startswith("tc")
    y_f, _ = O.moe_ffn("iq4_nl", slabs["gate"], slabs["up"], slabs["down"], K, n_ff, x, slots, w,
                       mode="f16" if f16 else "q8")
    y_ex, _ = O.moe_ffn("iq4_nl", slabs["gate"], slabs["up"], slabs["down"], K, n_ff, x, slots, w,
                        mode="exact")
    assert O.max_abs_normalized(y, y_f) < (1e-3 if f16 else 2e-3)
    assert O.max_abs_normalized(y, y_ex) < max(1e-2, O.max_abs_normalized(y_f, y_ex) + 5e-4)
    # The shared expert contributes to every token: without it y differs.
    y_routed, _ = O.moe_ffn("iq4_nl", slabs["gate"], slabs["up"], slabs["down"], K, n_ff, x,
                            slots[:, :top_k], w[:, :top_k], mode="exact")
    assert O.max_abs_normalized(y_routed, y_ex) > 1e-2


def test_unweighted_top1_writes_expert_output(path):
    """w omitted with top_k 1: y is the expert output itself, identical to
    weighting by 1.0."""
    from moestream_b200 import ops
    pools, slabs, slot_of = build_layer("mxfp4", 512, 256, 6, 4, False, seed=5)
    rng = np.random.default_rng(9)
    x = torch.from_numpy(rng.normal(0, 1, size=(12, 512)).astype(np.float32)).cuda()
    ids = torch.from_numpy(rng.integers(-1, 6, size=(12, 1)).astype(np.int32)).cuda()
    table = np.full(6, -1, dtype=np.int32)
    for e, s in slot_of.items():
        table[e] = s
    r = ops.remap_group(ids, 4, table=torch.from_numpy(table).cuda(), n_expert=6)
    ones = torch.ones(12, 1, dtype=torch.float32, device="cuda")
    want = ops.moe_ffn(pools["gate"], pools["up"], pools["down"], x, r, ones, 1)
    got = ops.moe_ffn(pools["gate"], pools["up"], pools["down"], x, r, None, 1)
    torch.cuda.synchronize()
    assert torch.equal(got, want)


@pytest.mark.parametrize("wtype,K,n_ff,n_expert,n_slot,n_tok,top_k,fused", [
    ("mxfp4", 2880, 2880, 6, 4, 3, 4, False),    # tensor cores
    ("mxfp4", 512, 256, 8, 8, 40, 4, True),      # tensor cores, fused gate_up, several passes
    ("iq4_nl", 2048, 512, 10, 8, 8, 8, False),   # CUDA cores and tensor cores (iq4_form)
])
def test_gpt_oss_activation_matches_oracle(wtype, K, n_ff, n_expert, n_slot, n_tok, top_k, fused,
                                           iq4_form):
    """gpt-oss's clamped SwiGLU (alpha 1.702, limit 7) in every path. The
    activations are scaled by 8 so that many gate and up values pass the
    clamp; tolerances as for plain SwiGLU."""
    from moestream_b200 import ops
    pools, slabs, slot_of = build_layer(wtype, K, n_ff, n_expert, n_slot, fused, seed=K + 7)
    rng = np.random.default_rng(3)
    x = (8 * rng.normal(0, 1, size=(n_tok, K))).astype(np.float32)
    ids_e, w = topk_ids(rng, n_tok, n_expert, top_k)
    table = np.full(n_expert, -1, dtype=np.int32)
    for e, s in slot_of.items():
        table[e] = s
    slots = O.remap_table(ids_e, table, n_slot)
    r = ops.remap_group(torch.from_numpy(ids_e).cuda(), n_slot,
                        table=torch.from_numpy(table).cuda(), n_expert=n_expert)
    act = torch.empty(n_tok, top_k, n_ff, dtype=torch.float32, device="cuda")
    y = ops.moe_ffn(pools["gate"], pools["up"], pools["down"], torch.from_numpy(x).cuda(), r,
                    torch.from_numpy(w).cuda(), top_k, up_row0=n_ff if fused else 0, act=act,
                    activation=("swiglu_oai", 1.702, 7.0))
    torch.cuda.synchronize()
    form = "e2m1x4" if wtype == "mxfp4" else iq4_form
    tc = form != "q8"
    up = slabs["gate"] if fused else slabs["up"]
    y_f, h_f = O.moe_ffn(wtype, slabs["gate"], up, slabs["down"], K, n_ff, x, slots, w,
                         mode=form, up_row0=n_ff if fused else 0, act=(1.702, 7.0))
    _, h_silu = O.moe_ffn(wtype, slabs["gate"], up, slabs["down"], K, n_ff, x, slots, w,
                          mode=form, up_row0=n_ff if fused else 0)
    assert np.abs(h_f).max() > 0 and not np.allclose(h_f, h_silu)  # not plain SwiGLU
    assert O.max_abs_normalized(act.cpu().numpy(), h_f) < (1e-4 if tc else 1e-5)
    assert O.max_abs_normalized(y.cpu().numpy(), y_f) < (1e-3 if tc else 2e-3)


def test_unknown_activation_is_refused():
    from moestream_b200 import MsbError, ops
    pools, _, _ = build_layer("iq4_nl", 256, 128, 4, 2, False, seed=1)
    r = ops.remap_group(torch.zeros(1, 1, dtype=torch.int32, device="cuda"), 2)
    x = torch.zeros(1, 256, device="cuda")
    for bad in (("swiglu_oai", 1.702, 0.0),):
        with pytest.raises(MsbError, match="activation"):
            ops.moe_ffn(pools["gate"], pools["up"], pools["down"], x, r, None, 1,
                        activation=bad)


@pytest.mark.parametrize("n_ff,pad", [(256, 32), (256, 96), (320, 0), (256, 64)])
def test_up_view_off_the_tile_grid(n_ff, pad):
    """A gate_up tensor whose up rows start 32, 64 or 96 rows into a 128-row
    tile (up_row0 = n_ff + pad, pad rows unused): the tensor cores take the
    up view's scale factors from two tiles. With n_ff = 320 the last window
    has no second tile in the pool."""
    from moestream_b200 import ops
    wtype, K, n_expert, n_slot, n_tok, top_k = "mxfp4", 512, 6, 5, 20, 4
    rows = 2 * n_ff + pad
    up_row0 = n_ff + pad
    gu = experts(wtype, n_expert, K, rows, seed=rows)
    dn = experts(wtype, n_expert, n_ff, K, seed=rows + 1)
    p_gu = ops.SlotPool(wtype, K, rows, n_slot)
    p_dn = ops.SlotPool(wtype, n_ff, K, n_slot)
    for p, m in ((p_gu, gu), (p_dn, dn)):
        p.fill(list(range(n_slot)), [torch.from_numpy(m[e]).pin_memory() for e in range(n_slot)])
    rng = np.random.default_rng(n_ff + pad)
    x = rng.normal(0, 1, size=(n_tok, K)).astype(np.float32)
    ids_e, w = topk_ids(rng, n_tok, n_expert, top_k)   # expert n_slot is not resident
    table = np.full(n_expert, -1, dtype=np.int32)
    table[:n_slot] = np.arange(n_slot)
    slots = O.remap_table(ids_e, table, n_slot)
    r = ops.remap_group(torch.from_numpy(ids_e).cuda(), n_slot,
                        table=torch.from_numpy(table).cuda(), n_expert=n_expert)
    act = torch.empty(n_tok, top_k, n_ff, dtype=torch.float32, device="cuda")
    y = ops.moe_ffn(p_gu, p_gu, p_dn, torch.from_numpy(x).cuda(), r, torch.from_numpy(w).cuda(),
                    top_k, up_row0=up_row0, act=act)
    torch.cuda.synchronize()
    pad_slab = lambda m: np.concatenate([m[:n_slot], np.zeros((1, m.shape[1]), np.uint8)])
    y_f, h_f = O.moe_ffn(wtype, pad_slab(gu), pad_slab(gu), pad_slab(dn), K, n_ff, x, slots, w,
                         mode="e2m1x4", up_row0=up_row0)
    assert O.max_abs_normalized(act.cpu().numpy(), h_f) < 1e-4
    assert O.max_abs_normalized(y.cpu().numpy(), y_f) < 1e-3


@pytest.mark.parametrize("wtype,K,n_ff,n_expert,n_slot,n_tok,top_k,fused", [
    ("mxfp4", 2880, 2880, 6, 4, 2, 4, True),     # 8 pairs: split over K, the reduce adds them
    ("mxfp4", 2880, 2880, 6, 4, 5, 4, True),     # fused gate_up, up view off the tile grid
    ("mxfp4", 512, 256, 8, 6, 40, 4, False),     # several passes per slot
    ("iq4_nl", 2048, 512, 10, 8, 8, 8, False),   # CUDA cores and tensor cores (iq4_form)
])
def test_expert_biases_match_oracle(wtype, K, n_ff, n_expert, n_slot, n_tok, top_k, fused,
                                    iq4_form):
    """gpt-oss expert biases, looked up by the router's expert ids (not the
    slots), added to every pair not routed to the zero slot; non-resident
    experts go to the zero slot and contribute exactly 0."""
    from moestream_b200 import ops
    pools, slabs, slot_of = build_layer(wtype, K, n_ff, n_expert, n_slot, fused, seed=K + 3)
    rng = np.random.default_rng(n_tok + 11)
    x = rng.normal(0, 1, size=(n_tok, K)).astype(np.float32)
    ids_e, w = topk_ids(rng, n_tok, n_expert, top_k)
    table = np.full(n_expert, -1, dtype=np.int32)
    for e, s in slot_of.items():
        table[e] = s
    slots = O.remap_table(ids_e, table, n_slot)
    assert (slots == n_slot).any() and (slots < n_slot).any()
    gb = rng.normal(0, 0.5, size=(n_expert, 2 * n_ff if fused else n_ff)).astype(np.float32)
    ub = None if fused else rng.normal(0, 0.5, size=(n_expert, n_ff)).astype(np.float32)
    db = rng.normal(0, 0.5, size=(n_expert, K)).astype(np.float32)
    ids_t = torch.from_numpy(ids_e).cuda()
    gb_t, db_t = torch.from_numpy(gb).cuda(), torch.from_numpy(db).cuda()
    ub_t = gb_t[:, n_ff:] if fused else torch.from_numpy(ub).cuda()
    r = ops.remap_group(ids_t, n_slot, table=torch.from_numpy(table).cuda(), n_expert=n_expert)
    act = torch.empty(n_tok, top_k, n_ff, dtype=torch.float32, device="cuda")
    y = ops.moe_ffn(pools["gate"], pools["up"], pools["down"], torch.from_numpy(x).cuda(), r,
                    torch.from_numpy(w).cuda(), top_k, up_row0=n_ff if fused else 0, act=act,
                    bias=(gb_t, ub_t, db_t, ids_t), activation=("swiglu_oai", 1.702, 7.0))
    torch.cuda.synchronize()
    form = "e2m1x4" if wtype == "mxfp4" else iq4_form
    tc = form != "q8"
    up = slabs["gate"] if fused else slabs["up"]
    ub_o = gb[:, n_ff:] if fused else ub
    y_f, h_f = O.moe_ffn(wtype, slabs["gate"], up, slabs["down"], K, n_ff, x, slots, w,
                         mode=form, up_row0=n_ff if fused else 0,
                         act=(1.702, 7.0), bias=(gb[:, :n_ff], ub_o, db, ids_e, n_expert))
    y_0, _ = O.moe_ffn(wtype, slabs["gate"], up, slabs["down"], K, n_ff, x, slots, w,
                       mode=form, up_row0=n_ff if fused else 0, act=(1.702, 7.0))
    assert O.max_abs_normalized(y_f, y_0) > 1e-2   # the biases matter
    a = act.cpu().numpy()
    assert np.all(a[slots == n_slot] == 0.0)
    assert O.max_abs_normalized(a, h_f) < (1e-4 if tc else 1e-5)
    assert O.max_abs_normalized(y.cpu().numpy(), y_f) < (1e-3 if tc else 2e-3)


@pytest.mark.parametrize("wtype,K,n_ff,n_tok", [("mxfp4", 512, 256, 48), ("mxfp4", 512, 256, 2),
                                               ("iq4_nl", 512, 256, 48)])
def test_combine_runs_in_the_down_epilogue(wtype, K, n_ff, n_tok):
    """No separate combine or split-over-K reduce kernel: one FFN call
    launches the activation preparation, gate/up and down (batches of up to
    8 pairs split K and the last segment of each row block finishes it), and
    y is the same bits on every call whichever CTA finishes a token's rows
    or a block's segments last."""
    from moestream_b200 import ops
    from moestream_b200._lib import lib
    top_k, n_expert = 4, 8
    pools, slabs, slot_of = build_layer(wtype, K, n_ff, n_expert, n_expert, False, seed=5)
    rng = np.random.default_rng(1)
    x = torch.from_numpy(rng.normal(0, 1, size=(n_tok, K)).astype(np.float32)).cuda()
    ids_e, w = topk_ids(rng, n_tok, n_expert, top_k)
    table = np.full(n_expert, -1, dtype=np.int32)
    for e, s in slot_of.items():
        table[e] = s
    r = ops.remap_group(torch.from_numpy(ids_e).cuda(), n_expert,
                        table=torch.from_numpy(table).cuda(), n_expert=n_expert)
    w_t = torch.from_numpy(w).cuda()
    ws = ops.workspace(K, n_tok, top_k, n_expert)
    torch.cuda.synchronize()
    c0 = int(lib().msb_kernel_launches())
    y0 = ops.moe_ffn(pools["gate"], pools["up"], pools["down"], x, r, w_t, top_k, ws=ws)
    launched = int(lib().msb_kernel_launches()) - c0
    assert launched == 3
    ys = [ops.moe_ffn(pools["gate"], pools["up"], pools["down"], x, r, w_t, top_k, ws=ws).clone()
          for _ in range(3)]
    torch.cuda.synchronize()
    assert all(torch.equal(y0, yi) for yi in ys)
    slots = O.remap_table(ids_e, table, n_expert)
    # 48 tokens x top-4 over 8 slots is prompt-sized: IQ4_NL runs on the
    # tensor cores too (f16 form).
    want, _ = O.moe_ffn(wtype, slabs["gate"], slabs["up"], slabs["down"], K, n_ff,
                        x.cpu().numpy(), slots, w, mode="e2m1x4" if wtype == "mxfp4" else "f16")
    assert O.max_abs_normalized(y0.cpu().numpy(), want) < 1e-3

"""IQ4_NL on the tensor cores: the codebook dequantized to fp16 in shared
memory (d * kvalue, rounded once), tcgen05 kind::f16 MMAs, f32 accumulation.

Against the oracle's "f16" form (every weight d * kv and every activation
rounded to fp16, exact products): 1e-4 of the output's max for mul_mat_id,
1e-3 for the FFN; against exact f64: 1e-2 (this form is ~16x closer to exact
than ggml's q8_0 form, which is what shows that the tensor-core path ran).
Shapes: the 256-expert model's gate/up [512 x 2048] and down [2048 x 512],
the single-op shape [768 x 2048], passes of 1 to 64 pairs and several passes
per slot, and the zero slot.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import experts, topk_ids

pytestmark = pytest.mark.gpu


@pytest.fixture
def iq4nl_tc():
    from moestream_b200._lib import OPT_IQ4NL_PATH, check, lib
    check(lib().msb_set_option(OPT_IQ4NL_PATH, 2))
    yield
    check(lib().msb_set_option(OPT_IQ4NL_PATH, 0))


def pool_of(ex, K, N, n_slot, slot_of):
    from moestream_b200 import ops
    pool = ops.SlotPool("iq4_nl", K, N, n_slot)
    pool.fill(list(slot_of.values()), [torch.from_numpy(ex[e]).pin_memory() for e in slot_of])
    slab = np.zeros((n_slot + 1, ex.shape[1]), dtype=np.uint8)
    for e, s in slot_of.items():
        slab[s] = ex[e]
    torch.cuda.synchronize()
    return pool, slab


@pytest.mark.parametrize("K,N,n_expert,n_slot,n_tok,top_k,b_ne1", [
    (2048, 512, 12, 8, 16, 8, 1),     # gate/up width of the 256-expert model
    (512, 2048, 12, 8, 16, 8, 8),     # its down projection (one row per (token, k))
    (2048, 768, 16, 8, 1, 8, 1),      # the single-op shape: 1 pair per slot
    (512, 256, 6, 3, 100, 4, 1),      # ~130 pairs per slot: three passes of 64
    (192, 136, 6, 4, 9, 2, 1),        # N not a multiple of 128 (partial tile)
])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_mul_mat_id_on_tensor_cores(K, N, n_expert, n_slot, n_tok, top_k, b_ne1, dtype, iq4nl_tc):
    from moestream_b200 import ops
    rng = np.random.default_rng(K + N + n_tok)
    ex = experts("iq4_nl", n_expert, K, N, seed=K)
    resident = rng.permutation(n_expert)[:n_slot]
    slot_of = {int(resident[i]): int(s) for i, s in enumerate(rng.permutation(n_slot))}
    pool, slab = pool_of(ex, K, N, n_slot, slot_of)
    ids = rng.integers(0, n_slot + 1, size=(n_tok, top_k)).astype(np.int32)  # incl. zero slot
    b = rng.normal(0, 1, size=(n_tok, b_ne1, K)).astype(np.float32)
    if dtype == torch.bfloat16:
        b = torch.from_numpy(b).to(torch.bfloat16).float().numpy()
    bt = torch.from_numpy(b).cuda().to(dtype)
    r = ops.remap_group(torch.from_numpy(ids).cuda(), n_slot)
    got = ops.mul_mat_id(pool, bt, r, top_k)
    torch.cuda.synchronize()
    got = got.cpu().numpy()
    want = O.mul_mat_id("iq4_nl", slab, K, N, b, ids, mode="f16")
    exact = O.mul_mat_id("iq4_nl", slab, K, N, b, ids, mode="exact")
    assert O.max_abs_normalized(got, want) < 1e-4
    assert O.max_abs_normalized(got, exact) < 1e-2
    assert np.all(got[ids == n_slot] == 0.0)
    assert ops.device_status() == 0


@pytest.mark.parametrize("K,n_ff,n_expert,n_slot,n_tok,top_k,fused,act,bias", [
    (2048, 512, 12, 8, 24, 8, False, None, False),         # the 256-expert model's layer
    (2048, 512, 12, 8, 24, 8, True, None, False),          # fused gate_up (up rows from 512)
    (512, 256, 8, 6, 64, 4, False, (1.702, 7.0), True),    # gpt-oss activation and biases
])
def test_moe_ffn_on_tensor_cores(K, n_ff, n_expert, n_slot, n_tok, top_k, fused, act, bias,
                                 iq4nl_tc):
    from moestream_b200 import ops
    rng = np.random.default_rng(n_tok + K)
    resident = rng.permutation(n_expert)[:n_slot]
    slot_of = {int(e): int(s) for e, s in zip(resident, rng.permutation(n_slot))}
    if fused:
        gu = experts("iq4_nl", n_expert, K, 2 * n_ff, seed=1)
        p_gu, s_gu = pool_of(gu, K, 2 * n_ff, n_slot, slot_of)
        p_g = p_u = p_gu
        s_g = s_u = s_gu
    else:
        p_g, s_g = pool_of(experts("iq4_nl", n_expert, K, n_ff, seed=1), K, n_ff, n_slot, slot_of)
        p_u, s_u = pool_of(experts("iq4_nl", n_expert, K, n_ff, seed=2), K, n_ff, n_slot, slot_of)
    p_d, s_d = pool_of(experts("iq4_nl", n_expert, n_ff, K, seed=3), n_ff, K, n_slot, slot_of)
    x = rng.normal(0, 1, size=(n_tok, K)).astype(np.float32)
    ids_e, w = topk_ids(rng, n_tok, n_expert, top_k)
    table = np.full(n_expert, -1, dtype=np.int32)
    for e, s in slot_of.items():
        table[e] = s
    slots = O.remap_table(ids_e, table, n_slot)
    ids_t = torch.from_numpy(ids_e).cuda()
    r = ops.remap_group(ids_t, n_slot, table=torch.from_numpy(table).cuda(), n_expert=n_expert)
    up_row0 = n_ff if fused else 0
    kw = {}
    bias_o = None
    if bias:
        gb = rng.normal(0, 0.5, size=(n_expert, n_ff)).astype(np.float32)
        ub = rng.normal(0, 0.5, size=(n_expert, n_ff)).astype(np.float32)
        db = rng.normal(0, 0.5, size=(n_expert, K)).astype(np.float32)
        kw["bias"] = tuple(torch.from_numpy(a).cuda() for a in (gb, ub, db)) + (ids_t,)
        bias_o = (gb, ub, db, ids_e, n_expert)
    if act:
        kw["activation"] = ("swiglu_oai",) + act
    h = torch.empty(n_tok, top_k, n_ff, dtype=torch.float32, device="cuda")
    y = ops.moe_ffn(p_g, p_u, p_d, torch.from_numpy(x).cuda(), r, torch.from_numpy(w).cuda(),
                    top_k, up_row0=up_row0, act=h, **kw)
    torch.cuda.synchronize()
    y_f, h_f = O.moe_ffn("iq4_nl", s_g, s_u, s_d, K, n_ff, x, slots, w, mode="f16",
                         up_row0=up_row0, act=act, bias=bias_o)
    y_x, _ = O.moe_ffn("iq4_nl", s_g, s_u, s_d, K, n_ff, x, slots, w, mode="exact",
                       up_row0=up_row0, act=act, bias=bias_o)
    assert O.max_abs_normalized(h.cpu().numpy(), h_f) < 1e-4
    assert O.max_abs_normalized(y.cpu().numpy(), y_f) < 1e-3
    assert O.max_abs_normalized(y.cpu().numpy(), y_x) < 1e-2
    assert ops.device_status() == 0


def test_prompt_sized_batches_choose_the_tensor_cores():
    """With the default policy a batch of >= 4 pairs per reachable slot runs
    on the tensor cores (f16 form) and a decode batch on the CUDA cores
    (q8_0 form): the two forms are far enough apart to tell which ran."""
    from moestream_b200 import ops
    K, N, n_slot, top_k = 512, 256, 4, 4
    ex = experts("iq4_nl", n_slot, K, N, seed=9)
    pool, slab = pool_of(ex, K, N, n_slot, {e: e for e in range(n_slot)})
    rng = np.random.default_rng(1)
    for n_tok, form in ((40, "f16"), (1, "q8")):
        ids = np.stack([rng.permutation(n_slot)[:top_k] for _ in range(n_tok)]).astype(np.int32)
        b = rng.normal(0, 1, size=(n_tok, 1, K)).astype(np.float32)
        r = ops.remap_group(torch.from_numpy(ids).cuda(), n_slot)
        got = ops.mul_mat_id(pool, torch.from_numpy(b).cuda(), r, top_k)
        torch.cuda.synchronize()
        got = got.cpu().numpy()
        other = "q8" if form == "f16" else "f16"
        e_form = O.max_abs_normalized(got, O.mul_mat_id("iq4_nl", slab, K, N, b, ids, mode=form))
        e_other = O.max_abs_normalized(got, O.mul_mat_id("iq4_nl", slab, K, N, b, ids, mode=other))
        assert e_form < 1e-4 and e_other > 1e-3, (n_tok, e_form, e_other)

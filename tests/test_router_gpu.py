"""Device router (msb_router_topk) against a numpy restatement: ids equal to
a stable descending argsort's first top_k (lower expert index first among
equal logits, NaN as -inf), weights within 1e-6 of a float64 softmax over
the selected logits ("topk") or over all experts ("all"). Covers every
register layout (n_expert up to 1024), f32/f16/bf16 logits, strided rows,
ties, -inf/NaN rows, and the router feeding remap_group."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(logits, top_k, mode):
    l = np.where(np.isnan(logits), -np.inf, logits.astype(np.float64))
    ids = np.argsort(-l, axis=1, kind="stable")[:, :top_k].astype(np.int32)
    sel = np.take_along_axis(l, ids, axis=1)
    m = sel[:, :1]
    flat = np.isneginf(m)
    m = np.where(flat, 0.0, m)
    ex = np.where(flat, 1.0, np.exp(sel - m))
    if mode == "topk":
        z = ex.sum(axis=1, keepdims=True)
    else:
        z = np.where(flat, l.shape[1], np.exp(l - m).sum(axis=1, keepdims=True))
    return ids, ex / z


@pytest.mark.parametrize("n_expert", [8, 32, 100, 128, 256, 384, 1024])
@pytest.mark.parametrize("top_k", [1, 4, 8, 32])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("mode", ["topk", "all"])
def test_router_matches_reference(n_expert, top_k, dtype, mode):
    from moestream_b200 import ops
    if top_k > n_expert:
        pytest.skip("top_k > n_expert")
    rng = np.random.default_rng(n_expert * 100 + top_k)
    n_tok = 37
    base = rng.normal(0, 2, size=(n_tok, n_expert + 5)).astype(np.float32)
    base[3] = np.round(base[3])                         # many ties
    base[5] = rng.integers(-1, 2, size=n_expert + 5)     # three values only
    base[7, ::3] = -np.inf
    base[9, 1::4] = np.nan
    base[11] = -np.inf                                   # uniform weights
    dev = torch.from_numpy(base).to(dtype).cuda()[:, 2:2 + n_expert]   # strided rows
    ids, w = ops.router_topk(dev, top_k, mode=mode)
    torch.cuda.synchronize()
    want_ids, want_w = _ref(dev.float().cpu().numpy(), top_k, mode)
    assert np.array_equal(ids.cpu().numpy(), want_ids)
    assert np.abs(w.cpu().numpy() - want_w).max() < 1e-6


def test_router_feeds_the_remap():
    from moestream_b200 import ops
    rng = np.random.default_rng(4)
    n_tok, n_expert, top_k, n_slot = 64, 128, 4, 32
    logits = torch.from_numpy(rng.normal(size=(n_tok, n_expert)).astype(np.float32)).cuda()
    ids, w = ops.router_topk(logits, top_k)
    table = np.full(n_expert, -1, np.int32)
    table[rng.permutation(n_expert)[:n_slot]] = np.arange(n_slot, dtype=np.int32)
    route = ops.remap_group(ids, n_slot, table=torch.from_numpy(table).cuda(), n_expert=n_expert)
    torch.cuda.synchronize()
    want_ids, _ = _ref(logits.cpu().numpy(), top_k, "topk")
    slots = np.where(table[want_ids] >= 0, table[want_ids], n_slot)
    assert np.array_equal(route.slot_ids[:n_tok * top_k].cpu().numpy(), slots.ravel())
    assert np.allclose(w.sum(dim=1).cpu().numpy(), 1.0, atol=1e-6)


def test_router_rejects_bad_shapes():
    from moestream_b200 import MsbError, ops
    x = torch.zeros(4, 2048, device="cuda")
    with pytest.raises(MsbError):
        ops.router_topk(x, 4)                            # n_expert > 1024
    with pytest.raises(MsbError):
        ops.router_topk(x[:, :16], 17)                   # top_k > n_expert
    with pytest.raises(MsbError):
        ops.router_topk(x[:, :64], 33)                   # top_k > 32

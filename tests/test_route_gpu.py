"""Device remap + per-slot grouping, bit-exact against the oracle."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import topk_ids, zipf_bias

pytestmark = pytest.mark.gpu


def run_route(ids_np, n_slot, table=None, n_expert=None, strided=False):
    from moestream_b200 import ops
    ids = torch.from_numpy(ids_np).cuda()
    if strided:  # non-contiguous view: every other column of a wider tensor
        big = torch.zeros(ids.shape[0], ids.shape[1] * 2, dtype=torch.int32, device="cuda")
        big[:, ::2] = ids
        ids = big[:, ::2]
    tb = torch.from_numpy(table).cuda() if table is not None else None
    r = ops.remap_group(ids, n_slot, table=tb, n_expert=n_expert)
    torch.cuda.synchronize()
    return r


def check_route(r, ids_np, n_slot, table=None):
    if table is not None:
        slots = O.remap_table(ids_np, table, n_slot).reshape(-1)
    else:
        s = ids_np.reshape(-1).astype(np.int64)
        slots = np.where((s >= 0) & (s <= n_slot), s, n_slot).astype(np.int32)
    counts, offsets, rows, active = O.group(slots, n_slot)
    n_pairs = slots.size
    assert np.array_equal(r.slot_ids[:n_pairs].cpu().numpy(), slots)
    assert np.array_equal(r.counts.cpu().numpy(), counts)
    assert np.array_equal(r.offsets.cpu().numpy(), offsets)
    assert np.array_equal(r.rows[:n_pairs].cpu().numpy(), rows)
    act = r.active.cpu().numpy()
    assert act[0] == active.size
    assert np.array_equal(act[1:1 + active.size], active)


CASES = [
    # (n_tok, top_k, n_expert, n_slot, zipf)
    (1, 8, 128, 32, False),     # IQ4_NL single op
    (1, 4, 128, 32, False),     # gpt-oss decode
    (4, 4, 128, 32, False),
    (16, 4, 128, 32, False),
    (512, 4, 128, 32, True),    # prefill, Zipf(1.1) popularity
    (8, 8, 256, 64, False),     # 256-expert decode
    (2048, 4, 128, 128, True),  # all-resident prefill
    (3000, 8, 256, 1100, False),  # more slots than one thread block
]


@pytest.mark.parametrize("n_tok,top_k,n_expert,n_slot,zipf", CASES)
@pytest.mark.parametrize("strided", [False, True])
def test_remap_group_table(n_tok, top_k, n_expert, n_slot, zipf, strided):
    rng = np.random.default_rng(n_tok * 7 + top_k)
    bias = zipf_bias(rng, n_expert) if zipf else None
    ids, _ = topk_ids(rng, n_tok, n_expert, top_k, bias)
    # Table: a random subset of experts resident, the rest not (-1).
    table = np.full(n_expert, -1, dtype=np.int32)
    res = rng.permutation(n_expert)[:min(n_slot, n_expert)]
    table[res] = rng.permutation(n_slot)[:res.size]
    ids[0, 0] = -3  # invalid ids go to the zero slot
    ids[-1, -1] = n_expert + 1
    r = run_route(ids, n_slot, table, n_expert, strided)
    check_route(r, ids, n_slot, table)


@pytest.mark.parametrize("n_tok,top_k,n_slot", [(1, 8, 32), (64, 4, 128), (700, 4, 32)])
def test_remap_group_passthrough(n_tok, top_k, n_slot):
    """ids already hold slot ids (the host streamer's output)."""
    rng = np.random.default_rng(5)
    ids = rng.integers(-2, n_slot + 3, size=(n_tok, top_k)).astype(np.int32)
    r = run_route(ids, n_slot)
    check_route(r, ids, n_slot)


def test_remap_group_all_one_slot_and_empty():
    ids = np.full((300, 4), 7, dtype=np.int32)
    r = run_route(ids, 16)
    check_route(r, ids, 16)
    # zero tokens: counts all zero, no active slots
    from moestream_b200 import ops
    z = torch.zeros(0, 4, dtype=torch.int32, device="cuda")
    rr = ops.remap_group(z, 16)
    torch.cuda.synchronize()
    assert int(rr.active[0]) == 0 and int(rr.counts.sum()) == 0


@pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built")
def test_streamer_table_on_device_matches_reference_remap():
    """Host streamer -> expert->slot table -> device remap reproduces the
    reference ms_remap_fn loop (compiled reference ExpertCache) exactly."""
    from moestream_b200 import SlotStreamer
    n_expert, n_slot, top_k = 128, 32, 4
    st = SlotStreamer(1, n_expert, n_slot)
    ref = O.RefRemap(n_expert, n_slot)
    rng = np.random.default_rng(9)
    for n_tok in [1, 4, 16, 1, 4, 16, 64]:
        ids, _ = topk_ids(rng, n_tok, n_expert, top_k)
        _, _, table = st.remap(0, ids, want_table=True)
        want, _ = ref(ids)
        r = run_route(ids, n_slot, table, n_expert)
        assert np.array_equal(r.slot_ids[:ids.size].cpu().numpy(), want.reshape(-1))
        check_route(r, ids, n_slot, table)

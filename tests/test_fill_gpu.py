"""Slot fills: host (pinned and pageable) and device sources round-trip
bit-exactly through the pool's device layout; bad slots are rejected; fills
batch through the staging area in several rounds; fills on a side stream
ordered by an event before the matmul reads the slot."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import experts

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("wtype,K,N", [("iq4_nl", 2048, 768), ("mxfp4", 2880, 640),
                                       ("mxfp4", 96, 40), ("iq4_nl", 512, 2048)])
@pytest.mark.parametrize("source", ["pinned", "pageable", "device"])
def test_fill_round_trip(wtype, K, N, source):
    from moestream_b200 import ops
    n_slot = 5
    ex = experts(wtype, 7, K, N, seed=K)
    pool = ops.SlotPool(wtype, K, N, n_slot, max_fill_batch=2)  # 7 fills -> 4 batches
    slots = [3, 0, 4, 1, 2, 0, 3]  # later fills overwrite earlier ones
    srcs = [torch.from_numpy(ex[i]) for i in range(7)]
    if source == "pinned":
        srcs = [s.pin_memory() for s in srcs]
    elif source == "device":
        srcs = [s.cuda() for s in srcs]
    pool.fill(slots, srcs)
    torch.cuda.synchronize()
    last = {}
    for i, s in enumerate(slots):
        last[s] = i
    for s, i in last.items():
        got = pool.read_slot(s).cpu().numpy()
        assert np.array_equal(got, ex[i]), (s, i)
    assert int(pool.read_slot(n_slot).to(torch.int64).sum()) == 0  # zero slot untouched


def test_fill_rejects_bad_slot():
    from moestream_b200 import MsbError, ops
    pool = ops.SlotPool("iq4_nl", 64, 8, 2)
    src = torch.zeros(pool.expert_bytes, dtype=torch.uint8)
    for bad in (-1, 2, 99):  # 2 is the zero slot: not fillable
        with pytest.raises(MsbError):
            pool.fill([bad], [src])


def test_side_stream_fill_ordered_by_event():
    """A fill on a copy stream followed by an event wait on the compute
    stream: the matmul sees the new expert."""
    from moestream_b200 import ops
    wtype, K, N, n_slot = "mxfp4", 512, 256, 4
    ex = experts(wtype, 2, K, N, seed=8)
    pool = ops.SlotPool(wtype, K, N, n_slot)
    pool.fill([1], [torch.from_numpy(ex[0]).pin_memory()])
    copy = torch.cuda.Stream()
    done = torch.cuda.Event()
    with torch.cuda.stream(copy):
        pool.fill([1], [torch.from_numpy(ex[1]).pin_memory()], stream=copy)
        done.record(copy)
    torch.cuda.current_stream().wait_event(done)
    b = np.random.default_rng(1).normal(0, 1, size=(1, 1, K)).astype(np.float32)
    ids = np.array([[1]], dtype=np.int32)
    r = ops.remap_group(torch.from_numpy(ids).cuda(), n_slot)
    got = ops.mul_mat_id(pool, torch.from_numpy(b).cuda(), r, 1)
    torch.cuda.synchronize()
    slab = np.zeros((n_slot + 1, ex.shape[1]), dtype=np.uint8)
    slab[1] = ex[1]
    # MXFP4 with K % 64 == 0 runs on the tensor cores (activations as e2m1 terms)
    want = O.mul_mat_id(wtype, slab, K, N, b, ids, mode="e2m1x4")
    assert O.max_abs_normalized(got.cpu().numpy(), want) < 1e-4

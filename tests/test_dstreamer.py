"""Device slot streamer decisions (msb_dstreamer_*), run on the host.

The decision code the device kernel runs (dcache.cuh) is compiled for the
host too; a streamer made with on_host executes it on the calling thread.
On random traces (uniform and Zipf routing, duplicate ids within a call,
invalid ids, slot exhaustion, several layers) every call's slots, miss list
(expert, slot, first-seen order), expert -> slot table and the counters must
equal the host slot streamer's (msb_streamer_remap over the library's
ExpertCache, itself checked against the reference's compiled cache).
"""
import numpy as np
import pytest

from tests.helpers import topk_ids, zipf_bias


@pytest.mark.parametrize("n_layer,n_expert,n_slot,top_k,max_tok,zipf,seed", [
    (2, 128, 32, 4, 4, False, 0),      # gpt-oss decode shape
    (3, 128, 32, 4, 64, True, 1),      # batches beyond the slots: exhaustion
    (2, 256, 64, 8, 8, True, 2),       # 256 experts, top-8
    (1, 16, 8, 4, 6, False, 3),        # tiny: heavy eviction and ghost traffic
    (2, 64, 4, 2, 3, True, 4),         # fewer slots than pairs
])
def test_host_run_of_device_decisions_matches_streamer(n_layer, n_expert, n_slot, top_k,
                                                       max_tok, zipf, seed):
    from moestream_b200 import DeviceSlotStreamer, SlotStreamer
    rng = np.random.default_rng(seed)
    eb = 1000
    ref = SlotStreamer(n_layer, n_expert, n_slot, eb)
    dev = DeviceSlotStreamer(n_layer, n_expert, n_slot, max_tok * top_k, eb, on_host=True)
    bias = [zipf_bias(rng, n_expert) if zipf else None for _ in range(n_layer)]
    for step in range(60):
        for il in range(n_layer):
            n_tok = int(rng.integers(1, max_tok + 1))
            ids, _ = topk_ids(rng, n_tok, n_expert, top_k, bias=bias[il])
            if step % 7 == 3:
                ids[0, -1] = -1                              # invalid ids take the zero slot
                ids[-1, 0] = n_expert + 5
            if step % 5 == 1 and n_tok > 1:
                ids[1] = ids[0]                              # the same experts twice
            want, misses, table = ref.remap(il, ids, want_table=True)
            ids_t = np.ascontiguousarray(ids.T).T            # strided view, as ggml hands it
            got = dev.remap(il, ids_t)
            assert np.array_equal(got, want), (step, il)
            assert dev.misses(il) == misses, (step, il)
            assert np.array_equal(dev.table(il), table), (step, il)
    a, b = ref.stats(), dev.stats()
    assert a == b
    assert a["miss"] > 0 and a["hit"] > 0


def test_rejects_more_pairs_than_max_pairs():
    from moestream_b200 import DeviceSlotStreamer, MsbError
    dev = DeviceSlotStreamer(1, 16, 4, 8, on_host=True)
    with pytest.raises(MsbError, match="max_pairs"):
        dev.remap(0, np.zeros((3, 4), dtype=np.int32))
    with pytest.raises(MsbError):
        DeviceSlotStreamer(1, 16, 4, 8, on_host=True).remap(1, np.zeros((1, 4), np.int32))

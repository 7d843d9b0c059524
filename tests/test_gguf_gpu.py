"""Slot fills read from a GGUF file (msb_gguf_fill_slots_async) on the GPU.

- Bytes: experts read from a GGUF (single and split) land in the slots
  bit-exactly, over several calls in a row (both pinned staging halves, and a
  call that waits for the copies of the call before the previous one).
- The decode loop the reference runs per layer (ms_remap_fn,
  src/llama-moestream.cpp:1799-2105): the slot streamer remaps the router's
  expert ids, the misses are read from the GGUF into their slots, and
  mul_mat_id over the pool matches the oracle computed from the experts as
  written to the file.
- A tensor whose type or shape is not the pool's is refused.
"""
import numpy as np
import pytest
import torch
from gguf import GGMLQuantizationType as T

from oracle import oracle as O
from tests.helpers import experts, topk_ids, write_gguf

pytestmark = pytest.mark.gpu

GT = {"mxfp4": T.MXFP4, "iq4_nl": T.IQ4_NL}


def _file(tmp_path, wtype, n_layer, n_expert, K, N, split=0, seed=0):
    mats = {}
    tensors = []
    for il in range(n_layer):
        ex = experts(wtype, n_expert, K, N, seed=seed + il)
        mats[il] = ex
        tensors.append((f"blk.{il}.ffn_gate_exps.weight", ex.reshape(n_expert, N, -1), GT[wtype]))
    paths = write_gguf(tmp_path / "m.gguf", tensors, [("add_block_count", n_layer),
                                                      ("add_expert_count", n_expert)],
                       split_max_tensors=split)
    return paths, mats


@pytest.mark.parametrize("wtype,K,N,split", [("mxfp4", 2880, 256, 0), ("iq4_nl", 2048, 128, 1)])
def test_fill_from_gguf_round_trip(tmp_path, wtype, K, N, split):
    from moestream_b200 import ops
    from moestream_b200.gguf import GGUFFile
    n_expert, n_slot = 10, 6
    paths, mats = _file(tmp_path, wtype, 2, n_expert, K, N, split=split, seed=K)
    pool = ops.SlotPool(wtype, K, N, n_slot, max_fill_batch=2)
    with GGUFFile(paths[-1]) as g:
        ti = g.expert_tensor(1, "gate")
        assert g.tensors[ti]["shard"] == (1 if split else 0)
        calls = [([9, 2, 4], [0, 5, 1]), ([7], [3]), ([0, 8, 1, 6, 3], [2, 4, 0, 5, 1]),
                 ([5, 5], [3, 2])]
        last = {}
        for ex_ids, slots in calls:
            g.fill_slots(ti, pool, ex_ids, slots, n_threads=3)
            last.update(zip(slots, ex_ids))
        torch.cuda.synchronize()
        for s, e in last.items():
            assert np.array_equal(pool.read_slot(s).cpu().numpy(), mats[1][e]), (s, e)
        assert int(pool.read_slot(n_slot).to(torch.int64).sum()) == 0


def test_streamed_decode_from_gguf_matches_oracle(tmp_path):
    from moestream_b200 import SlotStreamer, ops
    from moestream_b200.gguf import GGUFFile
    wtype, K, N, n_layer, n_expert, n_slot, top_k, n_tok = "mxfp4", 512, 256, 2, 16, 8, 4, 2
    paths, mats = _file(tmp_path, wtype, n_layer, n_expert, K, N, seed=3)
    rng = np.random.default_rng(11)
    with GGUFFile(paths[0]) as g:
        streamer = SlotStreamer(n_layer, n_expert, n_slot, g.bytes_per_slot())
        pools = [ops.SlotPool(wtype, K, N, n_slot) for _ in range(n_layer)]
        n_miss = 0
        for step in range(4):
            for il in range(n_layer):
                ids, _ = topk_ids(rng, n_tok, n_expert, top_k)
                slots, misses, _ = streamer.remap(il, ids)
                n_miss += len(misses)
                if misses:
                    g.fill_slots(g.expert_tensor(il, "gate"), pools[il],
                                 [e for e, _ in misses], [s for _, s in misses])
                b = rng.normal(0, 1, size=(n_tok, 1, K)).astype(np.float32)
                route = ops.remap_group(torch.from_numpy(slots).cuda(), n_slot)
                got = ops.mul_mat_id(pools[il], torch.from_numpy(b).cuda(), route, top_k)
                slab = np.concatenate([mats[il], np.zeros((1, mats[il].shape[1]), np.uint8)])
                want = O.mul_mat_id(wtype, slab, K, N, b, ids, mode="e2m1x4")
                err = O.max_abs_normalized(got.cpu().numpy(), want)
                assert err < 1e-4, (step, il, err)
        assert n_miss > 0 and streamer.stats()["hit"] > 0


def test_fill_rejects_a_tensor_that_is_not_the_pools(tmp_path):
    from moestream_b200 import MsbError, ops
    from moestream_b200.gguf import GGUFFile
    paths, _ = _file(tmp_path, "mxfp4", 1, 4, 512, 64)
    with GGUFFile(paths[0]) as g:
        ti = g.expert_tensor(0, "gate")
        for pool in (ops.SlotPool("iq4_nl", 512, 64, 2), ops.SlotPool("mxfp4", 512, 128, 2)):
            with pytest.raises(MsbError, match="does not match the pool"):
                g.fill_slots(ti, pool, [0], [0])

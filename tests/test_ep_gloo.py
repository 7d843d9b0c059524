"""Expert-parallel host logic (moestream_b200.ep) with two gloo ranks on CPU.

Dispatch and combine are the oracle's CPU restatements of the device kernels;
the exchanges, buffer layout (activations plus the expert id in one row),
capacity blocks and the order of the steps are the product code. Each rank's
local FFN applies its own experts' matrices; the layer output of every rank
must equal the direct single-process computation for its tokens.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _expert_mats(n_expert, K, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(n_expert, K, K, generator=g) / K ** 0.5


def _rank_main(rank, port, n_expert, n_tok, top_k, K, seed, out_q):
    import torch.distributed as dist

    from moestream_b200.ep import ExpertParallel
    from oracle import oracle as O
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        mats = _expert_mats(n_expert, K, seed)
        g = torch.Generator().manual_seed(seed + 1)
        x_all = torch.randn(n_tok, K, generator=g)
        ids_all = torch.stack([torch.randperm(n_expert, generator=g)[:top_k]
                               for _ in range(n_tok)]).to(torch.int32)
        ids_all[0, 0] = -1                       # an invalid id contributes nothing
        w_all = torch.rand(n_tok, top_k, generator=g)
        ep = ExpertParallel(WORLD, rank, n_expert, n_tok, top_k, K, "cpu",
                            dispatch=O.ep_dispatch, combine=O.ep_combine)
        lo = rank * ep.t_loc
        x, ids, w = x_all[lo:lo + ep.t_loc], ids_all[lo:lo + ep.t_loc], w_all[lo:lo + ep.t_loc]
        local = mats[rank * ep.n_local:(rank + 1) * ep.n_local]

        def local_ffn(rows, local_ids, route, out):
            assert route is None
            out.zero_()
            for r in range(rows.shape[0]):
                e = int(local_ids[r, 0])
                if e >= 0:
                    out[r] = rows[r].float() @ local[e]

        y = torch.empty(ep.t_loc, K)
        ep.layer(x, ids, w, local_ffn, y)
        ep.layer(x, ids, w, local_ffn, y)        # buffers reused: same result
        want = torch.zeros(ep.t_loc, K)
        for t in range(ep.t_loc):
            for k in range(top_k):
                e = int(ids[t, k])
                if e >= 0:
                    want[t] += w[t, k] * (x[t].to(torch.bfloat16).float() @ mats[e])
        out_q.put((rank, float((y - want).abs().max() / want.abs().max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n_expert,n_tok,top_k,K", [(8, 6, 2, 16), (4, 4, 4, 8)])
def test_two_rank_layer_matches_single_process(n_expert, n_tok, top_k, K):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, port, n_expert, n_tok, top_k, K, 7, q))
             for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    codes = [p.exitcode for p in procs]
    assert codes == [0] * WORLD, codes
    errs = dict(q.get(timeout=5) for _ in range(WORLD))
    assert all(e < 1e-6 for e in errs.values()), errs


def test_rejects_uneven_split():
    from moestream_b200.ep import ExpertParallel
    with pytest.raises(ValueError):
        ExpertParallel(3, 0, 8, 6, 2, 16, "cpu", dispatch=lambda *a: None,
                       combine=lambda *a: None)


def test_owner_and_capacity():
    from moestream_b200.ep import ExpertParallel
    ep = ExpertParallel(4, 1, 128, 64, 4, 2880, "cpu", dispatch=lambda *a: None,
                        combine=lambda *a: None)
    assert ep.n_local == 32 and ep.t_loc == 16 and ep.cap == 64
    assert [ep.owner(e) for e in (0, 31, 32, 127)] == [0, 0, 1, 3]
    assert ep.send.shape == (256, 2882) and ep.recv_ids().shape == (256, 1)
    assert np.shares_memory(ep.send_ids().numpy(), ep.send.view(torch.int32).numpy())

"""A bounded device wait that runs out, on one GPU, without faulting it.

The expert-parallel exchange waits on flags that other GPUs raise. Here a
two-rank layout is built on one GPU: rank 0's own exchange buffer and a
second local buffer standing in for rank 1, which never dispatches. Rank 0
dispatches one layer of rows (raising its own layer count) and waits for
every rank's rows: rank 1's flag is never raised, so the wait gives up after
the configured limit (50 ms here instead of the default second), sets
status bit 32 and returns. The host sees MSB_ERR_TIMEOUT from
msb_stream_check, the message names the wait, and the device stays usable.
The reference has no waits of its kind (it fails safe to the zero slot,
src/llama-moestream.cpp:1913-1928).
"""
import ctypes
import time

import pytest
import torch

ERR_TIMEOUT = 5


@pytest.mark.gpu
def test_expert_parallel_wait_runs_out_and_reports():
    from moestream_b200 import ops
    from moestream_b200._lib import (EP_HANDLE_BYTES, OPT_WAIT_LIMIT_US, EpPeers, check, lib)
    L = lib()
    torch.cuda.set_device(0)
    n_rank, cap, K, n_local = 2, 8, 64, 4
    nbytes = int(L.msb_ep_buffer_bytes(n_rank, cap, K))
    bufs = []
    for _ in range(n_rank):
        b = ctypes.c_void_p()
        h = (ctypes.c_char * EP_HANDLE_BYTES)()
        check(L.msb_ep_buffer_create(nbytes, ctypes.byref(b), h))
        bufs.append(b)
    peers = EpPeers()
    peers.n_rank, peers.rank, peers.cap, peers.K = n_rank, 0, cap, K
    for r in range(n_rank):
        peers.peer[r] = bufs[r].value
    stream = torch.cuda.current_stream()
    st = ctypes.c_void_p(stream.cuda_stream)
    assert ops.device_status(clear=True) == 0
    check(L.msb_set_option(OPT_WAIT_LIMIT_US, 50_000))
    try:
        ids = torch.tensor([[0], [5], [2]], dtype=torch.int32, device="cuda")
        x = torch.randn(3, K, device="cuda").to(torch.bfloat16)
        pos = torch.empty(3, dtype=torch.int32, device="cuda")
        ops.ep_dispatch_peers(peers, ids, x, n_local, pos)
        t0 = time.perf_counter()
        check(L.msb_ep_wait(ctypes.byref(peers), 0, st))
        rc = L.msb_stream_check(st, 1)
        dt = time.perf_counter() - t0
        assert rc == ERR_TIMEOUT
        assert b"expert-parallel rows" in L.msb_last_error()
        assert 0.04 < dt < 5.0, dt
        # Cleared, and the device still runs work.
        assert ops.device_status() == 0
        r = ops.remap_group(torch.zeros(2, 2, dtype=torch.int32, device="cuda"), 4)
        assert L.msb_stream_check(st, 0) == 0
        assert r.counts[:5].cpu().tolist() == [4, 0, 0, 0, 0]
    finally:
        check(L.msb_set_option(OPT_WAIT_LIMIT_US, 1_000_000))
        torch.cuda.synchronize()
        for b in bufs:
            check(L.msb_ep_buffer_destroy(b))
        ops.device_status(clear=True)


def test_wait_limit_option_is_checked():
    from moestream_b200._lib import OPT_WAIT_LIMIT_US, lib
    L = lib()
    assert L.msb_set_option(OPT_WAIT_LIMIT_US, 0) != 0
    assert L.msb_set_option(OPT_WAIT_LIMIT_US, 60_000_001) != 0
    assert L.msb_set_option(OPT_WAIT_LIMIT_US, 1_000_000) == 0

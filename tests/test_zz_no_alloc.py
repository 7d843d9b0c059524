"""msb_mul_mat_id_noalloc: mul_mat_id for callers that cannot allocate device
memory (code running inside another runtime's allocator or memory hooks,
where cudaMalloc would re-enter them, and hosts that reserve all device
memory up front). It takes its workspace from a fixed 8 MiB array inside
the library instead of from the caller.

Called through the C ABI and compared with msb_mul_mat_id (caller-provided
workspace) on two calls in a row with different inputs, so that the second
call runs over the first call's leftovers in the shared array. The 1- and
2-token cases split K over idle CTAs, so their partial sums and the split
word also live in the shared array. Tolerances
are those of tests/test_mul_mat_id_gpu.py for the path each weight type
takes. This file is collected last on purpose.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import experts, topk_ids

pytestmark = pytest.mark.gpu

TOL = {"mxfp4": 1e-4, "iq4_nl": 1e-5}


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _call_noalloc(L, pool, b, route, top_k, out):
    n_tok, b_ne1, _ = b.shape
    es = b.element_size()
    return L.msb_mul_mat_id_noalloc(pool.handle, _ptr(b), 0 if b.dtype == torch.float32 else 30,
                                    b_ne1, b.stride(1) * es, b.stride(0) * es,
                                    ctypes.byref(route.c), top_k, n_tok, _ptr(out), None)


@pytest.mark.parametrize("wtype,K,N,n_expert,n_slot,n_tok,top_k", [
    ("mxfp4", 2880, 512, 16, 12, 64, 4),     # gpt-oss hidden width, decode batch
    ("mxfp4", 2880, 2880, 16, 12, 1, 4),     # 4 pairs: K split over idle CTAs, the
    ("mxfp4", 2880, 2880, 16, 12, 2, 4),     # partial sums in the shared array too
    ("iq4_nl", 2048, 256, 12, 8, 16, 8),
])
def test_noalloc_matches_mul_mat_id_twice(wtype, K, N, n_expert, n_slot, n_tok, top_k):
    from moestream_b200 import ops
    from moestream_b200._lib import check, lib
    L = lib()
    ex = experts(wtype, n_expert, K, N, seed=K + N)
    rng = np.random.default_rng(7)
    resident = rng.permutation(n_expert)[:n_slot]
    pool = ops.SlotPool(wtype, K, N, n_slot)
    pool.fill(list(range(n_slot)), [torch.from_numpy(ex[e]).pin_memory() for e in resident])
    table = np.full(n_expert, -1, dtype=np.int32)
    table[resident] = np.arange(n_slot, dtype=np.int32)
    for call in range(2):
        ids, _ = topk_ids(rng, n_tok, n_expert, top_k)
        b = torch.from_numpy(rng.normal(0, 1, size=(n_tok, 1, K)).astype(np.float32)).cuda()
        if call == 1:
            b = b.to(torch.bfloat16)
        route = ops.remap_group(torch.from_numpy(ids).cuda(), n_slot,
                                table=torch.from_numpy(table).cuda(), n_expert=n_expert)
        want = ops.mul_mat_id(pool, b, route, top_k)
        got = torch.full((n_tok, top_k, N), float("nan"), dtype=torch.float32, device="cuda")
        check(_call_noalloc(L, pool, b, route, top_k, got))
        torch.cuda.synchronize()
        err = O.max_abs_normalized(got.cpu().numpy(), want.cpu().numpy())
        assert err < TOL[wtype], (call, err)
        # Same kernels, same split over K, same summation order: the same bits.
        assert torch.equal(got, want), call


def test_noalloc_rejects_requests_beyond_its_scratch():
    from moestream_b200 import ops
    from moestream_b200._lib import lib
    L = lib()
    K, N, n_slot, n_tok, top_k = 2880, 128, 4, 512, 8    # needs far more than 8 MiB
    assert L.msb_workspace_bytes(K, n_tok, top_k, n_slot) > (8 << 20)
    pool = ops.SlotPool("mxfp4", K, N, n_slot)
    ids = np.zeros((n_tok, top_k), dtype=np.int32)
    route = ops.remap_group(torch.from_numpy(ids).cuda(), n_slot)
    b = torch.zeros(n_tok, 1, K, dtype=torch.float32, device="cuda")
    out = torch.empty(n_tok, top_k, N, dtype=torch.float32, device="cuda")
    rc = _call_noalloc(L, pool, b, route, top_k, out)
    assert rc != 0
    assert b"scratch" in L.msb_last_error()

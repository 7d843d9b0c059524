"""mul_mat_id over the slot pool against the CPU oracle.

Two arithmetic paths: MXFP4 with K a multiple of 64 runs on the tensor
cores (activations as four e2m1 terms per block), everything else on the
CUDA cores (int8 activations, ggml's q8_0 form); MXFP4 cases run both, the
tensor cores with passes chosen by batch size ("tc") and with 24-pair
passes forced ("tc_wide"). With "tc", IQ4_NL with K a multiple of 64 and
N of 8 runs on the tensor cores too (weights dequantized to fp16: the
oracle's f16 form, within 1e-4).
Tolerances (max |got - want| / max |want|):
  - vs the oracle in the path's own form: 1e-5 (q8; f32 block sums in
    another order) or 1e-4 (e2m1x4; f32 tensor-core accumulation);
  - vs the exact f64 oracle: 1e-2, the bound stated for this path.
Properties from the reference's spikes: bit-identical results under slot
permutation (s0 T3), unreferenced slots harmless (s0 T4), the zero slot
gives exactly 0 (s3), split expert sets add up (s4).
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import experts, topk_ids

pytestmark = pytest.mark.gpu

TOL_Q8 = 1e-5
TOL_TC = 1e-4
TOL_EXACT = 1e-2


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


def oracle_mode(wtype, K, path, N=None):
    from moestream_b200 import ops
    if not path.startswith("tc"):
        return "q8"
    if wtype == "iq4_nl":
        return "f16" if ops.f16_eligible(K, N) else "q8"
    return "e2m1x4" if ops.tc_eligible(wtype, K) else "q8"


def make_pool(wtype, K, N, n_slot, slab_bytes, slots):
    from moestream_b200 import ops
    pool = ops.SlotPool(wtype, K, N, n_slot)
    srcs = [torch.from_numpy(slab_bytes[i]).pin_memory() for i in range(len(slots))]
    pool.fill(slots, srcs)
    torch.cuda.synchronize()
    return pool


def gpu_mmid(pool, b_np, ids_np, dtype=torch.float32):
    from moestream_b200 import ops
    b = torch.from_numpy(b_np).cuda().to(dtype)
    ids = torch.from_numpy(ids_np).cuda()
    r = ops.remap_group(ids, pool.n_slot)
    out = ops.mul_mat_id(pool, b, r, ids_np.shape[1])
    torch.cuda.synchronize()
    return out.cpu().numpy()


def slab_for(ex, slot_of_expert, n_slot):
    """ggml-layout slab [n_slot + 1, bytes] holding expert e in slot_of_expert[e]."""
    slab = np.zeros((n_slot + 1, ex.shape[1]), dtype=np.uint8)
    for e, s in slot_of_expert.items():
        slab[s] = ex[e]
    return slab


SHAPES = [
    # wtype, K, N, n_expert, n_slot, n_tok, top_k, b_ne1
    ("iq4_nl", 2048, 768, 16, 8, 1, 8, 1),    # single-op shape (fewer experts)
    ("iq4_nl", 512, 2048, 12, 8, 8, 8, 8),    # 256-expert model's down projection shape
    ("mxfp4", 2880, 256, 10, 6, 4, 4, 1),     # gpt-oss K (90 blocks: uneven warp split)
    ("mxfp4", 2880, 2880, 6, 4, 3, 4, 4),     # gpt-oss down: last 128-row tile half full
    ("mxfp4", 256, 96, 8, 5, 60, 4, 4),       # many pairs per slot (> 8 and > 32: passes)
    ("mxfp4", 2880, 384, 6, 3, 64, 4, 1),     # prompt-sized: ~8 passes per slot, 3 row tiles
    ("mxfp4", 96, 64, 6, 4, 5, 2, 1),         # K not a multiple of 64: CUDA cores
    ("iq4_nl", 96, 40, 6, 4, 5, 2, 1),        # N not a multiple of 32
]


@pytest.mark.parametrize("wtype,K,N,n_expert,n_slot,n_tok,top_k,b_ne1", SHAPES)
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_mul_mat_id_matches_oracle(wtype, K, N, n_expert, n_slot, n_tok, top_k, b_ne1, dtype,
                                   path):
    rng = np.random.default_rng(K + N + n_tok)
    ex = experts(wtype, n_expert, K, N, seed=0)
    resident = rng.permutation(n_expert)[:n_slot]
    slot_of = {int(resident[i]): int(s) for i, s in enumerate(rng.permutation(n_slot))}
    pool = make_pool(wtype, K, N, n_slot, [ex[e] for e in slot_of], list(slot_of.values()))
    ids = rng.integers(0, n_slot + 1, size=(n_tok, top_k)).astype(np.int32)  # incl. zero slot
    b = rng.normal(0, 1, size=(n_tok, b_ne1, K)).astype(np.float32)
    if dtype == torch.bfloat16:
        b = torch.from_numpy(b).to(torch.bfloat16).float().numpy()  # oracle sees bf16 values
    got = gpu_mmid(pool, b, ids, dtype)
    slab = slab_for(ex, slot_of, n_slot)
    mode = oracle_mode(wtype, K, path, N)
    want_form = O.mul_mat_id(wtype, slab, K, N, b, ids, mode=mode)
    want = O.mul_mat_id(wtype, slab, K, N, b, ids, mode="exact")
    assert O.max_abs_normalized(got, want_form) < (TOL_Q8 if mode == "q8" else TOL_TC)
    assert O.max_abs_normalized(got, want) < TOL_EXACT
    # Rows routed to the zero slot are exactly zero.
    z = ids == n_slot
    assert np.all(got[z] == 0.0)


def test_slot_permutation_is_bit_identical(path):
    wtype, K, N, n_slot = "mxfp4", 512, 128, 6
    ex = experts(wtype, 6, K, N, seed=1)
    rng = np.random.default_rng(2)
    b = rng.normal(0, 1, size=(9, 1, K)).astype(np.float32)
    ids_e = rng.integers(0, 6, size=(9, 4)).astype(np.int32)  # expert ids
    outs = []
    for perm_seed in (0, 1):
        perm = np.random.default_rng(perm_seed).permutation(n_slot)  # expert e -> slot perm[e]
        pool = make_pool(wtype, K, N, n_slot, [ex[e] for e in range(6)], perm.tolist())
        outs.append(gpu_mmid(pool, b, perm[ids_e].astype(np.int32)))
    assert np.array_equal(outs[0], outs[1])


def test_unreferenced_slots_do_not_matter():
    wtype, K, N, n_slot = "iq4_nl", 256, 64, 5
    ex = experts(wtype, 8, K, N, seed=3)
    rng = np.random.default_rng(4)
    b = rng.normal(0, 1, size=(4, 1, K)).astype(np.float32)
    ids = np.array([[0, 2], [2, 0], [0, 2], [2, 0]], dtype=np.int32)
    p1 = make_pool(wtype, K, N, n_slot, [ex[0], ex[1], ex[2]], [0, 1, 2])
    p2 = make_pool(wtype, K, N, n_slot, [ex[0], ex[5], ex[2], ex[7]], [0, 1, 2, 3])
    assert np.array_equal(gpu_mmid(p1, b, ids), gpu_mmid(p2, b, ids))


def test_split_expert_sets_add_up(path):
    """FFN-style additivity at the matmul: routing half the ids to the zero
    slot in each of two calls sums to the full call (s4's property)."""
    wtype, K, N, n_slot = "mxfp4", 256, 64, 8
    ex = experts(wtype, 8, K, N, seed=5)
    pool = make_pool(wtype, K, N, n_slot, [ex[e] for e in range(8)], list(range(8)))
    rng = np.random.default_rng(6)
    b = rng.normal(0, 1, size=(6, 1, K)).astype(np.float32)
    ids = rng.integers(0, 8, size=(6, 4)).astype(np.int32)
    full = gpu_mmid(pool, b, ids)
    lo = np.where(ids < 4, ids, n_slot).astype(np.int32)
    hi = np.where(ids >= 4, ids, n_slot).astype(np.int32)
    s = gpu_mmid(pool, b, lo) + gpu_mmid(pool, b, hi)
    assert np.array_equal(full, s)  # each row comes entirely from one call


def test_zero_slot_exact_zero_even_from_memory(path):
    """The zero slot's bytes are zeros and a row routed there is 0."""
    from moestream_b200 import ops
    pool = ops.SlotPool("mxfp4", 128, 32, 3)
    z = pool.read_slot(3)
    torch.cuda.synchronize()
    assert int(z.to(torch.int64).sum()) == 0
    b = np.random.default_rng(0).normal(0, 1, size=(2, 1, 128)).astype(np.float32)
    got = gpu_mmid(pool, b, np.full((2, 3), 3, dtype=np.int32))
    assert np.all(got == 0.0)


def test_device_status_clear_after_tensor_core_runs():
    """Every bounded wait of the tensor-core kernels completed in the runs
    above and in this one (the status word holds no bit)."""
    from moestream_b200 import ops
    ops.set_mxfp4_path("tc")
    wtype, K, N, n_slot = "mxfp4", 512, 256, 6
    ex = experts(wtype, n_slot, K, N, seed=11)
    pool = make_pool(wtype, K, N, n_slot, [ex[e] for e in range(n_slot)], list(range(n_slot)))
    rng = np.random.default_rng(12)
    b = rng.normal(0, 1, size=(20, 1, K)).astype(np.float32)
    ids = rng.integers(0, n_slot + 1, size=(20, 4)).astype(np.int32)
    gpu_mmid(pool, b, ids)
    torch.cuda.synchronize()
    assert ops.device_status() == 0

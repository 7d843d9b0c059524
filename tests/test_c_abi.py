"""The C ABI library loads and exports every entry point include/msb.h declares
(no compute calls: these run without a GPU)."""
import ctypes
import os
import re

from tests.conftest import ROOT

HEADER = os.path.join(ROOT, "include", "msb.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(msb_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_boundary():
    names = declared_functions()
    for must in ("msb_remap_group", "msb_mul_mat_id", "msb_moe_ffn", "msb_pool_create",
                 "msb_fill_slots_async", "msb_cache_acquire", "msb_streamer_remap",
                 "msb_last_error"):
        assert must in names


def test_library_exports_every_declared_symbol():
    from moestream_b200._lib import LIB_PATH, SIGNATURES
    assert os.path.exists(LIB_PATH), "build libmsb.so first (moestream_b200/csrc/build.py)"
    lib = ctypes.CDLL(LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing
    # The Python binding covers the whole header, nothing more.
    assert sorted(SIGNATURES) == declared_functions()


def test_host_only_entry_points():
    from moestream_b200._lib import TYPE_IQ4_NL, TYPE_MXFP4, lib
    L = lib()
    assert L.msb_version() >= 100
    # Expert sizes of the workloads (per role, ggml bytes).
    assert L.msb_expert_bytes(TYPE_IQ4_NL, 2048, 768) == 884736
    assert L.msb_expert_bytes(TYPE_MXFP4, 2880, 5760) == 8812800
    assert L.msb_expert_bytes(TYPE_MXFP4, 2880, 2880) == 4406400
    assert L.msb_expert_bytes(TYPE_IQ4_NL, 2048, 512) == 589824
    assert L.msb_expert_bytes(TYPE_IQ4_NL, 100, 4) == -1
    assert L.msb_expert_bytes(7, 64, 4) == -1


def test_slab_sizing_and_arena_threshold():
    """Slot counts and the arena threshold follow the reference's formulas
    (src/llama-moestream.cpp:1017-1086, :1530-1543)."""
    from moestream_b200._lib import lib
    L = lib()
    # 128 experts, frac 0.25 -> 32 slots; union of a 2-token ubatch is small.
    assert L.msb_slab_slots(128, 0.25, 4, 2) == 32
    assert L.msb_slab_slots(256, 0.25, 8, 2) == 64
    # frac too small for a ubatch union is raised; clamps to [8, n_expert].
    assert L.msb_slab_slots(128, 0.01, 4, 2) == 13
    assert L.msb_slab_slots(16, 0.01, 4, 1) == 8
    assert L.msb_slab_slots(128, 2.0, 4, 2) == 128
    assert L.msb_slab_slots(1, 0.5, 4, 2) == 0
    # Thresholds stated for the gpt-oss and 256-expert shapes: 6 tokens.
    assert L.msb_arena_threshold(128, 4, 32) == 6
    assert L.msb_arena_threshold(256, 8, 64) == 6


def test_errors_are_reported_not_raised():
    import ctypes as C
    from moestream_b200._lib import MsbError, c_vp, check, lib
    h = c_vp()
    rc = lib().msb_pool_create(5, 64, 4, 2, 1, C.byref(h))
    assert rc != 0
    assert b"IQ4_NL or MXFP4" in lib().msb_last_error()
    try:
        check(rc)
    except MsbError as e:
        assert "weight type" in str(e)
    else:
        raise AssertionError("check() did not raise")


def test_router_rejects_bad_shapes_before_any_device_work():
    """msb_router_topk validates its arguments before touching the device
    (these calls pass no device memory)."""
    from moestream_b200._lib import lib
    L = lib()
    for ne, k, mode in ((1024 + 1, 4, 0),   # n_expert above 1024
                        (128, 33, 0),       # top_k above 32
                        (16, 17, 0),        # top_k above n_expert
                        (128, 4, 2)):       # unknown mode
        assert L.msb_router_topk(None, 0, 512, 4, ne, k, mode, None, None, None) != 0
    assert L.msb_router_topk(None, 7, 512, 4, 128, 4, 0, None, None, None) != 0  # logit type
    assert L.msb_router_topk(None, 0, 512, 4, 128, 4, 0, None, None, None) != 0  # null pointers
    # An empty batch is a no-op.
    assert L.msb_router_topk(None, 0, 512, 0, 128, 4, 0, None, None, None) == 0

"""Host expert cache and slot streamer.

Part 1 mirrors the reference's unit tests (research/tests/
test_expert_cache.cpp:43-137) on this library's ExpertCache. Part 2 replays
seeded traces through this cache and through the reference's own
ExpertCache (compiled from its source into oracle/_ref) and requires
identical slots, hit/miss outcomes, statistics and quotas. Part 3 checks the
slot streamer (ms_remap_fn's host half) against the restated remap loop
over the reference cache.
"""
import numpy as np
import pytest

from moestream_b200 import NO_SLOT, ExpertCache, SlotStreamer
from oracle import oracle as O

needs_ref = pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built")


def touch(c, layer, e, origin=0):
    hit, slot = c.acquire(layer, e, origin)
    if not hit:
        c.mark_resident(layer, e, 1024)
    c.release(layer, e)
    return hit


# ---- part 1: the reference's invariants -----------------------------------
def test_cold_miss_then_hit():
    c = ExpertCache(n_layer=2, n_expert=32, n_slot=16)
    assert not touch(c, 0, 5)
    assert touch(c, 0, 5)
    assert not touch(c, 1, 5)  # another layer is another object


def test_residency_never_exceeds_slots():
    c = ExpertCache(n_layer=1, n_expert=256, n_slot=32)
    slots = set()
    for e in range(256):
        hit, s = c.acquire(0, e)
        if not hit:
            c.mark_resident(0, e, 1024)
        assert s < 32
        slots.add(s)
        c.release(0, e)
        c.end_step()
    assert len(slots) <= 32


def test_referenced_slot_is_never_evicted():
    c = ExpertCache(n_layer=1, n_expert=64, n_slot=8)
    _, held = c.acquire(0, 0)
    c.mark_resident(0, 0, 1024)
    for e in range(1, 64):
        hit, s = c.acquire(0, e)
        if not hit:
            c.mark_resident(0, e, 1024)
        assert s != held
        c.release(0, e)
        c.end_step()
    c.release(0, 0)


def test_eviction_survives_saturated_frequency():
    c = ExpertCache(n_layer=1, n_expert=128, n_slot=16)
    for _ in range(50):
        for e in range(16):
            touch(c, 0, e)
            c.end_step()
    for e in range(16, 128):
        hit, s = c.acquire(0, e)
        if not hit:
            c.mark_resident(0, e, 1024)
        assert s < 16
        c.release(0, e)
        c.end_step()


def test_sweep_is_not_admitted():
    c = ExpertCache(n_layer=1, n_expert=64, n_slot=8)
    for e in range(64):
        hit, s = c.acquire(0, e, 3)
        assert not hit and s == NO_SLOT
        c.release(0, e)
    assert c.stats()["bypass"] == 64


def test_stats_consistency():
    c = ExpertCache(n_layer=4, n_expert=64, n_slot=32)
    rng = np.random.default_rng(1234)
    n = 0
    for _ in range(5000):
        for layer in range(4):
            touch(c, layer, int(rng.integers(0, 64)))
            n += 1
        c.end_step()
    st = c.stats()
    assert st["hit"] + st["miss"] == n
    assert 0 < st["hit"] < n
    assert st["hit"] == st["hit_pinned"] + st["hit_small"] + st["hit_main"]


def test_exhaustion_returns_no_slot():
    c = ExpertCache(n_layer=1, n_expert=16, n_slot=4)
    for e in range(4):
        c.acquire(0, e)  # held, never released
    hit, s = c.acquire(0, 9)
    assert not hit and s == NO_SLOT


# ---- part 2: replay against the reference ExpertCache ---------------------
CONFIGS = [
    dict(n_layer=1, n_expert=128, n_slot=32, pin_ratio=0.0, layer_quota_adapt=False),
    dict(n_layer=1, n_expert=256, n_slot=64, pin_ratio=0.0, layer_quota_adapt=False),
    dict(n_layer=4, n_expert=64, n_slot=40, quota_period=64, quota_min=4),
    dict(n_layer=3, n_expert=50, n_slot=0, cache_frac=0.3, ghost_mult=1, quota_period=16,
         quota_eta=0.5, quota_min=2),
]


@needs_ref
@pytest.mark.parametrize("cfg", CONFIGS)
@pytest.mark.parametrize("seed", [0, 1])
def test_replay_matches_reference_cache(cfg, seed):
    mine = ExpertCache(**cfg)
    ref = O.RefCache(**cfg)
    rng = np.random.default_rng(seed)
    nl, ne = cfg["n_layer"], cfg["n_expert"]
    held = [[] for _ in range(nl)]
    zipf = 1.0 / np.arange(1, ne + 1) ** 1.1
    zipf /= zipf.sum()
    for step in range(3000):
        for layer in range(nl):
            for e in held[layer]:
                mine.release(layer, e)
                ref.release(layer, e)
            held[layer] = []
            k = int(rng.integers(1, 9))
            skew = step % 2 == 0
            es = rng.choice(ne, size=k, p=zipf) if skew else rng.integers(0, ne, size=k)
            for e in es.tolist():
                origin = int(rng.choice(4, p=[0.85, 0.05, 0.05, 0.05]))
                a = mine.acquire(layer, e, origin)
                b = ref.acquire(layer, e, origin)
                assert a == b, (step, layer, e, origin, a, b)
                if a[1] != NO_SLOT:
                    if not a[0]:
                        mine.mark_resident(layer, e, 1000 + e)
                        ref.mark_resident(layer, e, 1000 + e)
                    held[layer].append(e)
        mine.end_step()
        ref.end_step()
        if step % 97 == 0:
            for layer in range(nl):
                for e in range(ne):
                    assert mine.slot_of(layer, e) == ref.slot_of(layer, e)
    assert mine.stats() == ref.stats()
    assert np.array_equal(mine.layer_quota(), ref.layer_quota())


@needs_ref
def test_pinned_matches_reference_with_distinct_frequencies():
    cfg = dict(n_layer=2, n_expert=40, n_slot=12, pin_ratio=0.1, layer_quota_adapt=False)
    mine, ref = ExpertCache(**cfg), O.RefCache(**cfg)
    freq = np.random.default_rng(3).permutation(80).astype(np.uint32)
    mine.build_pinned(freq)
    ref.build_pinned(freq)
    rng = np.random.default_rng(4)
    for _ in range(500):
        layer, e = int(rng.integers(0, 2)), int(rng.integers(0, 40))
        a, b = mine.acquire(layer, e), ref.acquire(layer, e)
        assert a == b
        if a[1] != NO_SLOT:
            mine.release(layer, e)
            ref.release(layer, e)
    assert mine.stats() == ref.stats()


# ---- part 3: the slot streamer against the restated remap loop ------------
@needs_ref
@pytest.mark.parametrize("n_expert,n_slot,top_k,sizes", [
    (128, 32, 8, [1] * 40),                 # IQ4_NL decode shape
    (128, 32, 4, [1, 4, 16, 4, 1, 16, 2]),  # gpt-oss decode batches (16 exhausts)
    (256, 64, 8, [1, 8, 8, 1, 32]),         # 256-expert shape
])
def test_streamer_matches_reference_remap(n_expert, n_slot, top_k, sizes):
    n_layer = 3
    st = SlotStreamer(n_layer, n_expert, n_slot, expert_bytes_total=777)
    refs = [O.RefRemap(n_expert, n_slot, 777) for _ in range(n_layer)]
    rng = np.random.default_rng(11)
    for rep in range(6):
        for n_tok in sizes:
            for layer in range(n_layer):
                ids = np.stack([rng.permutation(n_expert)[:top_k] for _ in range(n_tok)])
                ids = ids.astype(np.int32)
                if rep % 3 == 2:  # invalid ids map to the zero slot
                    ids[0, 0] = -1
                    ids[-1, -1] = n_expert + 5
                if rep % 2 == 1:  # a strided view, as the reference's ids may be
                    big = np.zeros((n_tok, top_k * 2), dtype=np.int32)
                    big[:, ::2] = ids
                    ids = big[:, ::2]
                got, misses, table = st.remap(layer, ids, want_table=True)
                want, pend = refs[layer](ids)
                assert np.array_equal(got, want)
                assert misses == pend
                # The table reproduces every pair's slot (zero slot otherwise).
                assert np.array_equal(O.remap_table(ids, table, n_slot), want)
    s = st.stats()
    ref_tot = {}
    for r in refs:
        for k, v in r.stats().items():
            ref_tot[k] = ref_tot.get(k, 0) + v
    assert s == ref_tot

"""GGUF expert source (msb_gguf_*) on CPU.

Files are written by the gguf package's writer and read back both by its
reader (GGUFReader) and by the library's own parser: tensor tables, data
offsets, metadata integers and expert bytes must agree exactly. Covers the
reference's behaviour on this path: split files opened from any shard's
name ("<base>-NNNNN-of-MMMMM.gguf", src/llama-moestream.cpp:571-598), a
missing shard refused (:1455-1466), tensors past the end of their file
refused (:1478-1506), integer metadata by key suffix (:610-693), the byte
cost of one slot across layers (:771-830) and parallel expert reads
(:1230-1263).
"""
import os
import shutil

import numpy as np
import pytest
from gguf import GGML_QUANT_SIZES, GGMLQuantizationType as T, GGUFReader

from tests.helpers import experts, write_gguf

E, N_FF, K = 6, 64, 128


def _model_tensors(n_layer=2, wtype=T.MXFP4, seed=0):
    name = {T.MXFP4: "mxfp4", T.IQ4_NL: "iq4_nl"}[wtype]
    out = []
    for il in range(n_layer):
        for r, (kk, nn) in (("gate", (K, N_FF)), ("up", (K, N_FF)), ("down", (N_FF, K))):
            ex = experts(name, E, kk, nn, seed=seed + 10 * il + len(r))
            out.append((f"blk.{il}.ffn_{r}_exps.weight", ex.reshape(E, nn, -1), wtype))
        out.append((f"blk.{il}.attn_norm.weight",
                    np.random.default_rng(il).normal(size=K).astype(np.float32), None))
    return out


KVS = [("add_block_count", 2), ("add_expert_count", E), ("add_expert_used_count", 4),
       ("add_context_length", 4096), ("add_string", "tokenizer.ggml.model", "gpt2"),
       ("add_array", "tokenizer.ggml.tokens", [f"tok{i}" for i in range(300)]),
       ("add_array", "tokenizer.ggml.scores", [float(i) for i in range(300)]),
       ("add_float32", "gpt-oss.rope.freq_base", 150000.0), ("add_bool", "x.flag", True)]


def _reader_table(paths):
    """(name, type, ne, shard, absolute offset, nbytes) from GGUFReader."""
    rows = []
    for s, p in enumerate(paths):
        r = GGUFReader(p)
        for t in r.tensors:
            rows.append((t.name, int(t.tensor_type), tuple(int(x) for x in t.shape), s,
                         int(t.data_offset), int(t.n_bytes)))
    return rows


def _lib_table(g):
    return [(t["name"], t["type"], t["ne"], t["shard"], t["offset"], t["nbytes"])
            for t in g.tensors]


@pytest.mark.parametrize("alignment", [None, 64, 4096])
def test_table_and_metadata_match_gguf_reader(tmp_path, alignment):
    from moestream_b200.gguf import GGUFFile
    tensors = _model_tensors()
    paths = write_gguf(tmp_path / "m.gguf", tensors, KVS, alignment=alignment)
    with GGUFFile(paths[0]) as g:
        assert g.n_shard == 1
        assert _lib_table(g) == _reader_table(paths)
        assert g.kv_int(".block_count") == 2
        assert g.kv_int(".expert_count") == E
        assert g.kv_int(".expert_used_count") == 4
        assert g.kv_int(".context_length") == 4096
        assert g.kv_int(".rope.freq_base") is None          # a float is not an integer
        assert g.kv_int(".no_such_key") is None
        if alignment:
            assert g.kv_int("general.alignment") == alignment
            assert all(t["offset"] % alignment == 0 for t in g.tensors)
        # One slot = one expert of every role in every layer.
        per = sum(ex.nbytes // E for n, ex, raw in tensors if raw is not None)
        assert g.bytes_per_slot() == per


@pytest.mark.parametrize("wtype", [T.MXFP4, T.IQ4_NL])
@pytest.mark.parametrize("n_threads", [1, 3, 16])
def test_read_experts_returns_the_written_bytes(tmp_path, wtype, n_threads):
    from moestream_b200.gguf import GGUFFile
    tensors = _model_tensors(wtype=wtype, seed=5)
    paths = write_gguf(tmp_path / "m.gguf", tensors, KVS)
    want = {n: a for n, a, _ in tensors}
    order = [5, 0, 3, 3, 1, 4, 2]                            # any order, repeats allowed
    with GGUFFile(paths[0]) as g:
        for il in range(2):
            for role in ("gate", "up", "down"):
                ti = g.expert_tensor(il, role)
                name = f"blk.{il}.ffn_{role}_exps.weight"
                assert ti == g.index(name) >= 0
                assert g.expert_bytes(ti) == want[name][0].nbytes
                got = g.read_experts(ti, order, n_threads=n_threads)
                for row, e in zip(got, order):
                    assert np.array_equal(row, want[name][e].reshape(-1)), (name, e)
        assert g.expert_tensor(2, "gate") == -1
        assert g.expert_tensor(0, 3) == -1                    # no such role
        assert g.read_experts(g.expert_tensor(0, "up"), []).shape == (0, g.expert_bytes(1))


def test_read_rejects_expert_out_of_range(tmp_path):
    from moestream_b200 import MsbError
    from moestream_b200.gguf import GGUFFile
    paths = write_gguf(tmp_path / "m.gguf", _model_tensors(), KVS)
    with GGUFFile(paths[0]) as g:
        ti = g.expert_tensor(1, "down")
        for bad in (-1, E):
            with pytest.raises(MsbError, match="expert"):
                g.read_experts(ti, [0, bad])


def test_every_known_type_size_matches_the_format(tmp_path):
    """Tensor byte sizes for every ggml type the parser knows equal the gguf
    package's (two rows of two blocks each)."""
    from moestream_b200.gguf import GGUFFile
    tensors = []
    for qt, (blck, size) in GGML_QUANT_SIZES.items():
        if int(qt) in (40, 41):                              # not in the parser's table
            continue
        a = np.arange(2 * 2 * size, dtype=np.uint8).reshape(2, 2 * size)
        tensors.append((f"t{int(qt)}", a, qt))
    paths = write_gguf(tmp_path / "types.gguf", tensors)
    with GGUFFile(paths[0]) as g:
        assert _lib_table(g) == _reader_table(paths)
        assert len(g.tensors) == len(tensors)


def test_split_file_opens_from_any_shard(tmp_path):
    from moestream_b200.gguf import GGUFFile
    tensors = _model_tensors(seed=9)
    paths = write_gguf(tmp_path / "m.gguf", tensors, KVS, split_max_tensors=3)
    assert len(paths) == 3 and paths[0].endswith("m-00001-of-00003.gguf")
    want = {n: a for n, a, _ in tensors}
    for start in (paths[0], paths[2]):
        with GGUFFile(start) as g:
            assert g.n_shard == 3
            assert _lib_table(g) == _reader_table(paths)
            assert sorted({t["shard"] for t in g.tensors}) == [0, 1, 2]
            assert g.kv_int(".expert_count") == E            # metadata lives in shard 1
            assert g.kv_int("split.count") == 3
            for il in range(2):
                ti = g.expert_tensor(il, "down")
                got = g.read_experts(ti, [4, 1], n_threads=2)
                assert np.array_equal(got[0], want[f"blk.{il}.ffn_down_exps.weight"][4].ravel())
                assert np.array_equal(got[1], want[f"blk.{il}.ffn_down_exps.weight"][1].ravel())


def test_split_file_with_a_missing_shard_is_refused(tmp_path):
    from moestream_b200 import MsbError
    from moestream_b200.gguf import GGUFFile
    paths = write_gguf(tmp_path / "m.gguf", _model_tensors(), KVS, split_max_tensors=3)
    os.remove(paths[1])
    with pytest.raises(MsbError, match="every shard"):
        GGUFFile(paths[0])


def test_first_shard_under_another_name_is_refused(tmp_path):
    from moestream_b200 import MsbError
    from moestream_b200.gguf import GGUFFile
    paths = write_gguf(tmp_path / "m.gguf", _model_tensors(), KVS, split_max_tensors=3)
    alone = str(tmp_path / "alone.gguf")
    shutil.copy(paths[0], alone)
    with pytest.raises(MsbError, match="shard 1 of 3"):
        GGUFFile(alone)


def test_names_outside_the_split_pattern_are_single_files(tmp_path):
    """NNNNN > MMMMM or MMMMM >= 1000 is not a split name (the reference's
    rule); such a path opens as one file."""
    from moestream_b200.gguf import GGUFFile
    src = write_gguf(tmp_path / "m.gguf", _model_tensors(n_layer=1), KVS)[0]
    for name in ("x-00002-of-00001.gguf", "x-00001-of-01000.gguf", "x-00001-of-00002.bin"):
        p = str(tmp_path / name)
        shutil.copy(src, p)
        with GGUFFile(p) as g:
            assert g.n_shard == 1 and g.expert_tensor(0, "gate") >= 0


def _corrupt(tmp_path, fn):
    src = write_gguf(tmp_path / "m.gguf", _model_tensors(n_layer=1), KVS)[0]
    data = bytearray(open(src, "rb").read())
    data = fn(data)
    p = str(tmp_path / "bad.gguf")
    with open(p, "wb") as f:
        f.write(bytes(data))
    return p, src


@pytest.mark.parametrize("what,fn,match", [
    ("magic", lambda d: b"GGUX" + d[4:], "bad magic"),
    ("version 1", lambda d: d[:4] + (1).to_bytes(4, "little") + d[8:], "version 1"),
    ("big-endian", lambda d: d[:4] + (3).to_bytes(4, "big") + d[8:], "version"),
    ("cut data", lambda d: d[:len(d) - 100], "past the end"),
    ("cut header", lambda d: d[:200], "truncated|bad value"),
    ("empty", lambda d: d[:0], "magic"),
    ("tensor count", lambda d: d[:8] + (1 << 60).to_bytes(8, "little") + d[16:],
     "implausible"),
])
def test_malformed_files_are_refused(tmp_path, what, fn, match):
    from moestream_b200 import MsbError
    from moestream_b200.gguf import GGUFFile
    p, _ = _corrupt(tmp_path, fn)
    with pytest.raises(MsbError, match=match):
        GGUFFile(p)


def test_unknown_tensor_type_is_refused(tmp_path):
    from moestream_b200 import MsbError
    from moestream_b200.gguf import GGUFFile
    r = GGUFReader(write_gguf(tmp_path / "m.gguf", _model_tensors(n_layer=1), KVS)[0])
    # The type field of the first tensor record: the part before its offset.
    field = r.tensors[0].field
    type_off = int(field.offset) + sum(int(p.nbytes) for p in field.parts[:-2])

    def set_type(d):
        d[type_off:type_off + 4] = (33).to_bytes(4, "little")   # an id with no type
        return d
    p, _ = _corrupt(tmp_path, set_type)
    with pytest.raises(MsbError, match="unknown type 33"):
        GGUFFile(p)


def test_missing_file(tmp_path):
    from moestream_b200 import MsbError
    from moestream_b200.gguf import GGUFFile
    with pytest.raises(MsbError, match="cannot open"):
        GGUFFile(tmp_path / "nope.gguf")


def test_arena_bookkeeping_restatement():
    """The oracle's restatement of the reference's arena reads on a small
    schedule worked out by hand."""
    from oracle.oracle import ArenaPlan
    p = ArenaPlan(n_expert=4, n_buf=2)
    assert p.load(0, [1, 2]) == [1, 2]
    assert p.load(1) == [0, 1, 2, 3]                # no hint: every expert
    assert p.load(0, [2, 3]) == [3]                 # 2 is held already
    assert p.load(0, [1]) == [] and p.hits == 1
    assert p.load(2, [0]) == [0]                    # arena 0 switches layers: forgets
    assert p.load(0, [1]) == [1]
    assert (p.loads, p.read, p.asked) == (5, 9, 24)


def test_arena_refuses_files_without_experts(tmp_path):
    from moestream_b200 import MsbError
    from moestream_b200._lib import lib
    import ctypes
    path = write_gguf(tmp_path / "dense.gguf",
                      [("blk.0.ffn_up.weight", np.zeros((4, 32), np.float32), None)])[0]
    h = ctypes.c_void_p()
    assert lib().msb_arena_create(path.encode(), 2, 1, ctypes.byref(h)) != 0
    assert b"no expert tensors" in lib().msb_last_error()
    assert lib().msb_arena_create(str(tmp_path / "none.gguf").encode(), 2, 1,
                                  ctypes.byref(h)) != 0
    with pytest.raises(MsbError):
        from moestream_b200.gguf import ExpertArena
        ExpertArena(tmp_path / "none.gguf")

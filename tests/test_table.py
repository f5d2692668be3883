"""The drop-in host table (hl::alloc) against the reference.

* tests/cpp/test_host.cpp restates the reference's ABI, IdArena and
  HeteroBlockTable unit tests against this library's C++ API (linked to
  libhlkv.so);
* oracle/table_trace.cpp replays a seeded random walk over the whole table
  API; its word stream from this library must equal the reference's --
  compared live where the reference tree exists, and against the recorded
  hashes in tests/golden/table_traces.json everywhere;
* the C ABI view of the table (include/hlkv.h) against the same behaviour.
"""
import hashlib
import json
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BUILD = os.path.join(ROOT, "tests", "_build")
TRACES = os.path.join(ROOT, "tests", "golden", "table_traces.json")


def _compile(out: str, sources: list[str], shared: bool, hlkv_lib) -> str:
    os.makedirs(BUILD, exist_ok=True)
    deps = sources + [os.path.join(ROOT, "include", "hl_allocator", f) for f in
                      ("hetero_block_table.hpp", "id_arena.hpp", "block_descriptor.hpp", "status.hpp")]
    deps.append(hlkv_lib.LIB_PATH)
    if not os.path.exists(out) or os.path.getmtime(out) < max(os.path.getmtime(d) for d in deps):
        libdir = os.path.dirname(hlkv_lib.LIB_PATH)
        cmd = ["g++", "-std=c++20", "-O1", "-Wall", "-Wextra", "-Werror", "-I",
               os.path.join(ROOT, "include"), *sources, "-o", out + ".tmp",
               "-L", libdir, "-l:libhlkv.so", f"-Wl,-rpath,{libdir}"]
        if shared:
            cmd[1:1] = ["-shared", "-fPIC"]
        subprocess.run(cmd, check=True)
        os.replace(out + ".tmp", out)
    return out


@pytest.fixture(scope="module")
def host_tests(hlkv_lib):
    return _compile(os.path.join(BUILD, "test_host"), [os.path.join(ROOT, "tests", "cpp", "test_host.cpp")],
                    False, hlkv_lib)


@pytest.fixture(scope="module")
def trace_lib(hlkv_lib):
    import ctypes
    path = _compile(os.path.join(BUILD, "libtrace_hlkv.so"), [os.path.join(ROOT, "oracle", "table_trace.cpp")],
                    True, hlkv_lib)
    return ctypes.CDLL(path)


def test_restated_reference_unit_tests(host_tests):
    r = subprocess.run([host_tests], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
    assert "0 failures" in r.stdout


CASES = [(20261011, 20000, 96, (48, 48, 64)), (1, 5000, 8, (4, 4, 4)),
         (7, 30000, 300, (100, 200, 50)), (99, 3000, 2000, (3000, 3000, 3000))]


@pytest.mark.parametrize("seed,steps,max_blocks,slots", CASES)
def test_trace_matches_recorded_reference(trace_lib, seed, steps, max_blocks, slots):
    from oracle.oracle import table_trace
    t = table_trace(trace_lib, seed, steps, max_blocks, slots)
    rec = json.load(open(TRACES))[f"{seed}:{steps}:{max_blocks}:{','.join(map(str, slots))}"]
    assert t.size == rec["words"]
    assert hashlib.sha256(t.tobytes()).hexdigest() == rec["sha256"]


@pytest.mark.parametrize("seed", [3, 11, 2026])
def test_trace_matches_live_reference(trace_lib, ref, seed):
    from oracle.oracle import table_trace
    for max_blocks, slots in ((64, (20, 30, 40)), (16, (4, 8, 2))):
        a = table_trace(ref.lib, seed, 8000, max_blocks, slots)
        b = table_trace(trace_lib, seed, 8000, max_blocks, slots)
        if not np.array_equal(a, b):
            n = min(a.size, b.size)
            bad = np.nonzero(a[:n] != b[:n])[0]
            pytest.fail(f"trace differs at word {bad[0] if bad.size else n}")


def test_c_abi_table_matches_reference_behaviour(hlkv_lib):
    h = hlkv_lib
    t = h.Table(8, [(0, 4096, 4), (1, 2048, 4), (3, 1088, 4)])
    assert h.Table.validate_config(0, [(0, 4096, 4)]) == h.Status.INVALID_ARGUMENT
    assert h.Table.validate_config(8, [(15, 16, 1)]) == h.Status.UNKNOWN_FORMAT
    with pytest.raises(ValueError):
        h.Table(8, [])
    d = t.collect_delta()
    assert d.descriptor_table_size == 8 and d.descriptor_patches.shape == (8, 4)
    assert np.all(d.descriptor_patches[:, 0] == 0xFFFFFFFF) and np.all(d.descriptor_patches[:, 1] == 15)
    st, s = t.create_sequence()
    blocks = [t.append_block(s, f, 16)[1] for f in (0, 1, 3)]
    assert [b.id for b in blocks] == [0, 1, 2]
    st, rec = t.lookup(blocks[1])
    words = np.frombuffer(rec, dtype=np.uint32)
    assert st == 0 and words[0] == 0 and words[1] == h.pack_info(1, 0, 1, 16) and words[3] == 1
    assert t.seal(blocks[0]) == 0
    st, fc = t.begin_format_change(blocks[0], 3)
    assert st == 0 and fc == (0, 0, 3, 1)
    assert t.release_sequence(s) == h.Status.INVALID_STATE
    assert t.commit_format_change(blocks[0], 0, 0) == 0
    st, indptr, ex = t.build_exec_table([s])
    assert st == 0 and list(indptr) == [0, 3] and ex[0][1] & 0xF == 3
    d = t.collect_delta()
    assert d.id_patches.shape == (3, 2) and d.arena_size == 8
    assert t.release_sequence(s) == 0 and t.blocks_in_use() == 0
    assert t.validate() == (0, "")
    stats = t.stats()
    assert stats["format_changes_committed"] == 1 and stats["arena_free_entries"] == 8
    assert t.device_descriptor(100) == (0xFFFFFFFF, 15, 0, 100)


def test_append_tokens_decode_driver(hlkv_lib):
    """hlkv_table_append_tokens = per sequence: set_valid_tokens(tail, vt + 1) while the tail
    has room, else append_block(new format, 1 valid token); the same table state and the
    same delta as those calls made one by one on a second table."""
    h = hlkv_lib
    T = 4
    pools = [(1, 2048, 64), (3, 1088, 64)]
    a, b = h.Table(128, pools, block_tokens=T), h.Table(128, pools, block_tokens=T)
    seqs_a = [a.create_sequence()[1] for _ in range(3)]
    seqs_b = [b.create_sequence()[1] for _ in range(3)]
    for t, ss in ((a, seqs_a), (b, seqs_b)):       # sequence 0 starts with a partial tail
        t.append_block(ss[0], 1, 2)
    a.collect_delta()
    b.collect_delta()
    rng = np.random.default_rng(3)
    for step in range(11):
        fm = rng.choice([1, 3], size=3).astype(np.uint32)
        st, targets, done = a.append_tokens(seqs_a, fm, 1)
        assert st == 0 and done == 3
        for i, s in enumerate(seqs_b):               # the same step, one call at a time
            st_i, ids = b.sequence_block_ids(s)
            vt = None
            if ids:
                tail = b.handle_of(ids[-1])
                vt = (int(np.frombuffer(b.lookup(tail)[1], np.uint32)[1]) >> 10) & 0x3FF
            if vt is not None and vt < T:
                assert b.set_valid_tokens(tail, vt + 1) == 0
                want = (ids[-1], vt)
            else:
                st_b, nb = b.append_block(s, int(fm[i]), 1, 1)
                assert st_b == 0
                want = (nb.id, 0)
            assert tuple(targets[i]) == want, (step, i)
        da, db = a.collect_delta(), b.collect_delta()
        assert np.array_equal(da.descriptor_patches, db.descriptor_patches)
        assert np.array_equal(da.id_patches, db.id_patches)
    for sa, sb in zip(seqs_a, seqs_b):
        assert a.sequence_block_ids(sa) == b.sequence_block_ids(sb)
    # errors: a stale sequence handle stops the batch at that sequence
    assert a.release_sequence(seqs_a[1]) == 0
    st, targets, done = a.append_tokens(seqs_a, np.ones(3, np.uint32), 1)
    assert st == h.Status.STALE_HANDLE and done == 1

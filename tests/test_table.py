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


def _random_ops(t, rng, steps, seqs, transcoding, formats=(0, 1, 3)):
    """A reproducible random workload over the public table API (the mix of the reference's
    randomized test, test_hetero_block_table.cpp:675-784); returns what each step returned."""
    log = []

    def random_block():
        if not seqs:
            return None
        st, ids = t.sequence_block_ids(seqs[int(rng.integers(len(seqs)))])
        return t.handle_of(ids[int(rng.integers(len(ids)))]) if ids else None

    for _ in range(steps):
        op = int(rng.integers(12))
        if op == 0:
            st, s = t.create_sequence()
            log.append((op, st, (s.id, s.generation)))
            if st == 0:
                seqs.append(s)
        elif op in (1, 2) and seqs:
            st, b = t.append_block(seqs[int(rng.integers(len(seqs)))], formats[int(rng.integers(3))],
                                   int(rng.integers(0, 17)))
            log.append((op, st, (b.id, b.generation)))
        elif op == 3 and (b := random_block()) is not None:
            log.append((op, t.seal(b), t.append_shared_block(seqs[int(rng.integers(len(seqs)))], b)))
        elif op == 4 and (b := random_block()) is not None:
            t.seal(b)
            st, fc = t.begin_format_change(b, formats[int(rng.integers(3))])
            log.append((op, st, tuple(fc) if st == 0 else None))
            if st == 0:
                transcoding.append(b)
        elif op == 5 and transcoding:
            b = transcoding.pop(int(rng.integers(len(transcoding))))
            log.append((op, t.commit_format_change(b, 1, 0x3F800000) if rng.integers(2) else t.abort_format_change(b)))
        elif op == 6 and (b := random_block()) is not None:
            log.append((op, t.set_residency(b, int(rng.integers(3)))))
        elif op == 7 and (b := random_block()) is not None:
            log.append((op, t.set_valid_tokens(b, int(rng.integers(17)))))
        elif op == 8 and (b := random_block()) is not None:
            log.append((op, t.set_scale(b, int(rng.integers(3)), int(rng.integers(1 << 32)))))
        elif op >= 9 and seqs:
            i = int(rng.integers(len(seqs)))
            st = t.release_sequence(seqs[i])
            log.append((op, st))
            if st == 0:
                seqs.pop(i)
    return log


def _mirror_apply(mirror_table, mirror_arena, d):
    """The reference's ExecMirror::apply (tests/project1/exec_mirror.hpp:23-49) on arrays."""
    if d.arena_size > mirror_arena.size:
        grown = np.zeros(d.arena_size, np.uint32)
        grown[:mirror_arena.size] = mirror_arena
        mirror_arena = grown
    for p in d.descriptor_patches:
        mirror_table[p[3]] = p
    for off, bid in d.id_patches:
        mirror_arena[off] = bid
    return mirror_table, mirror_arena


def test_snapshot_restore_round_trip(hlkv_lib):
    """A restored table re-snapshots to the same bytes, its first delta rebuilds the same
    device mirror the original's deltas built, and from then on both tables answer the same
    random operations with the same statuses, handles and deltas."""
    h = hlkv_lib
    pools = [(0, 4096, 40), (1, 2048, 40), (3, 1088, 60)]
    a = h.Table(120, pools, block_tokens=16)
    rng = np.random.default_rng(77)
    seqs, transcoding = [], []
    mt = np.zeros((120, 4), np.uint32)
    ma = np.zeros(0, np.uint32)
    for _ in range(6):
        _random_ops(a, rng, 400, seqs, transcoding)
        mt, ma = _mirror_apply(mt, ma, a.collect_delta())
    image = a.snapshot()
    st, b = h.Table.restore(image)
    assert st == 0 and b is not None
    assert b.snapshot() == image
    # the restored table's first delta is the whole device image
    db = b.collect_delta()
    assert db.descriptor_patches.shape[0] == 120 and db.id_patches.shape[0] == db.arena_size
    mt_b, ma_b = _mirror_apply(np.zeros((120, 4), np.uint32), np.zeros(0, np.uint32), db)
    assert np.array_equal(mt_b, mt)
    for s in seqs:
        st, ids = a.sequence_block_ids(s)
        assert b.sequence_block_ids(s) == (st, ids)
    st, seg_a = a.batch_segments(seqs)
    st_b, seg_b = b.batch_segments(seqs)
    assert st == st_b == 0 and np.array_equal(seg_a, seg_b)
    for off, ln in seg_a:
        assert np.array_equal(ma_b[off:off + ln], ma[off:off + ln])
    # the same operations from here on: same answers, same deltas
    seqs_b, tr_b = list(seqs), list(transcoding)
    for k in range(4):
        la = _random_ops(a, np.random.default_rng(1000 + k), 300, seqs, transcoding)
        lb = _random_ops(b, np.random.default_rng(1000 + k), 300, seqs_b, tr_b)
        assert la == lb, k
        da, dbk = a.collect_delta(), b.collect_delta()
        assert np.array_equal(da.descriptor_patches, dbk.descriptor_patches), k
        assert np.array_equal(da.id_patches, dbk.id_patches), k
        assert (da.descriptor_table_size, da.arena_size) == (dbk.descriptor_table_size, dbk.arena_size)
    assert b.validate()[0] == 0


def test_snapshot_rejects_damaged_images(hlkv_lib):
    import ctypes as C
    h = hlkv_lib
    t = h.Table(16, [(1, 2048, 8), (3, 1088, 8)], block_tokens=4)
    st, s = t.create_sequence()
    for f in (1, 3, 1):
        assert t.append_block(s, f, 2)[0] == 0
    image = t.snapshot()
    corrupt = 10  # HLKV_STATUS_CORRUPT
    for bad in (b"", image[:-1], image[:40], image + b"\0",
                image[:100] + bytes([image[100] ^ 1]) + image[101:]):
        assert h.Table.restore(bad)[0] == corrupt
    # a foreign version with a valid checksum is still rejected
    body = bytearray(image[:-8])
    body[8] = 0xEE  # an image version this library does not know
    fnv = 0xCBF29CE484222325
    for byte in body:
        fnv = ((fnv ^ byte) * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    assert h.Table.restore(bytes(body) + fnv.to_bytes(8, "little"))[0] == corrupt
    # snapshot into a buffer that is too small: nothing written
    n = C.c_size_t()
    small = (C.c_char * 8)()
    assert h.lib().hlkv_table_snapshot(t.h, small, 8, C.byref(n)) == 6  # INVALID_ARGUMENT
    assert n.value == len(image) and bytes(small) == b"\0" * 8


def _apply_delta_model(dev: "np.ndarray", delta) -> "np.ndarray":
    """A device arena model: grow to the delta's arena size, then scatter its id patches."""
    if delta.arena_size > dev.size:
        dev = np.concatenate([dev, np.full(delta.arena_size - dev.size, 0xDEADBEEF, np.uint32)])
    for off, bid in delta.id_patches:
        dev[off] = bid
    return dev


def _apply_moves_model(dev: "np.ndarray", moves) -> "np.ndarray":
    """The two phases of hlkv_arena_relocate: every moved segment to scratch, then to its
    new offset (lengths rounded up to 4 entries, as the kernel copies them)."""
    dev = dev.copy()
    if len(moves) == 0:
        return dev
    n_scratch = int(moves[-1, 3]) + ((int(moves[-1, 2]) + 7) & ~7)
    scratch = np.zeros(n_scratch, np.uint32)
    for frm, to, ln, sc in moves:
        l4 = (int(ln) + 3) & ~3
        scratch[sc:sc + l4] = dev[frm:frm + l4]
    for frm, to, ln, sc in moves:
        l4 = (int(ln) + 3) & ~3
        dev[to:to + l4] = scratch[sc:sc + l4]
    return dev


def test_arena_compaction_keeps_sequences_and_packs_the_arena(hlkv_lib):
    """compact_arena over a random walk: every live sequence keeps its blocks, the arena
    shrinks to the live segments' capacity with no free storage, and a device arena model
    kept by the deltas plus the returned moves (made as the relocation kernels make them)
    equals the host's segments after every step."""
    h = hlkv_lib
    rng = np.random.default_rng(17)
    t = h.Table(4000, [(1, 2048, 2000), (3, 1088, 2000)], block_tokens=4)
    dev = np.zeros(0, np.uint32)
    seqs = []
    compactions = 0
    for step in range(1500):
        r = rng.random()
        if r < 0.08 or not seqs:
            st, s = t.create_sequence()
            assert st == 0
            seqs.append(s)
        elif r < 0.75:
            s = seqs[rng.integers(len(seqs))]
            for _ in range(int(rng.integers(1, 40 if rng.random() < 0.1 else 4))):
                st, _ = t.append_block(s, int(rng.choice([1, 3])), 2)
                if st != 0:
                    break
        elif r < 0.85:
            s = seqs.pop(int(rng.integers(len(seqs))))
            assert t.release_sequence(s) == 0
        else:
            dev = _apply_delta_model(dev, t.collect_delta())
            before = {(s.id, s.generation): list(t.sequence_block_ids(s)[1]) for s in seqs}
            stats0 = t.stats()
            st, moves = t.compact_arena()
            assert st == 0
            compactions += 1
            dev = _apply_moves_model(dev, moves)
            stats = t.stats()
            assert stats["arena_free_entries"] == 0
            assert stats["arena_entries"] == stats["arena_reserved_entries"] <= stats0["arena_entries"]
            assert stats["pending_id_patches"] == 0  # the moves replace patches
            assert t.validate()[0] == 0
            st, segs = t.batch_segments(seqs)
            assert st == 0
            offs = sorted(int(o) for o, n in segs if n)
            assert all(moves[k, 0] > moves[k, 1] for k in range(len(moves)))
            for s, (off, n) in zip(seqs, segs):
                ids = list(t.sequence_block_ids(s)[1])
                assert ids == before[(s.id, s.generation)]
                assert list(dev[off:off + n]) == ids, (step, s)
            dev = dev[:stats["arena_entries"]]
    dev = _apply_delta_model(dev, t.collect_delta())
    st, segs = t.batch_segments(seqs)
    for s, (off, n) in zip(seqs, segs):
        assert list(dev[off:off + n]) == list(t.sequence_block_ids(s)[1])
    assert compactions > 50


def test_arena_compaction_refusals_change_nothing(hlkv_lib):
    import ctypes as C
    h = hlkv_lib
    t = h.Table(64, [(1, 2048, 64)], block_tokens=4)
    seqs = [t.create_sequence()[1] for _ in range(3)]
    for s in seqs:
        for _ in range(9):
            assert t.append_block(s, 1, 1)[0] == 0
    image = t.snapshot()
    st, _ = t.compact_arena()  # id patches pending: collect first
    assert st == h.Status.INVALID_STATE
    t.collect_delta()
    image = t.snapshot()
    n = C.c_size_t()
    moves = (C.c_uint32 * 8)()
    assert h.lib().hlkv_table_compact_arena(t.h, moves, 2, C.byref(n)) == h.Status.INVALID_ARGUMENT  # 3 live
    assert t.snapshot() == image
    assert t.compact_arena()[0] == 0

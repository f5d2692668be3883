"""Kernel (3), hlkv_apply_delta, and hl::kv::DeviceTables: the device tables track the host
table through the delta protocol (the reference's ExecMirror, run on the GPU)."""
import numpy as np
import pytest

from helpers import d2h

pytestmark = pytest.mark.gpu


def _device_state(dt):
    table = d2h(dt.table_ptr, dt.table_size * 16).view(np.uint32).reshape(-1, 4)
    arena = d2h(dt.arena_ptr, dt.arena_size * 4).view(np.uint32)
    return table, arena


def test_random_operations_device_tables_track_host(hlkv_lib, cuda_device):
    """The reference's randomized differential test (test_hetero_block_table.cpp:675-784) with the
    mirror on the GPU: irregular syncs, arena relocations, residency changes, format changes."""
    h = hlkv_lib
    t = h.Table(96, [(0, 4096, 48), (1, 2048, 48), (3, 1088, 64)])
    dt = h.DeviceTables()
    rng = np.random.default_rng(20261011)
    seqs, transcoding = [], []
    formats = (0, 1, 3)

    def random_block():
        if not seqs:
            return None
        st, ids = t.sequence_block_ids(seqs[rng.integers(len(seqs))])
        return t.handle_of(ids[rng.integers(len(ids))]) if ids else None

    checks = 0
    for step in range(6000):
        op = int(rng.integers(11))
        if op == 0:
            st, s = t.create_sequence()
            if st == 0:
                seqs.append(s)
        elif op in (1, 2) and seqs:
            t.append_block(seqs[rng.integers(len(seqs))], formats[rng.integers(3)], 16)
        elif op == 3 and (b := random_block()) is not None:
            t.seal(b)
            t.append_shared_block(seqs[rng.integers(len(seqs))], b)
        elif op == 4 and (b := random_block()) is not None:
            t.seal(b)
            if t.begin_format_change(b, formats[rng.integers(3)])[0] == 0:
                transcoding.append(b)
        elif op == 5 and transcoding:
            b = transcoding.pop(int(rng.integers(len(transcoding))))
            assert (t.commit_format_change(b) if rng.integers(2) else t.abort_format_change(b)) == 0
        elif op == 6 and (b := random_block()) is not None:
            t.set_residency(b, int(rng.integers(3)))
        elif op == 7 and (b := random_block()) is not None:
            t.set_valid_tokens(b, int(rng.integers(17)))
        elif op >= 8 and seqs:
            i = int(rng.integers(len(seqs)))
            if t.release_sequence(seqs[i]) == 0:
                seqs.pop(i)
        if rng.integers(23) == 0:
            dt.sync(t)
            table, arena = _device_state(dt)
            want = np.array([t.device_descriptor(i) for i in range(96)], np.uint32)
            assert np.array_equal(table, want), f"step {step}"
            st, segs = t.batch_segments(seqs)
            for s, (off, ln) in zip(seqs, segs):
                assert list(arena[off:off + ln]) == t.sequence_block_ids(s)[1], f"step {step}"
            checks += 1
    assert checks > 100
    assert d2h(dt.error_word_ptr, 4).view(np.uint32)[0] == 0


def test_apply_delta_kernel_matches_oracle_and_flags_range(hlkv_lib, oracle, cuda_device):
    import torch
    rng = np.random.default_rng(4)
    n_table, n_arena = 300, 1000
    table0 = rng.integers(0, 2 ** 32, size=(n_table, 4), dtype=np.uint64).astype(np.uint32)
    arena0 = rng.integers(0, 2 ** 32, size=n_arena, dtype=np.uint64).astype(np.uint32)
    ids = rng.permutation(n_table + 20)[:150].astype(np.uint32)          # some out of range
    desc = rng.integers(0, 2 ** 32, size=(150, 4), dtype=np.uint64).astype(np.uint32)
    desc[:, 3] = ids
    offs = rng.permutation(n_arena + 50)[:700].astype(np.uint32)         # some out of range
    idp = np.stack([offs, rng.integers(0, 2 ** 32, size=700, dtype=np.uint64).astype(np.uint32)], 1)
    t_host, a_host = table0.copy(), arena0.copy()
    oerr = oracle.apply_delta(t_host, a_host, desc, idp)
    d_table = torch.from_numpy(table0.view(np.int32)).cuda()
    d_arena = torch.from_numpy(arena0.view(np.int32)).cuda()
    d_desc = torch.from_numpy(desc.view(np.int32)).cuda()
    d_ids = torch.from_numpy(idp.view(np.int32)).cuda()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    hlkv_lib.apply_delta(d_table.data_ptr(), n_table, d_arena.data_ptr(), n_arena, d_desc, d_ids, err)
    torch.cuda.synchronize()
    assert oerr == (1 << 11) == int(err.item())
    assert np.array_equal(d_table.cpu().numpy().view(np.uint32), t_host)
    assert np.array_equal(d_arena.cpu().numpy().view(np.uint32), a_host)


def test_large_delta_and_arena_growth(hlkv_lib, cuda_device):
    """Thousands of sequences: many relocations, a delta larger than the first staging buffer."""
    h = hlkv_lib
    t = h.Table(40000, [(1, 33792, 40000)])
    dt = h.DeviceTables()
    seqs = [t.create_sequence()[1] for _ in range(500)]
    rng = np.random.default_rng(1)
    for rnd in range(4):
        for s in seqs:
            for _ in range(int(rng.integers(1, 20))):
                t.append_block(s, 1, 16)
        dt.sync(t)
    table, arena = _device_state(dt)
    st, segs = t.batch_segments(seqs)
    for s, (off, ln) in zip(seqs, segs):
        assert list(arena[off:off + ln]) == t.sequence_block_ids(s)[1]
    want = np.array([t.device_descriptor(i) for i in range(t.max_blocks())], np.uint32)
    assert np.array_equal(table, want)


def test_collect_flush_split_merges_pending_changes(hlkv_lib, cuda_device):
    """DeviceTables.collect (host) twice before one flush (device): the merged delta --
    later patches winning, one patch per target -- leaves the device tables equal to the
    host table, as one sync would."""
    h = hlkv_lib
    t = h.Table(64, [(1, 2048, 64), (3, 1088, 64)], block_tokens=4)
    dt = h.DeviceTables()
    rng = np.random.default_rng(9)
    seqs = [t.create_sequence()[1] for _ in range(6)]
    for rnd in range(30):
        for _ in range(int(rng.integers(1, 4))):       # several collects per flush
            st, tg, done = t.append_tokens(seqs, rng.choice([1, 3], size=len(seqs)).astype(np.uint32), 1)
            assert st == 0 and done == len(seqs)
            if rng.integers(4) == 0:
                i = int(rng.integers(len(seqs)))
                assert t.release_sequence(seqs[i]) == 0
                seqs[i] = t.create_sequence()[1]
            dt.collect(t)
        dt.flush()
        table, arena = _device_state(dt)
        want = np.array([t.device_descriptor(i) for i in range(64)], np.uint32)
        assert np.array_equal(table, want), rnd
        st, segs = t.batch_segments(seqs)
        for s, (off, ln) in zip(seqs, segs):
            assert list(arena[off:off + ln]) == t.sequence_block_ids(s)[1], rnd
    dt.flush()  # nothing pending: a no-op
    assert d2h(dt.error_word_ptr, 4).view(np.uint32)[0] == 0


def test_large_first_sync_then_small_deltas(hlkv_lib, cuda_device):
    """A table of 80,000 block ids: its first delta (every descriptor, 1.28 MB) is copied to
    the device before kernel (3); the small deltas after it are read in place from pinned
    staging.  After each sync the device tables equal the host's."""
    h = hlkv_lib
    n_ids = 80_000
    t = h.Table(n_ids, [(1, 2048, 40_000), (3, 1088, 40_000)])
    dt = h.DeviceTables()
    rng = np.random.default_rng(5)
    seqs = [t.create_sequence()[1] for _ in range(64)]
    for s in seqs:
        for _ in range(int(rng.integers(1, 200))):
            assert t.append_block(s, int(rng.choice([1, 3])), 16)[0] == 0
    assert t.pending()[0] >= 65_536  # at least 1 MiB of descriptor patches
    for step in range(4):
        if step:
            for s in seqs[: 8 * step]:
                st, ids = t.sequence_block_ids(s)
                assert t.set_valid_tokens(t.handle_of(ids[-1]), int(rng.integers(1, 17))) == 0
                assert t.append_block(s, 1, 3)[0] == 0
        dt.sync(t)
        import torch
        torch.cuda.synchronize()
        table, arena = _device_state(dt)
        want = np.array([np.asarray(t.device_descriptor(i), np.uint32) for i in range(n_ids)])
        assert np.array_equal(table, want), step
        st, segs = t.batch_segments(seqs)
        for s, (off, ln) in zip(seqs, segs):
            assert list(arena[off:off + ln]) == list(t.sequence_block_ids(s)[1]), step
    assert int(d2h(dt.error_word_ptr, 4).view(np.uint32)[0]) == 0


def test_restored_table_gathers_like_the_original(hlkv_lib, oracle, cuda_device):
    """Snapshot a table in use, restore it, sync a fresh device mirror from the restored
    table (its first delta is the whole image): the gather through it is bit-identical to
    the gather through the original's mirror."""
    import torch
    from hlkv.workload import build_workload, mixed_formats
    fm = mixed_formats(5, [4, 9, 1, 13, 6], probs=(0.25, 0.3, 0.2, 0.25), seed=41)
    wl = build_workload(fm, T=16, H=4, D=128, seed=42)
    st, restored = hlkv_lib.Table.restore(wl.table.snapshot())
    assert st == 0
    dt = hlkv_lib.DeviceTables()
    dt.sync(restored)
    st, segs = restored.batch_segments(wl.seqs)
    assert st == 0 and np.array_equal(segs, wl.segs_host)
    outs = []
    for tables in (wl.dt, dt):
        out = torch.empty(wl.total_blocks * wl.block_elems, dtype=torch.int16, device="cuda")
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        hlkv_lib.gather_dequant(wl.hlkv_pools(), wl.layout, tables.table_ptr, tables.table_size,
                                tables.arena_ptr, tables.arena_size, wl.segs, out, err)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        outs.append(out.cpu().numpy())
    assert np.array_equal(outs[0], outs[1])


def test_arena_compaction_relocates_the_device_arena(hlkv_lib, oracle, cuda_device):
    """Bursts of long sequences, releases and arena compactions: after each compaction
    (HeteroBlockTable::compact_arena + DeviceTables::relocate, i.e. the two relocation
    launches) and after each later delta, every live sequence's device arena entries equal
    its block ids; the arena pointer never changes (virtual memory management); a gather
    through the compacted tables equals the oracle's."""
    import torch
    from helpers import oracle_gather
    from hlkv.workload import KVWorkload
    h = hlkv_lib
    T, H, D = 4, 2, 64
    layout = h.Layout(T, H, D, 1)
    sb = {f: (h.layout_slot_bytes(f, layout) + 15) // 16 * 16 for f in (1, 3)}
    t = h.Table(30000, [(1, sb[1], 15000), (3, sb[3], 15000)], block_tokens=T)
    dt = h.DeviceTables()
    rng = np.random.default_rng(99)
    seqs = []
    arena_ptr = None
    for rnd in range(12):
        # a burst: a few long sequences, many short ones
        for _ in range(int(rng.integers(20, 60))):
            st, s = t.create_sequence()
            assert st == 0
            seqs.append(s)
            n = int(rng.integers(200, 900)) if rng.random() < 0.15 else int(rng.integers(1, 12))
            for _ in range(n):
                if t.append_block(s, int(rng.choice([1, 3])), int(rng.integers(1, T + 1)))[0] != 0:
                    break
        dt.sync(t)
        arena_ptr = arena_ptr or dt.arena_ptr
        assert dt.arena_ptr == arena_ptr  # growth mapped more memory behind the same address
        # release most of the long ones, then compact
        for i in sorted(rng.choice(len(seqs), size=len(seqs) // 2, replace=False), reverse=True):
            assert t.release_sequence(seqs.pop(int(i))) == 0
        dt.sync(t)
        st, moves = t.compact_arena()
        assert st == 0
        dt.relocate(moves, t.stats()["arena_entries"])
        torch.cuda.synchronize()
        assert dt.arena_ptr == arena_ptr
        assert dt.arena_size == t.stats()["arena_entries"]
        _, arena = _device_state(dt)
        st, segs = t.batch_segments(seqs)
        for s, (off, ln) in zip(seqs, segs):
            assert list(arena[off:off + ln]) == t.sequence_block_ids(s)[1], f"round {rnd}"
        # more appends after the compaction go through ordinary deltas
        for s in seqs[: len(seqs) // 3]:
            t.append_block(s, 3, 1)
        dt.sync(t)
        _, arena = _device_state(dt)
        st, segs = t.batch_segments(seqs)
        for s, (off, ln) in zip(seqs, segs):
            assert list(arena[off:off + ln]) == t.sequence_block_ids(s)[1], f"round {rnd} after"
    assert d2h(dt.error_word_ptr, 4).view(np.uint32)[0] == 0

    # A gather through the compacted tables, against the oracle on the same bytes.
    gen = torch.Generator(device="cuda")
    gen.manual_seed(5)
    pools = {}
    for f in (1, 3):
        buf = torch.randint(0, 256, (15000, sb[f]), generator=gen, device="cuda", dtype=torch.uint8)
        if f == 1:  # keep the scales finite and moderate: bytes of binary32 values in [1/4, 1)
            rows = 2 * T * H
            scales = torch.rand((15000, rows), generator=gen, device="cuda") * 0.75 + 0.25
            buf[:, T * H * D * 2:T * H * D * 2 + 4 * rows] = scales.view(torch.uint8)
        else:
            rows = 2 * T * H
            sbias = torch.rand((15000, rows, 2), generator=gen, device="cuda") + 0.1
            buf[:, T * H * D:T * H * D + 8 * rows] = sbias.reshape(15000, -1).view(torch.uint8)
        pools[f] = (buf, sb[f], 15000)
    st, segs_host = t.batch_segments(seqs)
    wl = KVWorkload(T, H, D, layout, t, dt, pools, seqs,
                    torch.from_numpy(segs_host.astype(np.int32).reshape(-1, 2)).cuda(), segs_host)
    out = torch.empty(max(1, wl.total_blocks) * wl.block_elems, dtype=torch.int16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    h.gather_dequant(wl.hlkv_pools(), layout, dt.table_ptr, dt.table_size, dt.arena_ptr, dt.arena_size,
                     wl.segs, out, err)
    torch.cuda.synchronize()
    want, oerr = oracle_gather(oracle, wl)
    assert int(err.item()) == 0 and oerr == 0
    got = out.cpu().numpy().view(np.uint16)[:want.size]
    assert np.array_equal(got, want)


def test_arena_memory_returned_after_compaction(hlkv_lib, cuda_device):
    """An arena of several MB (16 sequences of 40,000 blocks), most of it released and
    compacted: the device memory behind the arena shrinks to about the packed size plus a
    quarter, at the same address, and the remaining sequences are intact."""
    h = hlkv_lib
    t = h.Table(700000, [(1, 64, 700000)], block_tokens=16)
    dt = h.DeviceTables()
    seqs = [t.create_sequence()[1] for _ in range(16)]
    for s in seqs:
        for _ in range(40000):
            assert t.append_block(s, 1, 16)[0] == 0
    dt.sync(t)
    ptr, cap0 = dt.arena_ptr, dt.arena_capacity_bytes
    assert cap0 >= 16 * 65536 * 4  # 16 segments of the 65,536-entry class
    for s in seqs[:14]:
        assert t.release_sequence(s) == 0
    seqs = seqs[14:]
    dt.sync(t)
    st, moves = t.compact_arena()
    assert st == 0
    size = t.stats()["arena_entries"]
    assert size == 2 * 65536
    dt.relocate(moves, size)
    assert dt.arena_ptr == ptr
    assert dt.arena_capacity_bytes < cap0
    assert size * 4 <= dt.arena_capacity_bytes <= size * 4 * 5 // 4 + (2 << 20)
    _, arena = _device_state(dt)
    st, segs = t.batch_segments(seqs)
    for s, (off, ln) in zip(seqs, segs):
        assert list(arena[off:off + ln]) == t.sequence_block_ids(s)[1]
    # and it grows again behind the same address
    for s in seqs:
        for _ in range(30000):
            assert t.append_block(s, 1, 16)[0] == 0
    dt.sync(t)
    assert dt.arena_ptr == ptr
    _, arena = _device_state(dt)
    st, segs = t.batch_segments(seqs)
    for s, (off, ln) in zip(seqs, segs):
        assert list(arena[off:off + ln]) == t.sequence_block_ids(s)[1]

"""Kernel (2), hlkv_append_encode, against the CPU oracle's append (quantize_reference
per row): every byte of every pool -- codes, parameters and untouched slots -- must
match, and the error bits must agree."""
import numpy as np
import pytest

from helpers import device_table_words, host_pools

pytestmark = pytest.mark.gpu


def _tokens(n: int, H: int, D: int, seed: int) -> np.ndarray:
    """FP16 tokens [n, 2, H, D] with the awkward cases: signed-zero rows, constants,
    subnormals, FP16 extremes, a ramp, big outliers."""
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((n, 2, H, D)) * rng.choice([0.01, 1, 30, 1000], size=(n, 2, H, 1))).astype(np.float16)
    x[0, 0, 0] = 0.0
    x[0, 0, 0, ::3] = -0.0                      # mixed signed zeros (min/max ties)
    x[0, 1, 0] = -0.0
    x[0, 1, 0, 5] = 0.0
    x[1, 0, 0] = 2.5                            # constant row: INT4 scale 0
    x[1, 1, 0] = np.float16(6e-8) * np.arange(D)  # subnormal ramp
    x[2, 0, 0, :4] = [65504, -65504, 1, -1]
    x[2, 1, 0] = np.linspace(-7, 7, D)
    if n > 3:
        # quotients exactly on rounding boundaries (the encoders' exact fallback path):
        # INT4 min 0 / max 15 -> scale 1 and .5 ties; E4M3 amax 448 -> scale 1 and FP8
        # midpoints (normal, subnormal, saturating); E5M2 amax 57344 likewise
        x[3, 0, 0] = np.tile([0, 15, 0.5, 1.5, 7.5, 14.5, 3.5, 8.5], D // 8)
        x[3, 1, 0] = np.tile([448, 1.0625, -3.25, 248, 464, 2.0 ** -10, -3 * 2.0 ** -10, 17], D // 8)
        x[3, 1, 1] = np.tile([57344, 1.125, -2.25, 2.0 ** -17, 3 * 2.0 ** -17, 40960, -5, 0.5], D // 8)
        x[3, 0, 1] = np.tile([-0.0, 0.0, 2.0, -0.0, 1.0, 0.0, 3.0, 0.5], D // 8)   # min -0 with +0 present
    return x


def _run(hlkv, wl, targets, tokens):
    import torch
    d_t = torch.from_numpy(targets.astype(np.int32)).cuda()
    d_x = torch.from_numpy(tokens.view(np.int16).copy()).cuda()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    hlkv.append_encode(wl.hlkv_pools(), wl.layout, wl.dt.table_ptr, wl.dt.table_size, d_t, d_x, err)
    torch.cuda.synchronize()
    return int(err.item())


def _all_ids(wl):
    ids = []
    for s in wl.seqs:
        st, b = wl.table.sequence_block_ids(s)
        ids += b
    return ids


@pytest.mark.parametrize("T,H,D", [(16, 8, 128), (4, 2, 64), (2, 2, 256), (5, 3, 64), (512, 2, 128)])
def test_append_encode_bit_exact(hlkv_lib, oracle, cuda_device, T, H, D):
    from hlkv.workload import build_workload
    fm = [[0, 1, 2, 3, 1, 3, 0], [3, 1, 2]]
    wl = build_workload(fm, T=T, H=H, D=D, seed=T + D, valid_tokens=[[0] * 7, [1] * 3],
                        outlier_channels=0)
    ids = _all_ids(wl)
    rng = np.random.default_rng(D)
    pairs = [(i, t) for i in ids for t in range(T)]
    pick = rng.choice(len(pairs), size=min(40, len(pairs)), replace=False)
    targets = np.array([pairs[k] for k in pick], dtype=np.uint32)
    tokens = _tokens(len(targets), H, D, seed=T * D)
    before = host_pools(wl)
    table = device_table_words(wl)
    err = _run(hlkv_lib, wl, targets, tokens)
    oerr = oracle.append_encode(before, T, H, D, 1, table, targets, tokens.view(np.uint16))
    assert err == oerr == 0
    after = host_pools(wl)
    for f in before:
        got, want = after[f][0], before[f][0]
        bad = np.nonzero(got != want)[0]
        assert bad.size == 0, f"format {f}: {bad.size} bytes differ, first at {bad[:4]}"


def test_append_rejects_bad_rows_and_targets(hlkv_lib, oracle, cuda_device):
    from hlkv.workload import build_workload
    T, H, D = 4, 2, 64
    wl = build_workload([[1, 3, 0]], T=T, H=H, D=D, seed=2, outlier_channels=0, spare_slots=1)
    ids = _all_ids(wl)
    free_id = next(i for i in range(wl.table.max_blocks()) if i not in ids)
    targets = np.array([[ids[0], 1], [ids[1], 2], [ids[2], 0],   # valid
                        [ids[0], T], [free_id, 0], [10 ** 6, 0],  # token range, not executable, id range
                        [ids[1], 3]], dtype=np.uint32)
    tokens = _tokens(len(targets), H, D, seed=5)
    tokens[1, 0, 1, 7] = np.inf    # one INT4 row rejected
    tokens[6, 1, 0, 0] = np.nan    # one INT4 row rejected
    before = host_pools(wl)
    table = device_table_words(wl)
    err = _run(hlkv_lib, wl, targets, tokens)
    oerr = oracle.append_encode(before, T, H, D, 1, table, targets, tokens.view(np.uint16))
    assert oerr == (1 << 9) | (1 << 10) | (1 << 0) | (1 << 4)
    assert err == oerr
    after = host_pools(wl)
    for f in before:
        assert np.array_equal(after[f][0], before[f][0]), f


def test_append_then_gather_round_trip(hlkv_lib, oracle, cuda_device):
    """Decode step: encode one token per sequence into the tail block, set valid_tokens on the
    host, apply the delta on the device, gather -- the new token decodes as the oracle says."""
    import torch
    from helpers import oracle_gather
    from hlkv.workload import build_workload
    T, H, D = 16, 8, 128
    wl = build_workload([[1, 3], [3, 1], [0, 1]], T=T, H=H, D=D, seed=8,
                        valid_tokens=[[16, 5], [16, 9], [16, 0]])
    targets, tokens = [], _tokens(3, H, D, seed=9)
    for s, vt in zip(wl.seqs, (5, 9, 0)):
        st, ids = wl.table.sequence_block_ids(s)
        tail = wl.table.handle_of(ids[-1])
        assert wl.table.set_valid_tokens(tail, vt + 1) == 0
        targets.append((ids[-1], vt))
    wl.dt.sync(wl.table)
    err = _run(hlkv_lib, wl, np.array(targets, np.uint32), tokens)
    assert err == 0
    n = wl.total_blocks * wl.block_elems
    out = torch.empty(n, dtype=torch.int16, device="cuda")
    e = torch.zeros(1, dtype=torch.int32, device="cuda")
    hlkv_lib.gather_dequant(wl.hlkv_pools(), wl.layout, wl.dt.table_ptr, wl.dt.table_size,
                            wl.dt.arena_ptr, wl.dt.arena_size, wl.segs, out, e)
    torch.cuda.synchronize()
    want, oerr = oracle_gather(oracle, wl)
    assert int(e.item()) == 0 and oerr == 0
    assert np.array_equal(out.cpu().numpy().view(np.uint16), want)


@pytest.mark.parametrize("D", [64, 128, 256])
def test_append_rejects_every_nonfinite_pattern(hlkv_lib, oracle, cuda_device, D):
    """Rows holding +-Inf, +-NaN (quiet, signalling-pattern, all-ones) at positions in either
    8-value chunk of a lane and either half of a word are rejected in E4M3, E5M2 and INT4
    blocks; rows at the finite extremes (+-65504, the largest subnormal) are encoded."""
    from hlkv.workload import build_workload
    T, H = 4, 2
    wl = build_workload([[1, 2, 3]], T=T, H=H, D=D, seed=D, outlier_channels=0)
    ids = _all_ids(wl)
    specials = [0x7C00, 0xFC00, 0x7E00, 0xFE00, 0x7C01, 0xFFFF, 0x7FFF, 0xFC01]
    where = [0, 1, 9, D // 2 + 3, D - 1, D - 2, 16 + 7, D // 2 - 8]
    targets = []
    for bid in ids:
        for t in range(T):
            targets.append((bid, t))
    targets = np.array(targets, dtype=np.uint32)
    tokens = _tokens(len(targets), H, D, seed=D + 1)
    bits = tokens.view(np.uint16)
    rng = np.random.default_rng(D)
    for k in range(len(targets)):
        for kv in range(2):
            for h in range(H):
                r = (k * 2 + kv) * H + h
                if r % 3 == 0:
                    bits[k, kv, h, where[r % len(where)]] = specials[r % len(specials)]
                elif r % 3 == 1:
                    bits[k, kv, h, rng.integers(0, D)] = rng.choice([0x7BFF, 0xFBFF, 0x03FF, 0x83FF])
    before = host_pools(wl)
    table = device_table_words(wl)
    err = _run(hlkv_lib, wl, targets, tokens)
    oerr = oracle.append_encode(before, T, H, D, 1, table, targets, bits)
    assert oerr == 1 << 9
    assert err == oerr
    after = host_pools(wl)
    for f in before:
        bad = np.nonzero(after[f][0] != before[f][0])[0]
        assert bad.size == 0, f"format {f}: {bad.size} bytes differ, first at {bad[:4]}"


def test_decode_step_queue_matches_oracle(hlkv_lib, oracle, cuda_device):
    """hlkv_decode_step_queue over several decode steps (T = 4, so new blocks open): after
    each step the device descriptor table mirrors the host table, every pool byte equals the
    oracle's append of the same tokens at the same targets, and the final gather through the
    device tables equals the oracle's."""
    import torch
    from helpers import oracle_gather
    from hlkv.workload import build_workload
    T, H, D = 4, 2, 128
    wl = build_workload([[1, 3], [3], [1, 1, 3]], T=T, H=H, D=D, seed=11,
                        valid_tokens=[[4, 1], [3], [4, 4, 0]], spare_slots=16)
    n = len(wl.seqs)
    h_targets = torch.empty((n, 2), dtype=torch.int32).pin_memory()
    d_targets = torch.empty((n, 2), dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    rng = np.random.default_rng(12)
    for step in range(9):
        fm = rng.choice([1, 3], size=n).astype(np.uint32)
        st, tg, done = wl.table.append_tokens(wl.seqs, fm, 1, out=h_targets.numpy().view(np.uint32))
        assert st == 0 and done == n
        targets = tg.copy()
        tokens = _tokens(n, H, D, seed=100 + step)
        before = host_pools(wl)
        wl.dt.collect(wl.table)
        # odd steps: the start and encode events (the kernels then do not overlap)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)] if step % 2 else None
        if ev:
            for e in ev:
                e.record()  # torch creates the CUDA event at its first record
        hlkv_lib.decode_step_queue(wl.dt, wl.hlkv_pools(), wl.layout, h_targets, d_targets,
                                   torch.from_numpy(tokens.view(np.int16).copy()).cuda(), err,
                                   start_event=ev[0] if ev else None, encode_event=ev[1] if ev else None)
        if ev:
            ev[2].record()
        torch.cuda.synchronize()
        if ev:
            assert ev[0].elapsed_time(ev[1]) > 0 and ev[1].elapsed_time(ev[2]) > 0
        assert int(err.item()) == 0
        assert np.array_equal(d_targets.cpu().numpy().view(np.uint32), targets)
        table = device_table_words(wl)
        for s in wl.seqs:
            for bid in wl.table.sequence_block_ids(s)[1]:
                assert np.array_equal(table[bid], np.asarray(wl.table.device_descriptor(bid), np.uint32))
        oerr = oracle.append_encode(before, T, H, D, 1, table, targets, tokens.view(np.uint16))
        assert oerr == 0
        after = host_pools(wl)
        for f in before:
            bad = np.nonzero(after[f][0] != before[f][0])[0]
            assert bad.size == 0, f"step {step} format {f}: {bad.size} bytes differ"
    import ctypes as C
    import hlkv
    from helpers import device_arena
    # pageable host memory cannot be read by kernel (3): rejected before anything is queued
    pageable = np.zeros((n, 2), np.uint32)
    st = hlkv.lib().hlkv_decode_step_queue(wl.dt.h, C.byref(wl.hlkv_pools()), C.byref(wl.layout),
                                           pageable.ctypes.data, d_targets.data_ptr(), n,
                                           d_targets.data_ptr(), err.data_ptr(), None, None, None)
    assert st == hlkv.INVALID_ARGUMENT
    st, segs_host = wl.table.batch_segments(wl.seqs)
    assert st == hlkv.Status.OK
    wl.dt.sync(wl.table)
    wl.segs_host = segs_host
    wl.segs = torch.from_numpy(segs_host.astype(np.int32).reshape(-1, 2)).cuda()
    arena = device_arena(wl)
    for s, (off, ln) in zip(wl.seqs, segs_host):
        assert list(arena[off:off + ln]) == list(wl.table.sequence_block_ids(s)[1])
    out = torch.empty(wl.total_blocks * wl.block_elems, dtype=torch.int16, device="cuda")
    e = torch.zeros(1, dtype=torch.int32, device="cuda")
    hlkv_lib.gather_dequant(wl.hlkv_pools(), wl.layout, wl.dt.table_ptr, wl.dt.table_size,
                            wl.dt.arena_ptr, wl.dt.arena_size, wl.segs, out, e)
    torch.cuda.synchronize()
    want, oerr = oracle_gather(oracle, wl)
    assert int(e.item()) == 0 and oerr == 0
    assert np.array_equal(out.cpu().numpy().view(np.uint16), want)

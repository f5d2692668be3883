"""Kernel (1), hlkv_gather_dequant, against the CPU oracle: bit-exact on every element.

The oracle (oracle/hlkv_oracle.c) restates the reference's
dequantize_reference_to_fp16 and walks the same device tables; the kernel must
produce the same bits (NaN payloads included) and the same error bits, and
leave skipped blocks untouched.
"""
import numpy as np
import pytest

from helpers import assert_bits_equal, device_arena, device_table_words, oracle_gather

pytestmark = pytest.mark.gpu


def _run(hlkv, wl, out_elems=None, out_offsets=None, fill=0xABCD, table=None, arena=None, segs=None):
    import torch
    n = out_elems if out_elems is not None else wl.total_blocks * wl.block_elems
    out = torch.from_numpy(np.full(max(n, 1), fill, dtype=np.uint16).view(np.int16)).cuda()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    offs = None if out_offsets is None else torch.from_numpy(out_offsets.astype(np.int64)).cuda()
    tptr, tsz = (wl.dt.table_ptr, wl.dt.table_size) if table is None else (table.data_ptr(), table.shape[0])
    aptr, asz = (wl.dt.arena_ptr, wl.dt.arena_size) if arena is None else (arena.data_ptr(), arena.numel())
    sg = wl.segs if segs is None else segs
    hlkv.gather_dequant(wl.hlkv_pools(), wl.layout, tptr, tsz, aptr, asz, sg, out, err,
                        out_offsets=offs)
    torch.cuda.synchronize()
    return out.cpu().numpy().view(np.uint16)[:n], int(err.item())


@pytest.fixture(scope="module")
def small_mixed(cuda_device, hlkv_lib):
    from hlkv.workload import build_workload, mixed_formats
    rng = np.random.default_rng(5)
    lens = [3, 0, 7, 1, 12, 2]
    fm = mixed_formats(len(lens), lens, probs=(0.25, 0.3, 0.2, 0.25), seed=5)
    vt = [[int(rng.integers(0, 17)) for _ in range(n)] for n in lens]
    return build_workload(fm, T=16, H=8, D=128, seed=5, valid_tokens=vt, spare_slots=3)


def test_mixed_ragged_bit_exact(hlkv_lib, oracle, small_mixed):
    got, err = _run(hlkv_lib, small_mixed)
    want, oerr = oracle_gather(oracle, small_mixed)
    assert err == 0 and oerr == 0
    assert_bits_equal(got, want, "mixed ragged")


def test_device_tables_match_host(hlkv_lib, small_mixed):
    from hlkv.workload import host_arena, host_table
    wl = small_mixed
    assert np.array_equal(device_table_words(wl), host_table(wl))
    arena = device_arena(wl)
    for off, ln in wl.segs_host:
        assert np.array_equal(arena[off:off + ln], host_arena(wl)[off:off + ln])


@pytest.mark.parametrize("T,H,D", [(4, 2, 64), (16, 8, 128), (2, 3, 256), (1, 1, 64), (32, 1, 128),
                                   (128, 4, 128), (512, 1, 64)])  # 512: the largest block_tokens
def test_geometries(hlkv_lib, oracle, cuda_device, T, H, D):
    from hlkv.workload import build_workload, mixed_formats
    rng = np.random.default_rng(T * 100 + H * 10 + D)
    lens = [int(x) for x in rng.integers(0, 9, size=5)]
    fm = mixed_formats(5, lens, probs=(0.25, 0.25, 0.25, 0.25), seed=T + H + D)
    vt = [[int(rng.integers(0, T + 1)) for _ in range(n)] for n in lens]
    wl = build_workload(fm, T=T, H=H, D=D, seed=D + T, valid_tokens=vt, outlier_channels=2)
    got, err = _run(hlkv_lib, wl)
    want, oerr = oracle_gather(oracle, wl)
    assert err == oerr == 0
    assert_bits_equal(got, want, f"T={T} H={H} D={D}")


def test_homogeneous_e4m3_full_size(hlkv_lib, oracle, cuda_device):
    """The homogeneous E4M3 shape: 1 sequence x 4096 tokens, 16-token blocks, 8 x 128, K and V."""
    from hlkv.workload import build_workload
    wl = build_workload([[1] * 256], seed=1)
    got, err = _run(hlkv_lib, wl)
    want, oerr = oracle_gather(oracle, wl)
    assert err == oerr == 0
    assert_bits_equal(got, want, "homogeneous E4M3")


def test_mixed_single_layer_full_size(hlkv_lib, oracle, cuda_device):
    """The mixed single-layer shape at full size: 64 x 2048 tokens, FP16 .25 / E4M3 .5 / INT4 .25."""
    from hlkv.workload import build_workload, mixed_formats
    wl = build_workload(mixed_formats(64, 128, seed=2), seed=2)
    got, err = _run(hlkv_lib, wl)
    want, oerr = oracle_gather(oracle, wl, threads=32)
    assert err == oerr == 0
    assert_bits_equal(got, want, "mixed single layer")


def test_many_sequences_chunked_scan(hlkv_lib, oracle, cuda_device):
    """More than 256 sequences (several prefix-scan chunks), many of them empty."""
    from hlkv.workload import build_workload, mixed_formats
    rng = np.random.default_rng(9)
    lens = [int(x) for x in rng.integers(0, 4, size=700)]
    wl = build_workload(mixed_formats(700, lens, probs=(1, 1, 1, 1), seed=9), T=2, H=1, D=64, seed=9,
                        outlier_channels=0)
    got, err = _run(hlkv_lib, wl)
    want, oerr = oracle_gather(oracle, wl)
    assert err == oerr == 0
    assert_bits_equal(got, want, "700 sequences")


def test_out_offsets_leave_gaps_untouched(hlkv_lib, oracle, small_mixed):
    wl = small_mixed
    lens = wl.segs_host[:, 1].astype(np.int64)
    offs = np.zeros(len(lens), dtype=np.int64)
    pos = 24  # leading gap, multiple of 8 elements
    for i in reversed(range(len(lens))):  # reversed order and gaps between sequences
        offs[i] = pos
        pos += lens[i] * wl.block_elems + 8 * (i + 1)
    got, err = _run(hlkv_lib, wl, out_elems=pos, out_offsets=offs, fill=0x5A5A)
    want, oerr = oracle_gather(oracle, wl, out_elems=pos, out_offsets=offs, fill=0x5A5A)
    assert err == oerr == 0
    assert_bits_equal(got, want, "out_offsets")
    assert got[0] == 0x5A5A and got[pos - 1] == 0x5A5A


def test_special_codes_nan_inf(hlkv_lib, oracle, cuda_device):
    """NaN/Inf codes and zero/negative scales: the reference's x86 bits, NaN payloads included."""
    import torch
    from hlkv import FP16, FP8_E4M3, FP8_E5M2
    from hlkv.workload import build_workload, code_bytes
    wl = build_workload([[FP16, FP8_E4M3, FP8_E5M2, FP8_E5M2]], T=4, H=2, D=64, seed=4,
                        outlier_channels=0)
    rows, elems = 2 * 4 * 2, 2 * 4 * 2 * 64
    g = np.random.default_rng(4)
    for f in (FP8_E4M3, FP8_E5M2):
        buf, sb, ns = wl.pools[f]
        host = buf.cpu().numpy()
        host[:, :elems] = g.integers(0, 256, size=(ns, elems), dtype=np.uint8)  # every code incl. NaN/Inf
        scales = np.array([0.0, -0.0, -1.5, 2.0 ** -130, 65504.0 / 448.0, 1e4, 1.0, 3.7e-3],
                          dtype=np.float32)
        host[:, code_bytes(f, elems):code_bytes(f, elems) + 4 * rows] = \
            np.resize(scales, (ns, rows)).astype(np.float32).view(np.uint8).reshape(ns, -1)
        buf.copy_(torch.from_numpy(host))
    buf, sb, ns = wl.pools[FP16]
    host = buf.cpu().numpy()
    codes = g.integers(0, 65536, size=(ns, elems), dtype=np.uint16)
    codes[:, :8] = [0x7C01, 0xFC01, 0x7FFF, 0xFE00, 0x7C00, 0xFC00, 0x8000, 0x0001]
    host[:, :2 * elems] = codes.view(np.uint8)
    buf.copy_(torch.from_numpy(host))
    got, err = _run(hlkv_lib, wl)
    want, oerr = oracle_gather(oracle, wl)
    assert err == oerr == 0
    assert_bits_equal(got, want, "special codes")


def test_error_bits_and_skips(hlkv_lib, oracle, cuda_device):
    """Corrupt descriptors and indices: the same error bits as the oracle, skipped blocks untouched."""
    import torch
    from hlkv import FP8_E4M3, FP16, INT4, pack_info
    from hlkv.workload import build_workload
    wl = build_workload([[FP16, FP8_E4M3, INT4, FP8_E4M3]], T=4, H=2, D=64, seed=3,
                        outlier_channels=0, spare_slots=2)
    table = device_table_words(wl).copy()
    arena = device_arena(wl).copy()
    off, ln = wl.segs_host[0]
    ids = arena[off:off + ln]
    n = table.shape[0]
    # Extra sequences pointing at hand-made records.  Each entry: (arena ids, expected bit).
    extra_ids = []
    def add_record(slot, info, block_id_field=None):
        nonlocal table
        bid = table.shape[0]
        rec = np.array([[slot, info, 0, bid if block_id_field is None else block_id_field]], np.uint32)
        table = np.concatenate([table, rec])
        return bid
    cases = [
        add_record(0xFFFFFFFF, 15),                                   # not executable
        add_record(0, pack_info(5, 0, 1, 4)),                         # unknown format
        add_record(0, pack_info(FP8_E4M3, 0, 2, 4)),                  # layout mismatch
        add_record(0, pack_info(FP8_E4M3, 3, 1, 4)),                  # scale mode 3 (external)
        add_record(0, pack_info(INT4, 0, 1, 5)),                      # valid_tokens > T
        add_record(999, pack_info(FP16, 0, 1, 4)),                    # slot out of range
        add_record(0, pack_info(FP16, 0, 1, 4), block_id_field=7),    # block_id mismatch
    ]
    base = arena.size
    arena = np.concatenate([arena, np.array(cases + [n + 1000], dtype=np.uint32)])  # + id out of range
    segs = np.concatenate([wl.segs_host, [[base, len(cases) + 1]], [[arena.size - 1, 3]]]).astype(np.uint32)
    d_table = torch.from_numpy(table.view(np.int32)).cuda()
    d_arena = torch.from_numpy(arena.view(np.int32)).cuda()
    d_segs = torch.from_numpy(segs.view(np.int32)).cuda()
    total = int(segs[:, 1].sum())
    got, err = _run(hlkv_lib, wl, out_elems=total * wl.block_elems, table=d_table, arena=d_arena,
                    segs=d_segs, fill=0x1234)
    want, oerr = oracle_gather(oracle, wl, out_elems=total * wl.block_elems, table=table,
                               arena=arena, segs=segs, fill=0x1234)
    assert oerr == (1 | 2 | 4 | 8 | 16 | 32 | 64 | 128 | 256)
    assert err == oerr
    assert_bits_equal(got, want, "error injection")
    assert np.all(got[ln * wl.block_elems:] == 0x1234)  # every injected block was skipped
    assert not np.any(got[:ln * wl.block_elems] == 0x1234)


def test_misaligned_out_offset_is_reported(hlkv_lib, oracle, small_mixed):
    wl = small_mixed
    lens = wl.segs_host[:, 1].astype(np.int64)
    offs = np.concatenate([[0], np.cumsum(lens[:-1]) * wl.block_elems]).astype(np.int64)
    offs[2] += 4  # not a multiple of 8 elements
    n = int(lens.sum()) * wl.block_elems + 8
    got, err = _run(hlkv_lib, wl, out_elems=n, out_offsets=offs, fill=0x7777)
    want, oerr = oracle_gather(oracle, wl, out_elems=n, out_offsets=offs, fill=0x7777)
    assert err == oerr == 4096
    assert_bits_equal(got, want, "misaligned offset")


def test_argument_errors_launch_nothing(hlkv_lib, small_mixed):
    import torch
    wl = small_mixed
    out = torch.zeros(8, dtype=torch.int16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    bad = hlkv_lib.Layout(16, 8, 96, 1)  # unsupported head_dim
    with pytest.raises(hlkv_lib.HlkvError):
        hlkv_lib.gather_dequant(wl.hlkv_pools(), bad, wl.dt.table_ptr, wl.dt.table_size,
                                wl.dt.arena_ptr, wl.dt.arena_size, wl.segs, out, err)
    # nseq == 0 is a no-op
    hlkv_lib.gather_dequant(wl.hlkv_pools(), wl.layout, wl.dt.table_ptr, wl.dt.table_size,
                            wl.dt.arena_ptr, wl.dt.arena_size, wl.segs[:0], out, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0 and int(out.abs().sum().item()) == 0


def test_repeatable(hlkv_lib, small_mixed):
    a, _ = _run(hlkv_lib, small_mixed)
    b, _ = _run(hlkv_lib, small_mixed)
    assert np.array_equal(a, b)


@pytest.mark.parametrize("T,H,D", [(16, 8, 128), (4, 2, 64), (2, 2, 256)])
def test_block_wide_scale_modes(hlkv_lib, oracle, cuda_device, T, H, D):
    """Blocks whose descriptors carry block-wide parameters (scale mode 1: binary32 scale in
    scale_ref; mode 2: binary16 scale and bias) decode with those for every row; scale mode 3
    and parameters the reference's dequantizer rejects (non-finite, FP8 bias) skip the block
    with HLKV_ERR_SCALE_MODE.  Bit-exact against the oracle, which the reference-built
    gather pins (tests/test_oracle_golden.py)."""
    from helpers import block_wide_scale_refs
    from hlkv.workload import build_workload, mixed_formats
    rng = np.random.default_rng(T * D)
    lens = [5, 9, 3, 11]
    fm = mixed_formats(len(lens), lens, probs=(0.2, 0.3, 0.2, 0.3), seed=D)
    vt = [[int(rng.integers(1, T + 1)) for _ in range(n)] for n in lens]
    wl = build_workload(fm, T=T, H=H, D=D, seed=D + 1, valid_tokens=vt)
    ids = []
    for s in wl.seqs:
        ids += wl.table.sequence_block_ids(s)[1]
    refs = block_wide_scale_refs(rng, len(ids))
    for k, bid in enumerate(ids):
        if k % 3 == 2:
            continue  # per-row parameters
        mode, sref = (3, 12) if k == 4 else refs[k]
        assert wl.table.set_scale(wl.table.handle_of(bid), mode, sref) == 0
    wl.dt.sync(wl.table)
    out, err = _run(hlkv_lib, wl)
    want, oerr = oracle_gather(oracle, wl, fill=0xABCD)
    assert err == oerr and err & (1 << 7)
    assert_bits_equal(out, want)
    # block-wide blocks were decoded, not only skipped
    decoded = sum(1 for k in range(len(ids)) if k % 3 != 2)
    per_block = out.reshape(len(ids), -1)
    assert (per_block != 0xABCD).all(axis=1).sum() >= decoded // 2


def test_overlapped_layer_launches(hlkv_lib, oracle, cuda_device):
    """Back-to-back per-layer gathers launched with HLKV_LAUNCH_OVERLAP_PREVIOUS (programmatic
    dependent launch): each launch's prologue may overlap the previous layer's gather, but its
    output writes wait for it.  Eight layers into one shared scratch (the last layer must win)
    and into separate buffers (each layer exact), with an error-bit case in the middle layer."""
    import torch
    from hlkv.workload import build_workload, mixed_formats
    layers, nseq = 8, 6
    rows = []
    for l in range(layers):
        rows += mixed_formats(nseq, [5, 0, 9, 3, 17, 2], probs=(0.25, 0.3, 0.2, 0.25), seed=40 + l)
    wl = build_workload(rows, seed=41)
    segs = [wl.segs[l * nseq:(l + 1) * nseq] for l in range(layers)]
    lb = [int(wl.segs_host[l * nseq:(l + 1) * nseq, 1].sum()) for l in range(layers)]
    n = max(lb) * wl.block_elems
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    pools = wl.hlkv_pools()
    shared = torch.full((n,), 0x5A5A, dtype=torch.int16, device="cuda")
    sep = [torch.full((lb[l] * wl.block_elems,), 0x5A5A, dtype=torch.int16, device="cuda") for l in range(layers)]
    for rep in range(3):
        for l in range(layers):
            hlkv_lib.gather_dequant(pools, wl.layout, wl.dt.table_ptr, wl.dt.table_size, wl.dt.arena_ptr,
                                    wl.dt.arena_size, segs[l], shared, err, overlap_previous=True)
        for l in range(layers):
            hlkv_lib.gather_dequant(pools, wl.layout, wl.dt.table_ptr, wl.dt.table_size, wl.dt.arena_ptr,
                                    wl.dt.arena_size, segs[l], sep[l], err, overlap_previous=(l > 0))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    table, arena = device_table_words(wl), device_arena(wl)
    for l in range(layers):
        s = np.ascontiguousarray(wl.segs_host[l * nseq:(l + 1) * nseq])
        want, oerr = oracle_gather(oracle, wl, out_elems=lb[l] * wl.block_elems, table=table, arena=arena, segs=s)
        assert oerr == 0
        assert_bits_equal(sep[l].cpu().numpy().view(np.uint16), want, f"layer {l}")
        if l == layers - 1:
            got = shared.cpu().numpy().view(np.uint16)
            assert_bits_equal(got[:want.size], want, "shared scratch holds the last layer")
    # A bad arena entry in the middle layer: its bit arrives through the overlapped launch.
    bad = np.ascontiguousarray(wl.segs_host[3 * nseq:4 * nseq]).copy()
    bad[0, 0] = wl.dt.arena_size  # the first sequence's 5 blocks lie past the arena (same total)
    bad_t = torch.from_numpy(bad.astype(np.int32)).cuda()
    err.zero_()
    torch.cuda.synchronize()
    hlkv_lib.gather_dequant(pools, wl.layout, wl.dt.table_ptr, wl.dt.table_size, wl.dt.arena_ptr,
                            wl.dt.arena_size, segs[2], shared, err, overlap_previous=False)
    hlkv_lib.gather_dequant(pools, wl.layout, wl.dt.table_ptr, wl.dt.table_size, wl.dt.arena_ptr,
                            wl.dt.arena_size, bad_t, shared, err, overlap_previous=True)
    torch.cuda.synchronize()
    assert int(err.item()) == hlkv_lib.ERR_ARENA_RANGE

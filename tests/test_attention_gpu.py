"""Decode attention fused with the heterogeneous dequantization (hlkv_decode_attention)
against float64 attention over the oracle's bit-exact gather of the same blocks.  The
kernel computes in binary32 and rounds to binary16: the tolerance below is 2 binary16 ulps
of the result plus 1e-3 of the value scale."""
import numpy as np
import pytest

from helpers import oracle_attention

pytestmark = pytest.mark.gpu


def _close(got, want, vscale):
    tol = 2 * 2.0 ** -11 * np.abs(want) + 1e-3 * vscale
    bad = np.abs(got - want) > tol
    assert not bad.any(), (int(bad.sum()), got[bad][:4], want[bad][:4])


def _run(hlkv, wl, q_heads, scale, seed, segs=None):
    import torch
    rng = np.random.default_rng(seed)
    segs_host = wl.segs_host if segs is None else segs
    nseq = len(segs_host)
    q = rng.standard_normal((nseq, q_heads, wl.D)).astype(np.float16)
    d_q = torch.from_numpy(q.view(np.int16)).cuda()
    d_segs = wl.segs if segs is None else torch.from_numpy(segs.astype(np.int32)).cuda()
    out = torch.full((nseq, q_heads, wl.D), 0x7777, dtype=torch.int32, device="cuda").to(torch.int16)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    hlkv.decode_attention(wl.hlkv_pools(), wl.layout, wl.dt.table_ptr, wl.dt.table_size,
                          wl.dt.arena_ptr, wl.dt.arena_size, d_segs, d_q, q_heads, scale, out, err)
    torch.cuda.synchronize()
    return q, out.cpu().numpy().view(np.float16).astype(np.float64), int(err.item())


@pytest.mark.parametrize("T,H,D,group", [(16, 8, 128, 4), (16, 2, 64, 1), (4, 2, 128, 8), (32, 1, 64, 2),
                                         (128, 2, 128, 4), (512, 1, 64, 2)])
def test_attention_matches_oracle(hlkv_lib, oracle, cuda_device, T, H, D, group):
    from hlkv.workload import build_workload, mixed_formats
    fm = mixed_formats(5, [3, 17, 1, 40, 9], probs=(0.25, 0.35, 0.15, 0.25), seed=T + D)
    rng = np.random.default_rng(D)
    vt = [[T] * (len(r) - 1) + [int(rng.integers(1, T + 1))] for r in fm]
    vt[1][4] = 0   # a block without valid tokens inside a sequence
    wl = build_workload(fm, T=T, H=H, D=D, seed=T * H, valid_tokens=vt)
    scale = 1.0 / np.sqrt(D)
    q, got, err = _run(hlkv_lib, wl, H * group, scale, seed=H + group)
    want, oerr = oracle_attention(oracle, wl, q.astype(np.float64), scale)
    assert err == oerr == 0
    _close(got, want, vscale=20.0)


def test_attention_empty_sequence_and_bad_blocks(hlkv_lib, oracle, cuda_device):
    """A sequence of length 0 gives zeros; a descriptor that fails kernel (1)'s checks is left
    out of its sequence with its error bit, as the oracle's gather leaves it out."""
    from hlkv.workload import build_workload
    from helpers import device_arena, device_table_words
    import torch
    T, H, D = 16, 2, 128
    wl = build_workload([[1, 3, 0], [3, 3], [0]], T=T, H=H, D=D, seed=4)
    segs = wl.segs_host.copy()
    segs[2, 1] = 0                     # empty sequence
    # make sequence 1's first block non-executable on the device (format 15)
    table = device_table_words(wl).copy()
    bid = int(device_arena(wl)[segs[1, 0]])
    table[bid, 1] = (int(table[bid, 1]) & 0xFFFFFFF0) | 15
    d_table = torch.from_numpy(table.view(np.int32).reshape(-1)).cuda()
    import hlkv
    rng = np.random.default_rng(3)
    q = rng.standard_normal((3, 2 * H, D)).astype(np.float16)
    out = torch.full((3, 2 * H, D), 0x7777, dtype=torch.int32, device="cuda").to(torch.int16)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    hlkv_lib.decode_attention(wl.hlkv_pools(), wl.layout, d_table.data_ptr(), wl.dt.table_size,
                              wl.dt.arena_ptr, wl.dt.arena_size,
                              torch.from_numpy(segs.astype(np.int32)).cuda(),
                              torch.from_numpy(q.view(np.int16)).cuda(), 2 * H, 0.125, out, err)
    torch.cuda.synchronize()
    got = out.cpu().numpy().view(np.float16).astype(np.float64)
    want, oerr = oracle_attention(oracle, wl, q.astype(np.float64), 0.125, table=table, segs=segs)
    assert int(err.item()) == oerr == 1
    assert np.all(got[2] == 0)
    _close(got, want, vscale=20.0)


def test_attention_rejects_bad_arguments(hlkv_lib, cuda_device):
    import ctypes as C
    import hlkv
    lay = hlkv.Layout(16, 8, 128, 1)
    pools = hlkv.Pools()
    L = hlkv.lib()
    err = C.c_void_p(8)
    for qh, sc, l2 in ((12, 1.0, lay), (8 * 16, 1.0, lay), (8, 0.0, lay), (8, float("inf"), lay),
                       (8, 1.0, hlkv.Layout(16, 8, 256, 1))):
        assert L.hlkv_decode_attention(C.byref(pools), C.byref(l2), None, 0, None, 0, C.c_void_p(8), 1,
                                       C.c_void_p(8), qh, sc, C.c_void_p(8), err, None) == hlkv.INVALID_ARGUMENT


@pytest.mark.parametrize("splits", [2, 3, 7, 64])
def test_split_attention_matches_oracle(hlkv_lib, oracle, cuda_device, splits):
    """Split-KV attention (partials in a caller workspace, then a merge launch) against the same
    oracle; splits beyond a sequence's block count leave empty shares."""
    import torch
    from hlkv.workload import build_workload, mixed_formats
    T, H, D, group = 16, 4, 128, 2
    fm = mixed_formats(4, [1, 23, 9, 40], probs=(0.25, 0.35, 0.15, 0.25), seed=splits)
    rng = np.random.default_rng(splits)
    vt = [[T] * (len(r) - 1) + [int(rng.integers(1, T + 1))] for r in fm]
    wl = build_workload(fm, T=T, H=H, D=D, seed=splits, valid_tokens=vt)
    qh = H * group
    q = rng.standard_normal((4, qh, D)).astype(np.float16)
    ws = torch.empty(hlkv_lib.decode_attention_workspace_bytes(4, H, D, splits), dtype=torch.uint8,
                     device="cuda")
    outs = []
    for call in range(2):  # two calls in a row on the same workspace
        out = torch.full((4, qh, D), 0x7777, dtype=torch.int32, device="cuda").to(torch.int16)
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        hlkv_lib.decode_attention_split(wl.hlkv_pools(), wl.layout, wl.dt.table_ptr, wl.dt.table_size,
                                        wl.dt.arena_ptr, wl.dt.arena_size, wl.segs,
                                        torch.from_numpy(q.view(np.int16)).cuda(), qh, 0.1, splits, ws,
                                        out, err)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        outs.append(out.cpu().numpy().view(np.float16).astype(np.float64))
    assert np.array_equal(outs[0], outs[1])
    want, oerr = oracle_attention(oracle, wl, q.astype(np.float64), 0.1)
    assert oerr == 0
    _close(outs[0], want, vscale=20.0)


def test_split_attention_workspace_checks(hlkv_lib, cuda_device):
    import ctypes as C
    import hlkv
    lay = hlkv.Layout(16, 8, 128, 1)
    pools = hlkv.Pools()
    L = hlkv.lib()
    need = hlkv_lib.decode_attention_workspace_bytes(2, 8, 128, 4)
    assert need == 2 * 8 * 4 * (16 + 8 * 128) * 4
    assert hlkv_lib.decode_attention_workspace_bytes(2, 8, 128, 1) == 0
    args = lambda splits, ws, nbytes: (C.byref(pools), C.byref(lay), None, 0, None, 0, C.c_void_p(16), 2,
                                       C.c_void_p(16), 32, 0.1, splits, ws, nbytes, C.c_void_p(16),
                                       C.c_void_p(16), None)
    assert L.hlkv_decode_attention_split(*args(4, C.c_void_p(256), need - 1)) == hlkv.BUFFER_TOO_SMALL
    assert L.hlkv_decode_attention_split(*args(4, None, need)) == hlkv.INVALID_ARGUMENT
    assert L.hlkv_decode_attention_split(*args(4, C.c_void_p(264), need)) == hlkv.INVALID_ARGUMENT
    assert L.hlkv_decode_attention_split(*args(0, C.c_void_p(256), need)) == hlkv.INVALID_ARGUMENT


@pytest.mark.parametrize("T,H,D,group", [(16, 8, 128, 4), (4, 2, 64, 2)])
def test_attention_block_wide_scales(hlkv_lib, oracle, cuda_device, T, H, D, group):
    """Blocks with block-wide parameters (scale modes 1 and 2) enter the attention with the
    values kernel (1) decodes for them; against the same float64 oracle."""
    from helpers import block_wide_scale_refs
    from hlkv.workload import build_workload, mixed_formats
    fm = mixed_formats(4, [6, 13, 2, 21], probs=(0.2, 0.35, 0.15, 0.3), seed=T + D + 1)
    rng = np.random.default_rng(D + 1)
    vt = [[T] * (len(r) - 1) + [int(rng.integers(1, T + 1))] for r in fm]
    wl = build_workload(fm, T=T, H=H, D=D, seed=T * H + 1, valid_tokens=vt)
    ids = []
    for s in wl.seqs:
        ids += wl.table.sequence_block_ids(s)[1]
    refs = block_wide_scale_refs(rng, len(ids), moderate=True)
    for k, bid in enumerate(ids):
        if k % 3 != 2:
            assert wl.table.set_scale(wl.table.handle_of(bid), *refs[k]) == 0
    wl.dt.sync(wl.table)
    scale = 1.0 / np.sqrt(D)
    q, got, err = _run(hlkv_lib, wl, H * group, scale, seed=D)
    want, oerr = oracle_attention(oracle, wl, q.astype(np.float64), scale)
    assert err == oerr == 0
    _close(got, want, vscale=40.0)


@pytest.mark.parametrize("ctas", [1, 7, 64, 592, 5000])
def test_balanced_attention_matches_oracle(hlkv_lib, oracle, cuda_device, ctas):
    """The units' blocks cut into `ctas` equal ranges (ranges end inside units and span
    several; 5000 CTAs exceed the block count, leaving empty ranges), over sequences of very
    different lengths, empty ones included: the same oracle, and two calls in a row on one
    workspace agree bit for bit."""
    import torch
    from hlkv.workload import build_workload, mixed_formats
    T, H, D, group = 16, 4, 128, 2
    lens = [3, 0, 61, 1, 17, 0, 9]
    fm = mixed_formats(len(lens), lens, probs=(0.25, 0.35, 0.15, 0.25), seed=ctas)
    rng = np.random.default_rng(ctas)
    vt = [[T] * (len(r) - 1) + [int(rng.integers(1, T + 1))] if r else [] for r in fm]
    wl = build_workload(fm, T=T, H=H, D=D, seed=ctas + 3, valid_tokens=vt)
    qh = H * group
    q = rng.standard_normal((len(lens), qh, D)).astype(np.float16)
    ws = torch.empty(hlkv_lib.decode_attention_balanced_workspace_bytes(len(lens), H, D, ctas),
                     dtype=torch.uint8, device="cuda")
    outs = []
    for call in range(2):
        out = torch.full((len(lens), qh, D), 0x7777, dtype=torch.int32, device="cuda").to(torch.int16)
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        hlkv_lib.decode_attention_balanced(wl.hlkv_pools(), wl.layout, wl.dt.table_ptr, wl.dt.table_size,
                                           wl.dt.arena_ptr, wl.dt.arena_size, wl.segs,
                                           torch.from_numpy(q.view(np.int16)).cuda(), qh, 0.1, ctas, ws,
                                           out, err)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        outs.append(out.cpu().numpy().view(np.float16).astype(np.float64))
    assert np.array_equal(outs[0], outs[1])
    want, oerr = oracle_attention(oracle, wl, q.astype(np.float64), 0.1)
    assert oerr == 0
    _close(outs[0], want, vscale=20.0)
    assert (outs[0][[1, 5]] == 0).all()  # empty sequences give zeros


def test_balanced_attention_workspace_checks(hlkv_lib, cuda_device):
    import ctypes as C
    import hlkv
    lay = hlkv.Layout(16, 8, 128, 1)
    pools = hlkv.Pools()
    L = hlkv.lib()
    need = hlkv_lib.decode_attention_balanced_workspace_bytes(2, 8, 128, 100)
    assert need == 32 + (100 + 2 * 8) * (16 + 8 * 128) * 4
    args = lambda ctas, ws, nbytes: (C.byref(pools), C.byref(lay), None, 0, None, 0, C.c_void_p(16), 2,
                                     C.c_void_p(16), 32, 0.1, ctas, ws, nbytes, C.c_void_p(16),
                                     C.c_void_p(16), None)
    assert L.hlkv_decode_attention_balanced(*args(100, C.c_void_p(256), need - 1)) == hlkv.BUFFER_TOO_SMALL
    assert L.hlkv_decode_attention_balanced(*args(100, None, need)) == hlkv.INVALID_ARGUMENT
    assert L.hlkv_decode_attention_balanced(*args(100, C.c_void_p(264), need)) == hlkv.INVALID_ARGUMENT
    assert L.hlkv_decode_attention_balanced(*args(0, C.c_void_p(256), need)) == hlkv.INVALID_ARGUMENT
    assert L.hlkv_decode_attention_balanced(*args((1 << 20) + 1, C.c_void_p(256), 1 << 40)) == hlkv.INVALID_ARGUMENT

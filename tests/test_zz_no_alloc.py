"""hlkv_decode_attention_split_noalloc: split-KV decode attention with its partials in the
library's fixed per-device scratch (HLKV_NOALLOC_SCRATCH_BYTES) instead of a caller
workspace.  Each result is compared with hlkv_decode_attention_split (caller workspace, same
splits) on two calls in a row.  Both run the same kernels on the same inputs with the same
split, so the outputs must agree bit for bit.  Head dims 64 and 128 (their partials, split
limits and merge kernels differ), each up to the largest split count the scratch holds and one
beyond it.  Collected last, and also run alone in a fresh process: the first call in the
process does the scratch set-up."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

T, H, GROUP, NSEQ = 16, 4, 2, 4


def _workload(seed, D):
    from hlkv.workload import build_workload, mixed_formats
    fm = mixed_formats(NSEQ, [1, 23, 9, 40], probs=(0.25, 0.35, 0.15, 0.25), seed=seed)
    rng = np.random.default_rng(seed)
    vt = [[T] * (len(r) - 1) + [int(rng.integers(1, T + 1))] for r in fm]
    wl = build_workload(fm, T=T, H=H, D=D, seed=seed, valid_tokens=vt)
    q = rng.standard_normal((NSEQ, H * GROUP, D)).astype(np.float16)
    return wl, q


def _largest_fitting_splits(hlkv, D):
    per_split = hlkv.decode_attention_workspace_bytes(NSEQ, H, D, 1 + 1) // 2
    return hlkv.NOALLOC_SCRATCH_BYTES // per_split


@pytest.mark.parametrize("D,limit", [(128, 252), (64, 496)])
def test_scratch_limit_matches_workspace_sizes(hlkv_lib, cuda_device, D, limit):
    """4 sequences x 4 KV heads: 4160 B of partials per CTA at head_dim 128, 2112 B at 64."""
    s = _largest_fitting_splits(hlkv_lib, D)
    assert s == limit
    assert hlkv_lib.decode_attention_workspace_bytes(NSEQ, H, D, s) <= hlkv_lib.NOALLOC_SCRATCH_BYTES
    assert hlkv_lib.decode_attention_workspace_bytes(NSEQ, H, D, s + 1) > hlkv_lib.NOALLOC_SCRATCH_BYTES


@pytest.mark.parametrize("D,splits", [(128, 1), (128, 5), (128, 252), (64, 1), (64, 7), (64, 496)])
def test_noalloc_matches_split_with_workspace(hlkv_lib, cuda_device, D, splits):
    """The largest split counts (252 at head_dim 128, 496 at 64) fill the scratch to its limit
    and leave most shares empty (a sequence has at most 40 blocks)."""
    import torch
    wl, q = _workload(splits, D)
    qh = H * GROUP
    dq = torch.from_numpy(q.view(np.int16)).cuda()
    args = (wl.hlkv_pools(), wl.layout, wl.dt.table_ptr, wl.dt.table_size, wl.dt.arena_ptr,
            wl.dt.arena_size, wl.segs, dq, qh, 0.1, splits)
    nbytes = hlkv_lib.decode_attention_workspace_bytes(NSEQ, H, D, splits)
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda") if nbytes else None
    out = torch.full((NSEQ, qh, D), 0x7777, dtype=torch.int32, device="cuda").to(torch.int16)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    hlkv_lib.decode_attention_split(*args, ws, out, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    want = out.cpu().numpy().view(np.uint16).copy()
    assert not (want == 0x7777).any()  # every output was written
    for call in range(2):  # two calls in a row through the same scratch
        out = torch.full((NSEQ, qh, D), 0x7777, dtype=torch.int32, device="cuda").to(torch.int16)
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        hlkv_lib.decode_attention_split_noalloc(*args, out, err)
        torch.cuda.synchronize()
        assert int(err.item()) == 0, call
        got = out.cpu().numpy().view(np.uint16)
        bad = np.nonzero(got != want)
        assert bad[0].size == 0, (call, bad[0].size, got[bad][:4], want[bad][:4])


@pytest.mark.parametrize("D", [128, 64])
def test_noalloc_rejects_splits_beyond_the_scratch(hlkv_lib, cuda_device, D):
    """One split more than fits: HLKV_BUFFER_TOO_SMALL, and nothing is launched."""
    import torch
    wl, q = _workload(7, D)
    qh = H * GROUP
    dq = torch.from_numpy(q.view(np.int16)).cuda()
    splits = _largest_fitting_splits(hlkv_lib, D) + 1
    out = torch.full((NSEQ, qh, D), 0x7777, dtype=torch.int32, device="cuda").to(torch.int16)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    segs = wl.segs
    st = hlkv_lib.lib().hlkv_decode_attention_split_noalloc(
        C.byref(wl.hlkv_pools()), C.byref(wl.layout), wl.dt.table_ptr or None, wl.dt.table_size,
        wl.dt.arena_ptr or None, wl.dt.arena_size, C.c_void_p(segs.data_ptr()), int(segs.shape[0]),
        C.c_void_p(dq.data_ptr()), qh, 0.1, splits, C.c_void_p(out.data_ptr()),
        C.c_void_p(err.data_ptr()), None)
    assert st == hlkv_lib.BUFFER_TOO_SMALL
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert bool((out == 0x7777).all())
    # A grid of 2^31 CTAs or more (here 2^20 sequences x 4 KV heads x 2^10 splits) is an
    # invalid argument, not a scratch overflow; nothing is launched either.
    st = hlkv_lib.lib().hlkv_decode_attention_split_noalloc(
        C.byref(wl.hlkv_pools()), C.byref(wl.layout), wl.dt.table_ptr or None, wl.dt.table_size,
        wl.dt.arena_ptr or None, wl.dt.arena_size, C.c_void_p(segs.data_ptr()), 1 << 20,
        C.c_void_p(dq.data_ptr()), qh, 0.1, 1 << 10, C.c_void_p(out.data_ptr()),
        C.c_void_p(err.data_ptr()), None)
    assert st == hlkv_lib.INVALID_ARGUMENT
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert bool((out == 0x7777).all())

"""Format-change transcode (hlkv_transcode) against the CPU oracle: every byte of every
pool after the kernel equals the oracle's transcode of the same bytes, then the committed
format changes gather to what the oracle gathers from the same tables."""
import numpy as np
import pytest

from helpers import host_pools, oracle_gather

pytestmark = pytest.mark.gpu


def _jobs_for(wl, picks):
    """begin_format_change for each (block id, target format); returns the job rows."""
    jobs = []
    for bid, target in picks:
        h = wl.table.handle_of(bid)
        assert wl.table.seal(h) in (0, 5)  # sealed now, or already sealed
        st, fc = wl.table.begin_format_change(h, target)
        assert st == 0, (bid, target, st)
        vt = (int(np.frombuffer(wl.table.lookup(h)[1], np.uint32)[1]) >> 10) & 0x3FF
        jobs.append([fc[0], fc[1], fc[2], fc[3], vt, 0, 0, 0])
    return np.array(jobs, np.uint32)


@pytest.mark.parametrize("T,H,D", [(16, 8, 128), (4, 2, 64), (2, 2, 256), (5, 3, 64), (512, 1, 128)])
def test_transcode_bit_exact_then_gather(hlkv_lib, oracle, cuda_device, T, H, D):
    import torch
    from hlkv.workload import build_workload
    fm = [[0, 1, 3, 0, 2, 1], [3, 0, 1, 1, 3], [0, 0, 2]]
    vt = [[T, T, T, T, T, max(1, T // 2)], [T, T, T, T, 1], [T, T, 0]]
    wl = build_workload(fm, T=T, H=H, D=D, seed=T * H + D, valid_tokens=vt, spare_slots=16)
    ids = []
    for s in wl.seqs:
        ids += wl.table.sequence_block_ids(s)[1]
    rng = np.random.default_rng(D)
    picks = []
    for bid in ids:
        f = int(wl.table.device_descriptor(bid)[1] & 0xF)
        picks.append((bid, int(rng.choice([t for t in (0, 1, 2, 3) if t != f]))))
    jobs = _jobs_for(wl, picks)
    before = host_pools(wl)
    d_jobs = torch.from_numpy(jobs.view(np.int32)).cuda()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    hlkv_lib.transcode(wl.hlkv_pools(), wl.layout, d_jobs, err)
    torch.cuda.synchronize()
    oerr = oracle.transcode(before, T, H, D, jobs)
    assert int(err.item()) == oerr == 0
    after = host_pools(wl)
    for f in before:
        bad = np.nonzero(after[f][0] != before[f][0])[0]
        assert bad.size == 0, f"format {f}: {bad.size} bytes differ, first at {bad[:4]}"
    # commit, bring the device tables up to date, gather through the new formats
    for bid, _ in picks:
        assert wl.table.commit_format_change(wl.table.handle_of(bid), 0, 0) == 0
    wl.dt.sync(wl.table)
    n = wl.total_blocks * wl.block_elems
    out = torch.empty(n, dtype=torch.int16, device="cuda")
    e = torch.zeros(1, dtype=torch.int32, device="cuda")
    hlkv_lib.gather_dequant(wl.hlkv_pools(), wl.layout, wl.dt.table_ptr, wl.dt.table_size,
                            wl.dt.arena_ptr, wl.dt.arena_size, wl.segs, out, e)
    torch.cuda.synchronize()
    want, gerr = oracle_gather(oracle, wl)
    assert int(e.item()) == gerr == 0
    assert np.array_equal(out.cpu().numpy().view(np.uint16), want)


def test_transcode_rejects_nonfinite_rows_and_bad_jobs(hlkv_lib, oracle, cuda_device):
    import torch
    from hlkv.workload import build_workload
    T, H, D = 4, 2, 64
    wl = build_workload([[0, 0, 1, 3]], T=T, H=H, D=D, seed=3, outlier_channels=0, spare_slots=4)
    ids = wl.table.sequence_block_ids(wl.seqs[0])[1]
    # plant an Inf and a NaN in the two FP16 blocks' payloads (through the device pool)
    buf, sb, _ = wl.pools[0]
    for bid, code in ((ids[0], 0x7C00), (ids[1], 0xFE01)):
        slot = int(wl.table.device_descriptor(bid)[0])
        buf[slot].view(torch.int16)[D * 3 + 7] = int(np.array([code], np.uint16).view(np.int16)[0])
    jobs = _jobs_for(wl, [(ids[0], 1), (ids[1], 3), (ids[2], 3)])
    bad = np.array([[1, 10 ** 6, 3, 0, T, 0, 0, 0], [7, 0, 1, 0, T, 0, 0, 0],
                    [1, 0, 3, 0, T + 1, 0, 0, 0]], np.uint32)   # slot range, bad format, valid tokens
    jobs = np.concatenate([jobs, bad])
    before = host_pools(wl)
    d_jobs = torch.from_numpy(jobs.view(np.int32)).cuda()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    hlkv_lib.transcode(wl.hlkv_pools(), wl.layout, d_jobs, err)
    torch.cuda.synchronize()
    oerr = oracle.transcode(before, T, H, D, jobs)
    assert oerr == (1 << 9) | (1 << 2) | (1 << 1) | (1 << 5)
    assert int(err.item()) == oerr
    after = host_pools(wl)
    for f in before:
        assert np.array_equal(after[f][0], before[f][0]), f


def test_transcode_from_block_wide_sources(hlkv_lib, oracle, cuda_device):
    """Source blocks with block-wide parameters (their descriptors' scale modes 1 and 2,
    passed in the job) are decoded with those parameters; a job whose source mode is 3 is
    skipped with HLKV_ERR_SCALE_MODE.  Byte-exact against the oracle, then committed (scale
    mode kNone) and gathered."""
    import torch
    from helpers import block_wide_scale_refs
    from hlkv.workload import build_workload
    T, H, D = 16, 4, 128
    fm = [[1, 3, 2, 1, 3, 3], [2, 1, 3]]
    wl = build_workload(fm, T=T, H=H, D=D, seed=17, spare_slots=16)
    ids = []
    for s in wl.seqs:
        ids += wl.table.sequence_block_ids(s)[1]
    rng = np.random.default_rng(18)
    refs = block_wide_scale_refs(rng, len(ids), moderate=True)
    modes = {}
    for k, bid in enumerate(ids):
        if k % 4 != 3:
            assert wl.table.set_scale(wl.table.handle_of(bid), *refs[k]) == 0
            modes[bid] = refs[k]
    targets = {1: 3, 2: 1, 3: 1}
    picks = [(bid, targets[int(wl.table.device_descriptor(bid)[1] & 0xF)]) for bid in ids]
    jobs = _jobs_for(wl, picks)
    for r, (bid, _) in enumerate(picks):
        jobs[r, 5], jobs[r, 6] = modes.get(bid, (0, 0))
    bad = np.array([[1, 0, 3, 0, T, 3, 7, 0]], np.uint32)  # source scale mode 3
    jobs = np.concatenate([jobs, bad])
    before = host_pools(wl)
    d_jobs = torch.from_numpy(jobs.view(np.int32)).cuda()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    hlkv_lib.transcode(wl.hlkv_pools(), wl.layout, d_jobs, err)
    torch.cuda.synchronize()
    oerr = oracle.transcode(before, T, H, D, jobs)
    assert int(err.item()) == oerr == 1 << 7
    after = host_pools(wl)
    for f in before:
        diff = np.nonzero(after[f][0] != before[f][0])[0]
        assert diff.size == 0, f"format {f}: {diff.size} bytes differ"
    for bid, _ in picks:
        assert wl.table.commit_format_change(wl.table.handle_of(bid), 0, 0) == 0
    wl.dt.sync(wl.table)
    n = wl.total_blocks * wl.block_elems
    out = torch.empty(n, dtype=torch.int16, device="cuda")
    e = torch.zeros(1, dtype=torch.int32, device="cuda")
    hlkv_lib.gather_dequant(wl.hlkv_pools(), wl.layout, wl.dt.table_ptr, wl.dt.table_size,
                            wl.dt.arena_ptr, wl.dt.arena_size, wl.segs, out, e)
    torch.cuda.synchronize()
    want, gerr = oracle_gather(oracle, wl)
    assert int(e.item()) == gerr == 0
    assert np.array_equal(out.cpu().numpy().view(np.uint16), want)

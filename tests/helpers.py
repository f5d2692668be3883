"""Shared test helpers: device copies, oracle views of a workload, comparisons."""
from __future__ import annotations

import numpy as np


def d2h(ptr: int, nbytes: int) -> np.ndarray:
    """Copies raw device memory to a host uint8 array (for pointers torch does not own)."""
    from cuda.bindings import runtime as rt
    import torch
    torch.cuda.synchronize()
    out = np.empty(max(nbytes, 1), dtype=np.uint8)
    if nbytes:
        err, = rt.cudaMemcpy(out.ctypes.data, ptr, nbytes, rt.cudaMemcpyKind.cudaMemcpyDeviceToHost)
        assert err == rt.cudaError_t.cudaSuccess, err
    return out[:nbytes]


def host_pools(wl) -> dict:
    """{fmt: (uint8 numpy array, slot_bytes, num_slots)} copies of a workload's device pools."""
    return {f: (buf.cpu().numpy().reshape(-1), sb, ns) for f, (buf, sb, ns) in wl.pools.items()}


def device_table_words(wl) -> np.ndarray:
    return d2h(wl.dt.table_ptr, wl.dt.table_size * 16).view(np.uint32).reshape(-1, 4)


def device_arena(wl) -> np.ndarray:
    return d2h(wl.dt.arena_ptr, wl.dt.arena_size * 4).view(np.uint32)


def oracle_gather(oracle, wl, out_elems: int | None = None, out_offsets=None, table=None,
                  arena=None, segs=None, fill: int = 0xABCD, threads: int = 8):
    """Runs the CPU oracle on the exact bytes the kernel reads."""
    table = device_table_words(wl) if table is None else table
    arena = device_arena(wl) if arena is None else arena
    segs = wl.segs_host if segs is None else segs
    n = out_elems if out_elems is not None else wl.total_blocks * wl.block_elems
    out = np.full(max(n, 1), fill, dtype=np.uint16)
    err = oracle.gather_dequant(host_pools(wl), wl.T, wl.H, wl.D, wl.layout.layout_id, table,
                                arena, segs, out, out_offsets, threads)
    return out[:n], err


def fp16_nan(h: np.ndarray) -> np.ndarray:
    h = h.astype(np.uint16)
    return ((h & 0x7C00) == 0x7C00) & ((h & 0x03FF) != 0)


def assert_bits_equal(got: np.ndarray, want: np.ndarray, what: str = "") -> None:
    got = np.asarray(got).view(np.uint16).reshape(-1)
    want = np.asarray(want).view(np.uint16).reshape(-1)
    assert got.shape == want.shape, (got.shape, want.shape)
    bad = np.nonzero(got != want)[0]
    if bad.size:
        i = bad[0]
        raise AssertionError(f"{what}: {bad.size} of {got.size} differ; first at {i}: "
                             f"got {got[i]:#06x} want {want[i]:#06x}")


def oracle_attention(oracle, wl, q: np.ndarray, scale: float, table=None, arena=None, segs=None):
    """Decode attention in float64 over the oracle's gather of the same tables: K and V
    are the binary16 values of the valid tokens of each block, in sequence order.
    q: float array [nseq, q_heads, D].  Returns (float64 [nseq, q_heads, D], gather error bits)."""
    table = device_table_words(wl) if table is None else table
    segs = wl.segs_host if segs is None else segs
    T, H, D = wl.T, wl.H, wl.D
    nblk = int(segs[:, 1].sum())
    out, err = oracle_gather(oracle, wl, out_elems=nblk * wl.block_elems, table=table, arena=arena,
                             segs=segs)
    blocks = out.view(np.float16).astype(np.float64).reshape(nblk, 2, T, H, D)
    arena = device_arena(wl) if arena is None else arena
    nseq, qh = q.shape[0], q.shape[1]
    g = qh // H
    res = np.zeros((nseq, qh, D))
    b0 = 0
    for i, (off, ln) in enumerate(segs):
        ks, vs = [], []
        for j in range(ln):
            pos = off + j
            ok = pos < arena.size and arena[pos] < table.shape[0]
            vt = int(table[arena[pos]][1] >> 10) & 0x3FF if ok else 0
            fmt = int(table[arena[pos]][1] & 0xF) if ok else 15
            if fmt <= 3 and vt <= T:
                ks.append(blocks[b0 + j, 0, :vt])
                vs.append(blocks[b0 + j, 1, :vt])
        b0 += ln
        if not ks:
            continue
        K = np.concatenate(ks)  # [tokens, H, D]
        V = np.concatenate(vs)
        if K.shape[0] == 0:
            continue
        for hq in range(qh):
            h = hq // g
            s = scale * (K[:, h, :] @ q[i, hq].astype(np.float64))
            p = np.exp(s - s.max())
            res[i, hq] = (p[:, None] * V[:, h, :]).sum(0) / p.sum()
    return res, err


def block_wide_scale_refs(rng, n: int, moderate: bool = False):
    """(scale_mode, scale_ref) pairs for block-wide parameters: binary32 scales (mode 1) and
    binary16 (scale, bias) pairs (mode 2).  By default they include zeros, negatives, tiny,
    huge, Inf and NaN (some of which the decoder must reject); `moderate` keeps scales in
    [-0.125, 1] with bias 0, so that codes written for per-row scales decode to finite
    binary16 values (E5M2 codes reach 57344)."""
    if moderate:
        f32 = np.array([0.25, 0.5, 0.75, 1.0, 0.375], np.float32)
        f16 = np.array([0.25, 0.5, 1.0, 0.875, -0.125, 0.0], np.float16)
    else:
        f32 = np.array([0.013, 1.0, -2.5, 0.0, -0.0, 3e-39, 1e-30, 7e4, 1e30, np.inf, np.nan, 448.0 / 17],
                       np.float32)
        f16 = np.array([0.01, 1.0, -0.75, 0.0, -0.0, 6e-8, 65504, np.inf, -np.inf, np.nan, 3.5, -100.0],
                       np.float16)
    out = []
    for _ in range(n):
        mode = int(rng.integers(1, 3))
        if mode == 1:
            ref = int(f32[rng.integers(f32.size)].view(np.uint32))
        else:
            lo = f16[rng.integers(f16.size)]
            hi = f16[rng.integers(f16.size)] if not moderate else np.float16(0.0)
            ref = int(lo.view(np.uint16)) | int(hi.view(np.uint16)) << 16
        out.append((mode, ref))
    return out

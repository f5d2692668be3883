"""CPU-built heterogeneous KV workloads for the reference arm of bench.py
(TEST INFRASTRUCTURE ONLY; no product code is involved).

kind "reference": built and gathered entirely by the reference's own code in
oracle/_ref (its HeteroBlockTable, quantize_reference and, when timed,
dequantize_reference_to_fp16 walked through its descriptor table).
kind "port": the C restatement (oracle/hlkv_oracle.c) when the reference
library is absent; descriptor table and arena are laid out directly with a
seeded permutation of ids and slots.
"""
from __future__ import annotations

import ctypes as C
import os
import time

import numpy as np

from .oracle import FP16, INT4, Oracle, Ref, packed_bytes

_FORMATS = np.array([0, 1, 2, 3], dtype=np.uint8)


def _formats(nseq: int, blocks: int, probs, seed: int) -> list:
    rng = np.random.default_rng(seed + 1)
    p = np.asarray(probs, dtype=np.float64)
    return [rng.choice(_FORMATS, size=blocks, p=p / p.sum()).astype(np.uint8) for _ in range(nseq)]


def _block_bytes(f: int, T: int, H: int, D: int) -> int:
    rows, elems = 2 * T * H, 2 * T * H * D
    params = 0 if f == FP16 else (8 * rows if f == INT4 else 4 * rows)
    return packed_bytes(f, elems) + params + 2 * elems + 20


def build_cpu_workload(kind: str, nseq: int = 0, blocks: int = 0, probs=None, seed: int = 0,
                       T: int = 16, H: int = 8, D: int = 128, outliers: int = 4, scale: float = 20.0,
                       formats: list | None = None) -> dict:
    """`formats` (one uint8 array of block formats per sequence) replaces the seeded draw of
    nseq x blocks formats from `probs`."""
    fm = [np.asarray(r, dtype=np.uint8) for r in formats] if formats is not None else \
        _formats(nseq, blocks, probs, seed)
    nseq = len(fm)
    nbytes = sum(_block_bytes(int(f), T, H, D) for row in fm for f in row)
    threads = os.cpu_count() or 1
    if kind == "reference":
        ref = Ref()
        L = ref.lib
        L.ref_workload_build.restype = C.c_void_p
        L.ref_workload_build.argtypes = [C.POINTER(C.c_uint8), C.POINTER(C.c_uint32), C.c_uint32,
                                         C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32,
                                         C.c_uint64, C.c_uint32, C.c_float, C.c_int]
        L.ref_workload_gather.restype = C.c_uint32
        L.ref_workload_gather.argtypes = [C.c_void_p, C.POINTER(C.c_uint16), C.c_int]
        L.ref_workload_free.argtypes = [C.c_void_p]
        flat = np.concatenate(fm) if fm else np.zeros(0, np.uint8)
        lens = np.array([len(r) for r in fm], dtype=np.uint32)
        h = L.ref_workload_build(flat.ctypes.data_as(C.POINTER(C.c_uint8)),
                                 lens.ctypes.data_as(C.POINTER(C.c_uint32)), nseq, T, H, D, 1,
                                 seed, outliers, scale, threads)
        out = np.empty(max(1, int(lens.sum()) * 2 * T * H * D), dtype=np.uint16)
        return {"kind": kind, "lib": L, "handle": h, "out": out, "bytes": nbytes,
                "blocks": int(lens.sum())}
    # port: the C restatement on a directly laid-out table
    orc = Oracle()
    rng = np.random.default_rng(seed)
    flat = np.concatenate(fm) if fm else np.zeros(0, np.uint8)
    total = flat.size
    rows, elems = 2 * T * H, 2 * T * H * D
    ids = rng.permutation(total).astype(np.uint32)
    table = np.zeros((total, 4), dtype=np.uint32)
    pools = {}
    for f in range(4):
        sel = np.nonzero(flat == f)[0]
        if sel.size == 0:
            continue
        slots = rng.permutation(sel.size).astype(np.uint32)
        params = 0 if f == FP16 else (8 * rows if f == INT4 else 4 * rows)
        sb = (packed_bytes(f, elems) + params + 15) // 16 * 16
        buf = np.zeros((sel.size, sb), dtype=np.uint8)
        x = orc.gaussian(seed * 7 + f, sel.size * elems).reshape(sel.size, elems)
        x = x.astype(np.float16).astype(np.float32)
        for s in range(sel.size):
            st, p, codes = orc.quantize(f, x[s], 0 if f == FP16 else D)
            assert st == 0
            cb = codes.size
            buf[s, :cb] = codes
            if f == INT4:
                buf[s, cb:cb + 8 * rows] = p.view(np.uint8).reshape(-1)
            elif f != FP16:
                buf[s, cb:cb + 4 * rows] = p[:, 0].copy().view(np.uint8)
        pools[f] = (buf.reshape(-1), sb, sel.size)
        for k, b in enumerate(sel):
            table[ids[b]] = (slots[k], f | (1 << 6) | (T << 10), 0, ids[b])
    arena = ids.copy()
    lens = np.array([len(r) for r in fm], dtype=np.uint32)
    segs = np.stack([np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.uint32), lens], axis=1)
    out = np.empty(max(1, total * elems), dtype=np.uint16)
    return {"kind": kind, "oracle": orc, "pools": pools, "table": table, "arena": arena,
            "segs": segs, "T": T, "H": H, "D": D, "out": out, "bytes": nbytes, "blocks": total}


def time_cpu_gather(wl: dict, threads: int) -> tuple[float, int]:
    """One gather over the workload; returns (wall seconds, error bits)."""
    t0 = time.perf_counter()
    if wl["kind"] == "reference":
        err = wl["lib"].ref_workload_gather(wl["handle"], wl["out"].ctypes.data_as(C.POINTER(C.c_uint16)),
                                            threads)
    else:
        err = wl["oracle"].gather_dequant(wl["pools"], wl["T"], wl["H"], wl["D"], 1, wl["table"],
                                          wl["arena"], wl["segs"], wl["out"], threads=threads)
    return time.perf_counter() - t0, int(err)

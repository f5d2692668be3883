"""ctypes bindings to the oracle libraries (TEST INFRASTRUCTURE ONLY).

``Oracle`` binds ``oracle/_build/liboracle.so`` (the C restatement in
hlkv_oracle.c); ``Ref`` binds ``oracle/_ref/libhlkv_ref.so`` (the reference's
own CPU library compiled from its sources, plus ref_shim.cpp).  Both expose
the same numpy-level calls so tests can run one against the other.  Only
tests/, __graft_entry__.smoke() and the cpu_baseline leg of bench.py import
this module.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import build as _build

u8p = C.POINTER(C.c_uint8)
u16p = C.POINTER(C.c_uint16)
u32p = C.POINTER(C.c_uint32)
u64p = C.POINTER(C.c_uint64)
f32p = C.POINTER(C.c_float)

FP16, E4M3, E5M2, INT4 = 0, 1, 2, 3


class Pool(C.Structure):
    """One payload pool: base pointer, bytes per slot, number of slots."""
    _fields_ = [("base", C.c_void_p), ("slot_bytes", C.c_uint64), ("num_slots", C.c_uint32),
                ("pad", C.c_uint32)]


def _p(a: np.ndarray, t):
    return a.ctypes.data_as(t)


def packed_bytes(fmt: int, n: int) -> int:
    if fmt == FP16:
        return 2 * n
    if fmt == INT4:
        return n // 2 + n % 2
    return n


def num_groups(n: int, g: int) -> int:
    return 0 if g == 0 else -(-n // g)


def _pool_array(pools: dict):
    parr = (Pool * 15)()
    keep = []
    for f, (buf, slot_bytes, num_slots) in pools.items():
        if not (isinstance(buf, np.ndarray) and buf.flags.c_contiguous):
            buf = np.ascontiguousarray(buf)
        keep.append(buf)
        parr[f].base = buf.ctypes.data
        parr[f].slot_bytes = slot_bytes
        parr[f].num_slots = num_slots
    return parr, keep


class _Common:
    prefix = ""

    def __init__(self, path: str):
        self.lib = C.CDLL(path)
        L, p = self.lib, self.prefix
        getattr(L, p + "encode_array").argtypes = [C.c_int, f32p, C.c_size_t, u16p]
        getattr(L, p + "decode_array").argtypes = [C.c_int, u16p, C.c_size_t, f32p]
        f = getattr(L, p + "quantize")
        f.argtypes = [C.c_int, f32p, C.c_size_t, C.c_size_t, f32p, C.c_size_t, u8p, C.c_size_t]
        f.restype = C.c_int
        f = getattr(L, p + "dequantize")
        f.argtypes = [C.c_int, u8p, C.c_size_t, C.c_size_t, f32p, C.c_size_t, C.c_size_t, f32p,
                      C.c_size_t]
        f.restype = C.c_int
        f = getattr(L, p + "dequantize_to_fp16")
        f.argtypes = [C.c_int, u8p, C.c_size_t, C.c_size_t, f32p, C.c_size_t, C.c_size_t, u16p,
                      C.c_size_t]
        f.restype = C.c_int
        f = getattr(L, p + "gather_dequant")
        f.argtypes = [C.POINTER(Pool), C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, u32p,
                      C.c_uint32, u32p, C.c_uint32, u32p, C.c_uint32, u64p, u16p, u64p, C.c_int]
        f.restype = C.c_uint32
        f = getattr(L, p + "quantize_rows")
        f.argtypes = [u8p, f32p, C.c_size_t, C.c_size_t, f32p, u8p, C.c_int]
        f.restype = C.c_size_t

    def quantize_rows(self, fmt: np.ndarray, x: np.ndarray, params: np.ndarray, codes: np.ndarray,
                      threads: int = 1) -> int:
        """quantize_reference per row of x [rows, D] (row r in format fmt[r], one group per
        row) into params [rows, 2] and codes [rows, D] (packed bytes at the row start), over
        `threads` threads; returns the number of rejected rows."""
        rows, D = x.shape
        fm = np.ascontiguousarray(fmt, dtype=np.uint8)
        assert x.dtype == np.float32 and x.flags.c_contiguous and fm.size == rows
        assert params.shape == (rows, 2) and codes.shape == (rows, D)
        return int(getattr(self.lib, self.prefix + "quantize_rows")(
            _p(fm, u8p), _p(x, f32p), rows, D, _p(params, f32p), _p(codes, u8p), threads))

    # -- codecs -------------------------------------------------------------------------
    def encode(self, fmt: int, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty(x.size, dtype=np.uint16)
        getattr(self.lib, self.prefix + "encode_array")(fmt, _p(x, f32p), x.size, _p(out, u16p))
        return out

    def decode(self, fmt: int, codes: np.ndarray) -> np.ndarray:
        c = np.ascontiguousarray(codes, dtype=np.uint16)
        out = np.empty(c.size, dtype=np.float32)
        getattr(self.lib, self.prefix + "decode_array")(fmt, _p(c, u16p), c.size, _p(out, f32p))
        return out

    def quantize(self, fmt: int, x: np.ndarray, group: int, n_params: int | None = None,
                 packed_size: int | None = None, params_init: float = 0.0, packed_init: int = 0):
        """Returns (status, params[n,2] float32, packed uint8)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        n = x.size
        if n_params is None:
            n_params = num_groups(n, group)
        if packed_size is None:
            packed_size = packed_bytes(fmt, n)
        params = np.full((max(n_params, 1), 2), params_init, dtype=np.float32)
        packed = np.full(max(packed_size, 1), packed_init, dtype=np.uint8)
        st = getattr(self.lib, self.prefix + "quantize")(fmt, _p(x, f32p), n, group,
                                                         _p(params, f32p), n_params,
                                                         _p(packed, u8p), packed_size)
        return st, params[:n_params], packed[:packed_size]

    def dequantize(self, fmt: int, packed: np.ndarray, n: int, params: np.ndarray, group: int,
                   out_size: int | None = None):
        packed = np.ascontiguousarray(packed, dtype=np.uint8)
        params = np.ascontiguousarray(params, dtype=np.float32).reshape(-1, 2)
        m = n if out_size is None else out_size
        out = np.full(max(m, 1), np.float32(7.0), np.float32)
        st = getattr(self.lib, self.prefix + "dequantize")(
            fmt, _p(packed, u8p), packed.size, n, _p(params, f32p), params.shape[0], group,
            _p(out, f32p), m)
        return st, out[:m]

    def dequantize_to_fp16(self, fmt: int, packed: np.ndarray, n: int, params: np.ndarray,
                           group: int, out_size: int | None = None):
        packed = np.ascontiguousarray(packed, dtype=np.uint8)
        params = np.ascontiguousarray(params, dtype=np.float32).reshape(-1, 2)
        m = n if out_size is None else out_size
        out = np.full(max(m, 1), 0xFFFF, np.uint16)
        st = getattr(self.lib, self.prefix + "dequantize_to_fp16")(
            fmt, _p(packed, u8p), packed.size, n, _p(params, f32p), params.shape[0], group,
            _p(out, u16p), m)
        return st, out[:m]

    # -- the block path -----------------------------------------------------------------
    def gather_dequant(self, pools: dict, T: int, H: int, D: int, layout_id: int,
                       table: np.ndarray, arena: np.ndarray, segs: np.ndarray,
                       out: np.ndarray, out_offsets: np.ndarray | None = None,
                       threads: int = 1) -> int:
        """pools: {format: (uint8 array num_slots*slot_bytes, slot_bytes, num_slots)}.

        table: uint32 [n,4]; arena: uint32; segs: uint32 [nseq,2]; out: uint16 (modified).
        Returns the OR of the error bits.
        """
        parr, keep = _pool_array(pools)
        table = np.ascontiguousarray(table, dtype=np.uint32).reshape(-1)
        arena = np.ascontiguousarray(arena, dtype=np.uint32).reshape(-1)
        segs = np.ascontiguousarray(segs, dtype=np.uint32).reshape(-1, 2)
        nseq = segs.shape[0]
        prefix = np.zeros(nseq + 1, dtype=np.uint64)
        prefix[1:] = np.cumsum(segs[:, 1].astype(np.uint64))
        offs = None
        if out_offsets is not None:
            offs = np.ascontiguousarray(out_offsets, dtype=np.uint64)
        assert out.dtype == np.uint16 and out.flags.c_contiguous
        return getattr(self.lib, self.prefix + "gather_dequant")(
            parr, T, H, D, layout_id, _p(table, u32p) if table.size else None, table.size // 4,
            _p(arena, u32p) if arena.size else None, arena.size,
            _p(segs.reshape(-1), u32p) if segs.size else None, nseq,
            _p(offs, u64p) if offs is not None else None, _p(out, u16p), _p(prefix, u64p),
            threads)


class Oracle(_Common):
    """The C restatement (hlkv_oracle.c)."""
    prefix = "orc_"

    def __init__(self):
        super().__init__(_build.build_oracle())
        L = self.lib
        L.orc_apply_delta.argtypes = [u32p, C.c_uint32, u32p, C.c_uint32, u32p, C.c_uint32, u32p,
                                      C.c_uint32]
        L.orc_apply_delta.restype = C.c_uint32
        L.orc_append_encode.argtypes = [C.POINTER(Pool), C.c_uint32, C.c_uint32, C.c_uint32,
                                        C.c_uint32, u32p, C.c_uint32, u32p, C.c_uint32, u16p]
        L.orc_append_encode.restype = C.c_uint32
        L.orc_transcode.argtypes = [C.POINTER(Pool), C.c_uint32, C.c_uint32, C.c_uint32, u32p,
                                    C.c_uint32]
        L.orc_transcode.restype = C.c_uint32
        L.orc_gaussian.argtypes = [C.c_uint64, C.c_float, f32p, C.c_size_t]
        L.orc_slot_bytes_needed.argtypes = [C.c_int, C.c_uint32, C.c_uint32, C.c_uint32]
        L.orc_slot_bytes_needed.restype = C.c_size_t

    def gaussian(self, seed: int, n: int, sigma: float = 1.0) -> np.ndarray:
        out = np.empty(n, dtype=np.float32)
        self.lib.orc_gaussian(seed, sigma, _p(out, f32p), n)
        return out

    def slot_bytes_needed(self, fmt: int, T: int, H: int, D: int) -> int:
        return self.lib.orc_slot_bytes_needed(fmt, T, H, D)

    def apply_delta(self, table: np.ndarray, arena: np.ndarray, desc_patches: np.ndarray,
                    id_patches: np.ndarray) -> int:
        """In-place scatter of the patches into table (uint32 [n,4]) and arena (uint32)."""
        assert table.dtype == np.uint32 and arena.dtype == np.uint32
        assert table.flags.c_contiguous and arena.flags.c_contiguous
        dp = np.ascontiguousarray(desc_patches, dtype=np.uint32).reshape(-1)
        ip = np.ascontiguousarray(id_patches, dtype=np.uint32).reshape(-1)
        return self.lib.orc_apply_delta(
            _p(table, u32p) if table.size else None, table.size // 4,
            _p(arena, u32p) if arena.size else None, arena.size,
            _p(dp, u32p) if dp.size else None, dp.size // 4,
            _p(ip, u32p) if ip.size else None, ip.size // 2)

    def append_encode(self, pools: dict, T: int, H: int, D: int, layout_id: int,
                      table: np.ndarray, targets: np.ndarray, tokens: np.ndarray) -> int:
        """pools as in gather_dequant; the uint8 arrays are modified in place."""
        for buf, _, _ in pools.values():
            assert buf.flags.c_contiguous and buf.dtype == np.uint8
        parr, keep = _pool_array(pools)
        table = np.ascontiguousarray(table, dtype=np.uint32).reshape(-1)
        tg = np.ascontiguousarray(targets, dtype=np.uint32).reshape(-1)
        tok = np.ascontiguousarray(tokens, dtype=np.uint16).reshape(-1)
        return self.lib.orc_append_encode(parr, T, H, D, layout_id, _p(table, u32p),
                                          table.size // 4, _p(tg, u32p) if tg.size else None,
                                          tg.size // 2, _p(tok, u16p) if tok.size else None)


    def transcode(self, pools: dict, T: int, H: int, D: int, jobs: np.ndarray) -> int:
        """jobs: uint32 [n, 8] = {from_format, from_slot, to_format, to_slot, valid_tokens,
        0, 0, 0}; the pool arrays are modified in place.  Returns the error bits."""
        for buf, _, _ in pools.values():
            assert buf.flags.c_contiguous and buf.dtype == np.uint8
        parr, keep = _pool_array(pools)
        j = np.ascontiguousarray(jobs, dtype=np.uint32).reshape(-1)
        return self.lib.orc_transcode(parr, T, H, D, _p(j, u32p) if j.size else None, j.size // 8)


class Ref(_Common):
    """The reference's own CPU library, compiled from its sources (oracle/_ref)."""
    prefix = "ref_"

    def __init__(self, path: str | None = None):
        path = path or _build.build_ref()
        if path is None or not os.path.exists(path):
            raise FileNotFoundError("oracle/_ref/libhlkv_ref.so is not built")
        super().__init__(path)


def table_trace(lib: C.CDLL, seed: int, steps: int, max_blocks: int = 96,
                slots: tuple[int, int, int] = (48, 48, 64)) -> np.ndarray:
    """Runs table_trace_run from a library (reference or this repository's build)."""
    lib.table_trace_run.argtypes = [C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32,
                                    C.c_uint32, u32p, C.c_size_t]
    lib.table_trace_run.restype = C.c_size_t
    n = lib.table_trace_run(seed, steps, max_blocks, *slots, None, 0)
    out = np.empty(n, dtype=np.uint32)
    lib.table_trace_run(seed, steps, max_blocks, *slots, _p(out, u32p), n)
    return out


def ref_available() -> bool:
    return os.path.exists(_build.REF_SO) or _build.reference_available()


class RefCuda:
    """The reference's own GPU kernel hl::quant::cuda::dequantize_fp8_to_fp16, compiled
    from its sources for sm_100a (oracle/_ref/libhlkv_ref_cuda.so)."""

    def __init__(self, path: str | None = None):
        path = path or _build.build_ref_cuda()
        if path is None or not os.path.exists(path):
            raise FileNotFoundError("oracle/_ref/libhlkv_ref_cuda.so is not built")
        self.lib = C.CDLL(path)
        f = self.lib.ref_cuda_dequantize_fp8_to_fp16
        f.argtypes = [C.c_int, C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t, C.c_void_p,
                      C.c_void_p, C.POINTER(C.c_int)]
        f.restype = C.c_int

    def dequantize_fp8_to_fp16(self, fmt: int, d_in: int, n: int, d_params: int, group: int,
                               d_out: int, stream: int | None = None) -> int:
        e = C.c_int(0)
        st = self.lib.ref_cuda_dequantize_fp8_to_fp16(fmt, d_in, n, d_params, group, d_out, stream,
                                                      C.byref(e))
        self.last_cuda_error = e.value
        return st


def ref_cuda_available() -> bool:
    p = _build.REF_CUDA_SO
    return os.path.exists(p) or _build.build_ref_cuda() is not None

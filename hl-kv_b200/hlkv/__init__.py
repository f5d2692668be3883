"""hlkv: Python binding of libhlkv.so, the HL-KV quantized KV-block path on B200.

Everything here goes through the C ABI of ``include/hlkv.h``.  PyTorch is only
the device-memory and stream plumbing (tensors are passed by ``data_ptr()``,
streams by their CUDA handle).  The CUDA kernels live in ``libhlkv.so`` and
nothing falls back to the CPU: when the library is missing or a CUDA call
fails, the call raises.

Module layout mirrors the reference's host API:
  * :class:`Table` -- hl::alloc::HeteroBlockTable (statuses as ``Status`` ints);
  * :class:`DeviceTables` -- the persistent device descriptor table + id arena;
  * :func:`gather_dequant`, :func:`append_encode`, :func:`apply_delta` -- kernels (1)-(3);
  * :func:`dequantize_fp8_to_fp16`, :func:`dequantize_to_fp16`, :func:`quantize` -- flat codecs.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass
from typing import Mapping, Sequence

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libhlkv.so")

# ---- constants (include/hlkv.h) --------------------------------------------------------------
FP16, FP8_E4M3, FP8_E5M2, INT4, INVALID_FORMAT = 0, 1, 2, 3, 15
OK, INVALID_ARGUMENT, BUFFER_TOO_SMALL, UNSUPPORTED_FORMAT, CUDA_ERROR = 0, 1, 2, 3, 4

ERR_NOT_EXECUTABLE = 1 << 0
ERR_BAD_FORMAT = 1 << 1
ERR_SLOT_RANGE = 1 << 2
ERR_ARENA_RANGE = 1 << 3
ERR_BLOCK_ID_RANGE = 1 << 4
ERR_VALID_TOKENS = 1 << 5
ERR_LAYOUT = 1 << 6
ERR_SCALE_MODE = 1 << 7
ERR_DESC_MISMATCH = 1 << 8
ERR_NONFINITE = 1 << 9
ERR_TOKEN_RANGE = 1 << 10
ERR_PATCH_RANGE = 1 << 11
ERR_OUT_ALIGN = 1 << 12


class Status:
    """hl::alloc::Status values (status.hpp)."""
    OK = 0
    OUT_OF_BLOCKS = 1
    OUT_OF_SLOTS = 2
    INVALID_HANDLE = 3
    STALE_HANDLE = 4
    INVALID_STATE = 5
    INVALID_ARGUMENT = 6
    UNKNOWN_FORMAT = 7
    NOT_DEVICE_RESIDENT = 8
    REFCOUNT_OVERFLOW = 9
    CORRUPT = 10
    CAPACITY_EXCEEDED = 11


class ScaleMode:
    NONE, INLINE_F32, INLINE_F16_PAIR, EXTERNAL = 0, 1, 2, 3


class Residency:
    DEVICE, HOST, DROPPED = 0, 1, 2


# ---- C structs ----------------------------------------------------------------------------------
class ExecDescriptor(C.Structure):
    _fields_ = [("slot", C.c_uint32), ("info", C.c_uint32), ("scale_ref", C.c_uint32),
                ("block_id", C.c_uint32)]


class IdPatch(C.Structure):
    _fields_ = [("offset", C.c_uint32), ("block_id", C.c_uint32)]


class Segment(C.Structure):
    _fields_ = [("offset", C.c_uint32), ("length", C.c_uint32)]


class Pool(C.Structure):
    _fields_ = [("base", C.c_void_p), ("slot_bytes", C.c_uint64), ("num_slots", C.c_uint32),
                ("reserved", C.c_uint32)]


class Pools(C.Structure):
    _fields_ = [("pool", Pool * 15)]


class Layout(C.Structure):
    _fields_ = [("block_tokens", C.c_uint32), ("kv_heads", C.c_uint32), ("head_dim", C.c_uint32),
                ("layout_id", C.c_uint32)]


class PoolConfig(C.Structure):
    _fields_ = [("format", C.c_uint32), ("slot_bytes", C.c_uint32), ("num_slots", C.c_uint32)]


class TableConfig(C.Structure):
    _fields_ = [("max_blocks", C.c_uint32), ("block_tokens", C.c_uint32),
                ("num_pools", C.c_uint32), ("pools", C.POINTER(PoolConfig))]


class AllocRequest(C.Structure):
    _fields_ = [("format", C.c_uint32), ("valid_tokens", C.c_uint32), ("layout", C.c_uint32),
                ("scale_mode", C.c_uint32), ("scale_ref", C.c_uint32)]


class Handle(C.Structure):
    _fields_ = [("id", C.c_uint32), ("generation", C.c_uint32)]

    def __repr__(self) -> str:
        return f"Handle({self.id}, {self.generation})"

    def __eq__(self, other) -> bool:
        return isinstance(other, Handle) and (self.id, self.generation) == (other.id, other.generation)

    def __hash__(self) -> int:
        return hash((self.id, self.generation))


INVALID_HANDLE = Handle(0xFFFFFFFF, 0)

_vp, _u32, _u64, _sz, _int = C.c_void_p, C.c_uint32, C.c_uint64, C.c_size_t, C.c_int
_P = C.POINTER

# (name, restype, argtypes) for every entry point of include/hlkv.h.
SIGNATURES: list[tuple[str, object, list]] = [
    ("hlkv_layout_slot_bytes", _u64, [_int, _P(Layout)]),
    ("hlkv_last_cuda_error", _int, []),
    ("hlkv_gather_dequant", _int, [_P(Pools), _P(Layout), _vp, _u32, _vp, _u32, _vp, _u32, _vp,
                                   _vp, _vp, _vp]),
    ("hlkv_gather_dequant_ex", _int, [_P(Pools), _P(Layout), _vp, _u32, _vp, _u32, _vp, _u32, _vp,
                                      _vp, _vp, _u32, _vp]),
    ("hlkv_decode_attention", _int, [_P(Pools), _P(Layout), _vp, _u32, _vp, _u32, _vp, _u32, _vp,
                                     _u32, C.c_float, _vp, _vp, _vp]),
    ("hlkv_decode_attention_workspace_bytes", _sz, [_u32, _u32, _u32, _u32]),
    ("hlkv_decode_attention_split", _int, [_P(Pools), _P(Layout), _vp, _u32, _vp, _u32, _vp, _u32, _vp,
                                           _u32, C.c_float, _u32, _vp, _sz, _vp, _vp, _vp]),
    ("hlkv_decode_attention_balanced_workspace_bytes", _sz, [_u32, _u32, _u32, _u32]),
    ("hlkv_decode_attention_balanced", _int, [_P(Pools), _P(Layout), _vp, _u32, _vp, _u32, _vp, _u32, _vp,
                                              _u32, C.c_float, _u32, _vp, _sz, _vp, _vp, _vp]),
    ("hlkv_decode_attention_split_noalloc", _int, [_P(Pools), _P(Layout), _vp, _u32, _vp, _u32, _vp,
                                                   _u32, _vp, _u32, C.c_float, _u32, _vp, _vp, _vp]),
    ("hlkv_transcode", _int, [_P(Pools), _P(Layout), _vp, _u32, _vp, _vp]),
    ("hlkv_append_encode", _int, [_P(Pools), _P(Layout), _vp, _u32, _vp, _u32, _vp, _vp, _vp]),
    ("hlkv_apply_delta", _int, [_vp, _u32, _vp, _u32, _vp, _u32, _vp, _u32, _vp, _vp]),
    ("hlkv_dequantize_fp8_to_fp16", _int, [_int, _vp, _sz, _vp, _sz, _vp, _vp]),
    ("hlkv_dequantize_to_fp16", _int, [_int, _vp, _sz, _sz, _vp, _sz, _sz, _vp, _sz, _vp, _vp]),
    ("hlkv_quantize", _int, [_int, _vp, _sz, _sz, _vp, _sz, _vp, _sz, _vp, _vp]),
    ("hlkv_table_validate_config", _int, [_P(TableConfig)]),
    ("hlkv_table_create", _int, [_P(TableConfig), _P(_vp)]),
    ("hlkv_table_destroy", None, [_vp]),
    ("hlkv_table_snapshot", _int, [_vp, _vp, _sz, _P(_sz)]),
    ("hlkv_table_restore", _int, [_vp, _sz, _P(_vp)]),
    ("hlkv_table_allocate", _int, [_vp, _P(AllocRequest), _P(Handle)]),
    ("hlkv_table_retain", _int, [_vp, Handle]),
    ("hlkv_table_release", _int, [_vp, Handle]),
    ("hlkv_table_set_valid_tokens", _int, [_vp, Handle, _u32]),
    ("hlkv_table_seal", _int, [_vp, Handle]),
    ("hlkv_table_set_residency", _int, [_vp, Handle, _u32]),
    ("hlkv_table_set_scale", _int, [_vp, Handle, _u32, _u32]),
    ("hlkv_table_begin_format_change", _int, [_vp, Handle, _u32, _P(_u32)]),
    ("hlkv_table_commit_format_change", _int, [_vp, Handle, _u32, _u32]),
    ("hlkv_table_abort_format_change", _int, [_vp, Handle]),
    ("hlkv_table_lookup", _int, [_vp, Handle, _vp]),
    ("hlkv_table_lookup_batch", _int, [_vp, _P(Handle), _sz, _P(ExecDescriptor), _sz]),
    ("hlkv_table_handle_of", Handle, [_vp, _u32]),
    ("hlkv_table_create_sequence", _int, [_vp, _P(Handle)]),
    ("hlkv_table_append_block", _int, [_vp, Handle, _P(AllocRequest), _P(Handle)]),
    ("hlkv_table_append_shared_block", _int, [_vp, Handle, Handle]),
    ("hlkv_table_release_sequence", _int, [_vp, Handle]),
    ("hlkv_table_sequence_block_ids", _int, [_vp, Handle, _P(_u32), _sz, _P(_sz)]),
    ("hlkv_table_batch_segments", _int, [_vp, _P(Handle), _sz, _P(Segment)]),
    ("hlkv_table_append_tokens", _int, [_vp, _P(Handle), _sz, _P(_u32), _u32, _vp, _P(_sz)]),
    ("hlkv_table_build_exec_table", _int, [_vp, _P(Handle), _sz, _P(_u32), _P(ExecDescriptor),
                                           _sz, _P(_sz)]),
    ("hlkv_table_pending", None, [_vp, _P(_sz), _P(_sz)]),
    ("hlkv_table_collect_delta", _int, [_vp, _P(ExecDescriptor), _sz, _P(IdPatch), _sz,
                                        _P(_sz), _P(_sz), _P(_u32), _P(_u32)]),
    ("hlkv_table_device_descriptor", ExecDescriptor, [_vp, _u32]),
    ("hlkv_table_block_tokens", _u32, [_vp]),
    ("hlkv_table_max_blocks", _u32, [_vp]),
    ("hlkv_table_blocks_in_use", _u32, [_vp]),
    ("hlkv_table_has_pool", _int, [_vp, _u32]),
    ("hlkv_table_free_slots", _u32, [_vp, _u32]),
    ("hlkv_table_pool_slots", _u32, [_vp, _u32]),
    ("hlkv_table_slot_bytes", _u32, [_vp, _u32]),
    ("hlkv_table_stats", None, [_vp, _P(_u64)]),
    ("hlkv_table_validate", _int, [_vp, C.c_char_p, _sz]),
    ("hlkv_device_tables_create", _int, [_P(_vp)]),
    ("hlkv_device_tables_destroy", None, [_vp]),
    ("hlkv_device_tables_sync", _int, [_vp, _vp, _vp]),
    ("hlkv_device_tables_collect", _int, [_vp, _vp]),
    ("hlkv_device_tables_flush", _int, [_vp, _vp]),
    ("hlkv_decode_step_queue", _int, [_vp, _P(Pools), _P(Layout), _vp, _vp, _u32, _vp, _vp, _vp, _vp, _vp]),
    ("hlkv_table_compact_arena", _int, [_vp, _vp, _sz, _P(_sz)]),
    ("hlkv_segment_moves_scratch_entries", _u64, [_vp, _sz]),
    ("hlkv_arena_relocate", _int, [_vp, _u32, _vp, _u32, _vp, _u64, _vp, _vp]),
    ("hlkv_device_tables_relocate", _int, [_vp, _vp, _sz, _u32, _vp]),
    ("hlkv_device_tables_arena_capacity_bytes", _u64, [_vp]),
    ("hlkv_device_tables_table", _vp, [_vp]),
    ("hlkv_device_tables_table_size", _u32, [_vp]),
    ("hlkv_device_tables_arena", _vp, [_vp]),
    ("hlkv_device_tables_arena_size", _u32, [_vp]),
    ("hlkv_device_tables_error_word", _vp, [_vp]),
]

_lib: C.CDLL | None = None


def lib() -> C.CDLL:
    """Loads libhlkv.so (once).  Raises when it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with python hl-kv_b200/build.py")
        L = C.CDLL(LIB_PATH)
        for name, res, args in SIGNATURES:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


class HlkvError(RuntimeError):
    pass


def check_table(status: int, what: str) -> None:
    """Raises on a non-OK table status."""
    if status != Status.OK:
        raise HlkvError(f"{what}: table status {status}")


def check(status: int, what: str) -> None:
    """Raises on a non-OK device status (with the CUDA error for CUDA_ERROR)."""
    if status != OK:
        extra = f" (cudaError {lib().hlkv_last_cuda_error()})" if status == CUDA_ERROR else ""
        raise HlkvError(f"{what}: status {status}{extra}")


# ---- ABI helpers --------------------------------------------------------------------------------
def pack_info(fmt: int, scale_mode: int, layout: int, valid_tokens: int) -> int:
    """BlockExecDescriptor::pack_info (block_descriptor.hpp:152-162)."""
    return (fmt & 0xF) | ((scale_mode & 3) << 4) | ((layout & 0xF) << 6) | ((valid_tokens & 0x3FF) << 10)


def layout_slot_bytes(fmt: int, layout: Layout) -> int:
    return int(lib().hlkv_layout_slot_bytes(fmt, C.byref(layout)))


def _stream_handle(stream) -> int | None:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def _ptr(t) -> int | None:
    return None if t is None else int(t.data_ptr())


# ---- host table -----------------------------------------------------------------------------------
@dataclass
class Delta:
    descriptor_patches: "object"  # numpy uint32 [n, 4]
    id_patches: "object"          # numpy uint32 [n, 2]
    descriptor_table_size: int
    arena_size: int


class Table:
    """hl::alloc::HeteroBlockTable through the C ABI.  Methods return Status ints
    (and handles/values where the C++ call returns a Result)."""

    def __init__(self, max_blocks: int, pools: Sequence[tuple[int, int, int]], block_tokens: int = 16):
        arr = (PoolConfig * max(len(pools), 1))(*[PoolConfig(f, sb, ns) for f, sb, ns in pools])
        self._keep = arr
        cfg = TableConfig(max_blocks, block_tokens, len(pools), C.cast(arr, _P(PoolConfig)))
        h = _vp()
        st = lib().hlkv_table_create(C.byref(cfg), C.byref(h))
        if st != Status.OK:
            raise ValueError(f"invalid TableConfig: status {st}")
        self.h = h

    @staticmethod
    def validate_config(max_blocks: int, pools: Sequence[tuple[int, int, int]], block_tokens: int = 16) -> int:
        arr = (PoolConfig * max(len(pools), 1))(*[PoolConfig(f, sb, ns) for f, sb, ns in pools])
        cfg = TableConfig(max_blocks, block_tokens, len(pools), C.cast(arr, _P(PoolConfig)))
        return lib().hlkv_table_validate_config(C.byref(cfg))

    def snapshot(self) -> bytes:
        """The table's versioned binary image (hlkv_table_snapshot)."""
        n = _sz()
        check_table(lib().hlkv_table_snapshot(self.h, None, 0, C.byref(n)), "hlkv_table_snapshot")
        buf = (C.c_char * max(n.value, 1))()
        check_table(lib().hlkv_table_snapshot(self.h, buf, n.value, C.byref(n)), "hlkv_table_snapshot")
        return bytes(buf[:n.value])

    @classmethod
    def restore(cls, image: bytes) -> tuple[int, "Table | None"]:
        """(status, table rebuilt from a snapshot image, or None) -- hlkv_table_restore."""
        h = _vp()
        st = lib().hlkv_table_restore(image, len(image), C.byref(h))
        if st != Status.OK:
            return st, None
        t = cls.__new__(cls)
        t._keep = None
        t.h = h
        return st, t

    def close(self) -> None:
        if getattr(self, "h", None):
            lib().hlkv_table_destroy(self.h)
            self.h = None

    __del__ = close

    # blocks
    def allocate(self, fmt: int, valid_tokens: int = 0, layout: int = 1, scale_mode: int = 0,
                 scale_ref: int = 0) -> tuple[int, Handle]:
        out = Handle()
        req = AllocRequest(fmt, valid_tokens, layout, scale_mode, scale_ref)
        st = lib().hlkv_table_allocate(self.h, C.byref(req), C.byref(out))
        return st, out

    def retain(self, b: Handle) -> int: return lib().hlkv_table_retain(self.h, b)
    def release(self, b: Handle) -> int: return lib().hlkv_table_release(self.h, b)
    def set_valid_tokens(self, b: Handle, n: int) -> int: return lib().hlkv_table_set_valid_tokens(self.h, b, n)
    def seal(self, b: Handle) -> int: return lib().hlkv_table_seal(self.h, b)
    def set_residency(self, b: Handle, r: int) -> int: return lib().hlkv_table_set_residency(self.h, b, r)
    def set_scale(self, b: Handle, mode: int, ref: int) -> int: return lib().hlkv_table_set_scale(self.h, b, mode, ref)

    def begin_format_change(self, b: Handle, target: int) -> tuple[int, tuple[int, int, int, int]]:
        out = (_u32 * 4)()
        st = lib().hlkv_table_begin_format_change(self.h, b, target, out)
        return st, tuple(out)

    def commit_format_change(self, b: Handle, mode: int = 0, ref: int = 0) -> int:
        return lib().hlkv_table_commit_format_change(self.h, b, mode, ref)

    def abort_format_change(self, b: Handle) -> int:
        return lib().hlkv_table_abort_format_change(self.h, b)

    def lookup(self, b: Handle) -> tuple[int, bytes]:
        buf = C.create_string_buffer(32)
        st = lib().hlkv_table_lookup(self.h, b, buf)
        return st, buf.raw

    def handle_of(self, block_id: int) -> Handle:
        return lib().hlkv_table_handle_of(self.h, block_id)

    # sequences
    def create_sequence(self) -> tuple[int, Handle]:
        out = Handle()
        st = lib().hlkv_table_create_sequence(self.h, C.byref(out))
        return st, out

    def append_block(self, seq: Handle, fmt: int, valid_tokens: int = 0, layout: int = 1,
                     scale_mode: int = 0, scale_ref: int = 0) -> tuple[int, Handle]:
        out = Handle()
        req = AllocRequest(fmt, valid_tokens, layout, scale_mode, scale_ref)
        st = lib().hlkv_table_append_block(self.h, seq, C.byref(req), C.byref(out))
        return st, out

    def append_shared_block(self, seq: Handle, b: Handle) -> int:
        return lib().hlkv_table_append_shared_block(self.h, seq, b)

    def release_sequence(self, seq: Handle) -> int:
        return lib().hlkv_table_release_sequence(self.h, seq)

    def sequence_block_ids(self, seq: Handle) -> tuple[int, list[int]]:
        n = _sz()
        st = lib().hlkv_table_sequence_block_ids(self.h, seq, None, 0, C.byref(n))
        if st != Status.OK and not (st == Status.INVALID_ARGUMENT and n.value > 0):
            return st, []
        buf = (_u32 * max(n.value, 1))()
        st = lib().hlkv_table_sequence_block_ids(self.h, seq, buf, n.value, C.byref(n))
        return st, list(buf[: n.value])

    def batch_segments(self, seqs: Sequence[Handle]):
        """Returns (status, numpy uint32 [n, 2])."""
        import numpy as np
        hs = (Handle * max(len(seqs), 1))(*seqs)
        out = np.zeros((max(len(seqs), 1), 2), dtype=np.uint32)
        st = lib().hlkv_table_batch_segments(self.h, hs, len(seqs), out.ctypes.data_as(_P(Segment)))
        return st, out[: len(seqs)]

    def append_tokens(self, seqs, new_formats, layout: int, out=None):
        """Decode-step driver: one more token per sequence.  seqs: a ctypes Handle array
        (or sequence of Handles); new_formats: uint32 per sequence.  Returns (status,
        targets uint32 [n, 2] = (block_id, token), n_done)."""
        import numpy as np
        n = len(seqs)
        hs = seqs if isinstance(seqs, C.Array) else (Handle * max(n, 1))(*seqs)
        fm = np.ascontiguousarray(new_formats, dtype=np.uint32)
        if out is None:
            out = np.zeros((max(n, 1), 2), dtype=np.uint32)
        done = _sz()
        st = lib().hlkv_table_append_tokens(self.h, hs, n, fm.ctypes.data_as(_P(_u32)), layout,
                                            out.ctypes.data, C.byref(done))
        return st, out[:n], done.value

    def build_exec_table(self, seqs: Sequence[Handle]):
        """Returns (status, indptr uint32 [n+1], blocks uint32 [m, 4])."""
        import numpy as np
        hs = (Handle * max(len(seqs), 1))(*seqs)
        total = _sz()
        indptr = np.zeros(len(seqs) + 1, dtype=np.uint32)
        st = lib().hlkv_table_build_exec_table(self.h, hs, len(seqs), indptr.ctypes.data_as(_P(_u32)),
                                               None, 0, C.byref(total))
        if st != Status.OK and not (st == Status.INVALID_ARGUMENT and total.value > 0):
            return st, indptr[:0], np.zeros((0, 4), np.uint32)
        blocks = np.zeros((max(total.value, 1), 4), dtype=np.uint32)
        st = lib().hlkv_table_build_exec_table(self.h, hs, len(seqs), indptr.ctypes.data_as(_P(_u32)),
                                               blocks.ctypes.data_as(_P(ExecDescriptor)), total.value,
                                               C.byref(total))
        return st, indptr, blocks[: total.value]

    def pending(self) -> tuple[int, int]:
        a, b = _sz(), _sz()
        lib().hlkv_table_pending(self.h, C.byref(a), C.byref(b))
        return a.value, b.value

    def collect_delta(self) -> Delta:
        import numpy as np
        nd, ni = self.pending()
        desc = np.zeros((max(nd, 1), 4), dtype=np.uint32)
        ids = np.zeros((max(ni, 1), 2), dtype=np.uint32)
        a, b, ts, ar = _sz(), _sz(), _u32(), _u32()
        st = lib().hlkv_table_collect_delta(self.h, desc.ctypes.data_as(_P(ExecDescriptor)), desc.shape[0],
                                            ids.ctypes.data_as(_P(IdPatch)), ids.shape[0],
                                            C.byref(a), C.byref(b), C.byref(ts), C.byref(ar))
        if st != Status.OK:
            raise HlkvError(f"collect_delta: status {st}")
        return Delta(desc[: a.value], ids[: b.value], ts.value, ar.value)

    def compact_arena(self):
        """HeteroBlockTable::compact_arena.  Returns (status, moves: uint32 [n, 4] of
        {from, to, length, scratch}); nothing changes on a non-OK status."""
        import numpy as np
        live = self.stats()["active_sequences"]
        moves = np.zeros((max(live, 1), 4), dtype=np.uint32)
        n = _sz()
        st = lib().hlkv_table_compact_arena(self.h, moves.ctypes.data, moves.shape[0], C.byref(n))
        return st, moves[: n.value].copy()

    def device_descriptor(self, block_id: int) -> tuple[int, int, int, int]:
        d = lib().hlkv_table_device_descriptor(self.h, block_id)
        return (d.slot, d.info, d.scale_ref, d.block_id)

    def block_tokens(self) -> int: return lib().hlkv_table_block_tokens(self.h)
    def max_blocks(self) -> int: return lib().hlkv_table_max_blocks(self.h)
    def blocks_in_use(self) -> int: return lib().hlkv_table_blocks_in_use(self.h)
    def has_pool(self, f: int) -> bool: return bool(lib().hlkv_table_has_pool(self.h, f))
    def free_slots(self, f: int) -> int: return lib().hlkv_table_free_slots(self.h, f)
    def pool_slots(self, f: int) -> int: return lib().hlkv_table_pool_slots(self.h, f)
    def slot_bytes(self, f: int) -> int: return lib().hlkv_table_slot_bytes(self.h, f)

    def stats(self) -> dict:
        out = (_u64 * 36)()
        lib().hlkv_table_stats(self.h, out)
        v = list(out)
        keys = ["valid_tokens", "token_capacity_in_use", "payload_bytes_in_use",
                "format_changes_committed", "arena_entries", "arena_live_entries",
                "arena_reserved_entries", "arena_free_entries", "pending_descriptor_patches",
                "pending_id_patches"]
        d = {"blocks_in_use": v[0], "blocks_capacity": v[1], "active_sequences": v[2],
             "blocks_per_format": v[3:18], "blocks_per_residency": v[18:22],
             "blocks_per_state": v[22:26]}
        d.update(dict(zip(keys, v[26:36])))
        return d

    def validate(self) -> tuple[int, str]:
        buf = C.create_string_buffer(512)
        st = lib().hlkv_table_validate(self.h, buf, 512)
        return st, buf.value.decode()


class DeviceTables:
    """The persistent device descriptor table + id arena of one Table (hl::kv::DeviceTables)."""

    def __init__(self):
        h = _vp()
        check(lib().hlkv_device_tables_create(C.byref(h)), "hlkv_device_tables_create")
        self.h = h

    def close(self) -> None:
        if getattr(self, "h", None):
            lib().hlkv_device_tables_destroy(self.h)
            self.h = None

    __del__ = close

    def sync(self, table: Table, stream=None) -> None:
        check(lib().hlkv_device_tables_sync(self.h, table.h, _stream_handle(stream)), "device_tables_sync")

    def collect(self, table: Table) -> None:
        """Host half of sync(): takes the table's pending changes (no CUDA call)."""
        check(lib().hlkv_device_tables_collect(self.h, table.h), "device_tables_collect")

    def flush(self, stream=None) -> None:
        """Device half of sync(): uploads and applies the collected changes on `stream`."""
        check(lib().hlkv_device_tables_flush(self.h, _stream_handle(stream)), "device_tables_flush")

    def relocate(self, moves, new_arena_size: int, stream=None) -> None:
        """Applies an arena compaction (moves from Table.compact_arena) to the device arena."""
        import numpy as np
        m = np.ascontiguousarray(moves, dtype=np.uint32).reshape(-1, 4)
        check(lib().hlkv_device_tables_relocate(self.h, m.ctypes.data if m.size else None, m.shape[0],
                                                new_arena_size, _stream_handle(stream)), "device_tables_relocate")

    @property
    def arena_capacity_bytes(self) -> int: return lib().hlkv_device_tables_arena_capacity_bytes(self.h)

    @property
    def table_ptr(self) -> int: return lib().hlkv_device_tables_table(self.h) or 0
    @property
    def table_size(self) -> int: return lib().hlkv_device_tables_table_size(self.h)
    @property
    def arena_ptr(self) -> int: return lib().hlkv_device_tables_arena(self.h) or 0
    @property
    def arena_size(self) -> int: return lib().hlkv_device_tables_arena_size(self.h)
    @property
    def error_word_ptr(self) -> int: return lib().hlkv_device_tables_error_word(self.h) or 0


# ---- kernels ------------------------------------------------------------------------------------
def make_pools(pools: Mapping[int, tuple[object, int, int]]) -> Pools:
    """{format: (device uint8 tensor | pointer, slot_bytes, num_slots)} -> Pools."""
    p = Pools()
    for f, (buf, slot_bytes, num_slots) in pools.items():
        p.pool[f].base = buf if isinstance(buf, int) else int(buf.data_ptr())
        p.pool[f].slot_bytes = slot_bytes
        p.pool[f].num_slots = num_slots
    return p


LAUNCH_OVERLAP_PREVIOUS = 1


def gather_dequant(pools: Pools, layout: Layout, table_ptr: int, table_size: int, arena_ptr: int,
                   arena_size: int, segs, out, err, out_offsets=None, stream=None,
                   overlap_previous: bool = False) -> int:
    """Kernel (1).  segs: device int32 tensor [nseq, 2]; out: device 16-bit tensor; err:
    device int32 tensor [1].  overlap_previous: launch with HLKV_LAUNCH_OVERLAP_PREVIOUS
    (only after a kernel that does not write the segments, offsets, arena or table, such as
    the previous layer's gather).  Raises on a non-OK status."""
    nseq = 0 if segs is None else int(segs.shape[0])
    if overlap_previous:
        st = lib().hlkv_gather_dequant_ex(C.byref(pools), C.byref(layout), table_ptr or None, table_size,
                                          arena_ptr or None, arena_size, _ptr(segs), nseq, _ptr(out),
                                          _ptr(out_offsets), _ptr(err), LAUNCH_OVERLAP_PREVIOUS,
                                          _stream_handle(stream))
    else:
        st = lib().hlkv_gather_dequant(C.byref(pools), C.byref(layout), table_ptr or None, table_size,
                                       arena_ptr or None, arena_size, _ptr(segs), nseq, _ptr(out),
                                       _ptr(out_offsets), _ptr(err), _stream_handle(stream))
    check(st, "hlkv_gather_dequant")
    return st


def append_encode(pools: Pools, layout: Layout, table_ptr: int, table_size: int, targets, tokens,
                  err, stream=None) -> int:
    """Kernel (2).  targets: device int32 [n, 2] (block_id, token); tokens: device fp16/int16
    [n, 2, H, D]."""
    n = int(targets.shape[0])
    st = lib().hlkv_append_encode(C.byref(pools), C.byref(layout), table_ptr or None, table_size,
                                  _ptr(targets), n, _ptr(tokens), _ptr(err), _stream_handle(stream))
    check(st, "hlkv_append_encode")
    return st


def decode_step_queue(dt: "DeviceTables", pools: Pools, layout: Layout, h_targets, d_targets, tokens, err,
                      encode_event=None, stream=None, start_event=None) -> int:
    """Device half of a decode step, queued from native code: targets H2D (h_targets: pinned
    host int32 [n, 2], as table.append_tokens wrote them), the collected delta's upload and
    kernel (3), then kernel (2) into d_targets' blocks.  start_event / encode_event: recorded
    torch.cuda.Events (or None) to record just before kernel (3) / kernel (2)."""
    n = int(d_targets.shape[0])
    st = lib().hlkv_decode_step_queue(dt.h, C.byref(pools), C.byref(layout), _ptr(h_targets), _ptr(d_targets),
                                      n, _ptr(tokens), _ptr(err), start_event, encode_event,
                                      _stream_handle(stream))
    check(st, "hlkv_decode_step_queue")
    return st


def decode_attention(pools: Pools, layout: Layout, table_ptr: int, table_size: int, arena_ptr: int,
                     arena_size: int, segs, q, q_heads: int, softmax_scale: float, out, err,
                     stream=None) -> int:
    """Decode attention over the quantized blocks.  q, out: device 16-bit tensors
    [nseq, q_heads, head_dim]; segs: device int32 [nseq, 2]."""
    nseq = int(segs.shape[0])
    st = lib().hlkv_decode_attention(C.byref(pools), C.byref(layout), table_ptr or None, table_size,
                                     arena_ptr or None, arena_size, _ptr(segs), nseq, _ptr(q), q_heads,
                                     softmax_scale, _ptr(out), _ptr(err), _stream_handle(stream))
    check(st, "hlkv_decode_attention")
    return st


def decode_attention_workspace_bytes(nseq: int, kv_heads: int, head_dim: int, splits: int) -> int:
    return lib().hlkv_decode_attention_workspace_bytes(nseq, kv_heads, head_dim, splits)


def decode_attention_split(pools: Pools, layout: Layout, table_ptr: int, table_size: int, arena_ptr: int,
                           arena_size: int, segs, q, q_heads: int, softmax_scale: float, splits: int,
                           workspace, out, err, stream=None) -> int:
    """Split-KV decode attention; workspace: a device tensor of at least
    decode_attention_workspace_bytes(...) bytes (or None when splits == 1)."""
    nseq = int(segs.shape[0])
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    st = lib().hlkv_decode_attention_split(C.byref(pools), C.byref(layout), table_ptr or None, table_size,
                                           arena_ptr or None, arena_size, _ptr(segs), nseq, _ptr(q), q_heads,
                                           softmax_scale, splits, _ptr(workspace), ws_bytes, _ptr(out),
                                           _ptr(err), _stream_handle(stream))
    check(st, "hlkv_decode_attention_split")
    return st


def decode_attention_balanced_workspace_bytes(nseq: int, kv_heads: int, head_dim: int, ctas: int) -> int:
    return lib().hlkv_decode_attention_balanced_workspace_bytes(nseq, kv_heads, head_dim, ctas)


def decode_attention_balanced(pools: Pools, layout: Layout, table_ptr: int, table_size: int, arena_ptr: int,
                              arena_size: int, segs, q, q_heads: int, softmax_scale: float, ctas: int,
                              workspace, out, err, stream=None) -> int:
    """Decode attention with the blocks of all (sequence, KV head) units balanced over
    `ctas` CTAs; workspace: a device tensor of decode_attention_balanced_workspace_bytes."""
    nseq = int(segs.shape[0])
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    st = lib().hlkv_decode_attention_balanced(C.byref(pools), C.byref(layout), table_ptr or None, table_size,
                                              arena_ptr or None, arena_size, _ptr(segs), nseq, _ptr(q),
                                              q_heads, softmax_scale, ctas, _ptr(workspace), ws_bytes,
                                              _ptr(out), _ptr(err), _stream_handle(stream))
    check(st, "hlkv_decode_attention_balanced")
    return st


NOALLOC_SCRATCH_BYTES = 16 << 20  # HLKV_NOALLOC_SCRATCH_BYTES


def decode_attention_split_noalloc(pools: Pools, layout: Layout, table_ptr: int, table_size: int,
                                   arena_ptr: int, arena_size: int, segs, q, q_heads: int,
                                   softmax_scale: float, splits: int, out, err, stream=None) -> int:
    """Split-KV decode attention with the partials in the library's fixed per-device scratch
    (NOALLOC_SCRATCH_BYTES); no workspace argument and no allocation."""
    nseq = int(segs.shape[0])
    st = lib().hlkv_decode_attention_split_noalloc(C.byref(pools), C.byref(layout), table_ptr or None,
                                                   table_size, arena_ptr or None, arena_size, _ptr(segs),
                                                   nseq, _ptr(q), q_heads, softmax_scale, splits, _ptr(out),
                                                   _ptr(err), _stream_handle(stream))
    check(st, "hlkv_decode_attention_split_noalloc")
    return st


def transcode(pools: Pools, layout: Layout, jobs, err, stream=None) -> int:
    """Format-change transcode.  jobs: device int32 [n, 8] = {from_format, from_slot,
    to_format, to_slot, valid_tokens, 0, 0, 0} (16-byte aligned)."""
    n = int(jobs.shape[0])
    st = lib().hlkv_transcode(C.byref(pools), C.byref(layout), _ptr(jobs), n, _ptr(err),
                              _stream_handle(stream))
    check(st, "hlkv_transcode")
    return st


def apply_delta(table_ptr: int, table_size: int, arena_ptr: int, arena_size: int, desc, ids, err,
                stream=None) -> int:
    """Kernel (3).  desc: device int32 [n, 4]; ids: device int32 [m, 2]."""
    nd = 0 if desc is None else int(desc.shape[0])
    ni = 0 if ids is None else int(ids.shape[0])
    st = lib().hlkv_apply_delta(table_ptr or None, table_size, arena_ptr or None, arena_size,
                                _ptr(desc) if nd else None, nd, _ptr(ids) if ni else None, ni,
                                _ptr(err), _stream_handle(stream))
    check(st, "hlkv_apply_delta")
    return st


def dequantize_fp8_to_fp16(fmt: int, d_in: int, n: int, d_params: int, group: int, d_out: int,
                           stream=None) -> int:
    """Drop-in for hl::quant::cuda::dequantize_fp8_to_fp16 (raw device pointers).  Returns the
    status without raising, like the reference's DeviceStatus."""
    return lib().hlkv_dequantize_fp8_to_fp16(fmt, d_in or None, n, d_params or None, group,
                                             d_out or None, _stream_handle(stream))


def dequantize_to_fp16(fmt: int, d_packed: int, packed_size: int, n: int, d_params: int,
                       n_params: int, group: int, d_out: int, out_size: int, d_err: int,
                       stream=None) -> int:
    return lib().hlkv_dequantize_to_fp16(fmt, d_packed or None, packed_size, n, d_params or None,
                                         n_params, group, d_out or None, out_size, d_err or None,
                                         _stream_handle(stream))


def quantize(fmt: int, d_in: int, n: int, group: int, d_params: int, n_params: int,
             d_packed: int, packed_size: int, d_err: int, stream=None) -> int:
    return lib().hlkv_quantize(fmt, d_in or None, n, group, d_params or None, n_params,
                               d_packed or None, packed_size, d_err or None, _stream_handle(stream))

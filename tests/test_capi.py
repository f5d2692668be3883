"""The C ABI without a GPU: libhlkv.so loads, exports every entry point that
include/hlkv.h declares, and rejects bad arguments before touching the device."""
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions() -> set[str]:
    text = open(os.path.join(ROOT, "include", "hlkv.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(hlkv_[a-z0-9_]+)\s*\(", text))


def test_every_declared_symbol_is_exported(hlkv_lib):
    names = declared_functions()
    assert len(names) >= 50
    lib = hlkv_lib.lib()
    missing = [n for n in sorted(names) if not hasattr(lib, n)]
    assert not missing, missing
    bound = {name for name, _, _ in hlkv_lib.SIGNATURES}
    assert names == bound, (names ^ bound)


def test_layout_slot_bytes(hlkv_lib):
    lay = hlkv_lib.Layout(16, 8, 128, 1)
    # 65 536 / 32 768 + 1 024 / 16 384 + 2 048 bytes per block-layer
    assert [hlkv_lib.layout_slot_bytes(f, lay) for f in range(4)] == [65536, 33792, 33792, 18432]
    assert hlkv_lib.layout_slot_bytes(4, lay) == 0
    assert hlkv_lib.layout_slot_bytes(1, hlkv_lib.Layout(16, 8, 96, 1)) == 0
    assert hlkv_lib.layout_slot_bytes(1, hlkv_lib.Layout(0, 8, 128, 1)) == 0


def test_flat_codecs_reject_bad_arguments_without_a_launch(hlkv_lib):
    L = hlkv_lib.lib()
    # Format and group rules (hl::quant::cuda::dequantize_fp8_to_fp16 contract).
    assert hlkv_lib.dequantize_fp8_to_fp16(0, 1, 16, 1, 16, 1, stream=0) == hlkv_lib.UNSUPPORTED_FORMAT
    assert hlkv_lib.dequantize_fp8_to_fp16(3, 1, 16, 1, 16, 1, stream=0) == hlkv_lib.UNSUPPORTED_FORMAT
    assert hlkv_lib.dequantize_fp8_to_fp16(4, 1, 16, 1, 16, 1, stream=0) == hlkv_lib.UNSUPPORTED_FORMAT
    assert hlkv_lib.dequantize_fp8_to_fp16(1, 1, 16, 1, 0, 1, stream=0) == hlkv_lib.INVALID_ARGUMENT
    assert hlkv_lib.dequantize_fp8_to_fp16(1, 1, 16, 1, 16, 0, stream=0) == hlkv_lib.INVALID_ARGUMENT
    assert hlkv_lib.dequantize_fp8_to_fp16(1, 0, 0, 0, 16, 0, stream=0) == hlkv_lib.OK  # n == 0
    # dequantize_to_fp16: the reference's check_args order.
    assert hlkv_lib.dequantize_to_fp16(9, 1, 64, 4, 1, 1, 4, 1, 64, 1, stream=0) == hlkv_lib.UNSUPPORTED_FORMAT
    assert hlkv_lib.dequantize_to_fp16(0, 1, 64, 4, 0, 0, 4, 1, 64, 1, stream=0) == hlkv_lib.INVALID_ARGUMENT
    assert hlkv_lib.dequantize_to_fp16(3, 1, 64, 4, 1, 1, 3, 1, 64, 1, stream=0) == hlkv_lib.INVALID_ARGUMENT
    assert hlkv_lib.dequantize_to_fp16(3, 1, 64, 8, 1, 1, 4, 1, 64, 1, stream=0) == hlkv_lib.INVALID_ARGUMENT
    assert hlkv_lib.dequantize_to_fp16(3, 1, 1, 4, 1, 1, 4, 1, 64, 1, stream=0) == hlkv_lib.BUFFER_TOO_SMALL
    assert hlkv_lib.dequantize_to_fp16(3, 1, 64, 4, 1, 1, 4, 1, 3, 1, stream=0) == hlkv_lib.BUFFER_TOO_SMALL
    # quantize_reference's rules.
    assert hlkv_lib.quantize(7, 1, 4, 4, 1, 1, 1, 8, 1, stream=0) == hlkv_lib.UNSUPPORTED_FORMAT
    assert hlkv_lib.quantize(3, 1, 4, 2, 1, 1, 1, 8, 1, stream=0) == hlkv_lib.INVALID_ARGUMENT
    assert hlkv_lib.quantize(3, 1, 4, 4, 1, 1, 1, 1, 1, stream=0) == hlkv_lib.BUFFER_TOO_SMALL
    assert hlkv_lib.quantize(3, 0, 0, 4, 0, 0, 0, 0, 0, stream=0) == hlkv_lib.OK
    assert L.hlkv_last_cuda_error() == 0


def test_kernel_entry_points_reject_bad_arguments(hlkv_lib):
    L = hlkv_lib.lib()
    pools = hlkv_lib.Pools()
    lay = hlkv_lib.Layout(16, 8, 128, 1)
    import ctypes as C
    # No error word -> invalid argument, nothing launched.
    assert L.hlkv_gather_dequant(C.byref(pools), C.byref(lay), None, 0, None, 0, 1, 1, 16, None, None, 0) == 1
    assert L.hlkv_append_encode(C.byref(pools), C.byref(lay), None, 0, 1, 1, 16, None, 0) == 1
    assert L.hlkv_apply_delta(None, 0, None, 0, 16, 1, None, 0, None, 0) == 1
    # Misaligned output / unsupported layout.
    assert L.hlkv_gather_dequant(C.byref(pools), C.byref(lay), None, 0, None, 0, 16, 1, 18, None, 64, 0) == 1
    bad = hlkv_lib.Layout(16, 8, 100, 1)
    assert L.hlkv_gather_dequant(C.byref(pools), C.byref(bad), None, 0, None, 0, 16, 1, 16, None, 64, 0) == 1
    # Empty work is a no-op.
    assert L.hlkv_gather_dequant(C.byref(pools), C.byref(lay), None, 0, None, 0, None, 0, None, None, 64, 0) == 0
    assert L.hlkv_apply_delta(None, 0, None, 0, None, 0, None, 0, 64, 0) == 0
    assert L.hlkv_append_encode(C.byref(pools), C.byref(lay), None, 0, None, 0, None, 64, 0) == 0


def test_attention_and_transcode_reject_bad_arguments(hlkv_lib):
    """Argument checks of the attention entry points and the transcode, which return before
    any CUDA call (the pointers below are never dereferenced)."""
    import ctypes as C
    L = hlkv_lib.lib()
    pools = hlkv_lib.Pools()
    lay = hlkv_lib.Layout(16, 8, 128, 1)
    p8, err = C.c_void_p(256), C.c_void_p(512)
    INV, OK, SMALL = hlkv_lib.INVALID_ARGUMENT, hlkv_lib.OK, hlkv_lib.BUFFER_TOO_SMALL

    def attn(layout=lay, nseq=1, qh=32, scale=0.1, e=err):
        return L.hlkv_decode_attention(C.byref(pools), C.byref(layout), None, 0, None, 0, p8, nseq, p8,
                                       qh, scale, p8, e, None)

    assert attn(e=None) == INV
    assert attn(qh=12) == INV                    # not a multiple of the 8 KV heads
    assert attn(qh=8 * 16) == INV                # group 16: groups are 1, 2, 4, 8
    assert attn(scale=0.0) == INV and attn(scale=float("inf")) == INV and attn(scale=float("nan")) == INV
    assert attn(layout=hlkv_lib.Layout(16, 8, 256, 1)) == INV  # head_dim 64 or 128 only
    assert attn(layout=hlkv_lib.Layout(1024, 8, 128, 1)) == INV  # more than 512 block tokens
    assert attn(nseq=0) == OK                    # empty batch: nothing to do

    def split(splits, ws, ws_bytes):
        return L.hlkv_decode_attention_split(C.byref(pools), C.byref(lay), None, 0, None, 0, p8, 4, p8,
                                             32, 0.1, splits, ws, ws_bytes, p8, err, None)

    need = hlkv_lib.decode_attention_workspace_bytes(4, 8, 128, 3)
    assert split(0, p8, need) == INV                       # no splits
    assert split(3, None, need) == INV                     # no workspace
    assert split(3, C.c_void_p(264), need) == INV          # workspace not 16-byte aligned
    assert split(3, p8, need - 1) == SMALL

    def balanced(ctas, ws_bytes):
        return L.hlkv_decode_attention_balanced(C.byref(pools), C.byref(lay), None, 0, None, 0, p8, 4, p8,
                                                32, 0.1, ctas, p8, ws_bytes, p8, err, None)

    bneed = hlkv_lib.decode_attention_balanced_workspace_bytes(4, 8, 128, 64)
    assert balanced((1 << 20) + 1, 1 << 40) == INV         # at most 2^20 CTAs
    assert balanced(64, bneed - 1) == SMALL

    def transcode(n, jobs, e=err, layout=lay):
        return L.hlkv_transcode(C.byref(pools), C.byref(layout), jobs, n, e, None)

    assert transcode(1, p8, e=None) == INV
    assert transcode(1, None) == INV
    assert transcode(1, C.c_void_p(264)) == INV            # jobs not 16-byte aligned
    assert transcode(1, p8, layout=hlkv_lib.Layout(16, 8, 100, 1)) == INV
    assert transcode(0, None) == OK
    assert L.hlkv_last_cuda_error() == 0


def test_product_does_not_load_the_oracle(hlkv_lib):
    """The product library links no oracle code."""
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", hlkv_lib.LIB_PATH], capture_output=True,
                         text=True).stdout
    assert "orc_" not in out and "ref_gather" not in out and "table_trace" not in out
    deps = subprocess.run(["ldd", hlkv_lib.LIB_PATH], capture_output=True, text=True).stdout
    assert "oracle" not in deps and "hlkv_ref" not in deps

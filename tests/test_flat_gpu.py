"""Flat device codecs against the reference: the drop-in dequantize_fp8_to_fp16 (the
reference's own GPU test plan, tests/project2/test_dequant_cuda.cpp:193-300), and the device
quantize / dequantize_to_fp16 against the reference-produced fixtures and the oracle."""
import os

import numpy as np
import pytest

from helpers import fp16_nan

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden.npz")


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


def _dev(arr: np.ndarray, offset_bytes: int = 0):
    """Device copy of a byte view of `arr` placed `offset_bytes` into a fresh allocation."""
    import torch
    raw = np.ascontiguousarray(arr).view(np.uint8).reshape(-1)
    buf = torch.zeros(raw.size + offset_bytes + 64, dtype=torch.uint8, device="cuda")
    buf[offset_bytes:offset_bytes + raw.size] = torch.from_numpy(raw).cuda()
    return buf, buf.data_ptr() + offset_bytes


def _fp8_run(hlkv, fmt, codes, params, group, in_off=0, out_off=0):
    import torch
    n = codes.size
    keep_din, din = _dev(codes, in_off)
    keep_dp, dp = _dev(params.astype(np.float32))
    out = torch.full((n + out_off + 8,), 0x7777, dtype=torch.int32, device="cuda").to(torch.int16)
    st = hlkv.dequantize_fp8_to_fp16(fmt, din, n, dp, group, out.data_ptr() + 2 * out_off)
    torch.cuda.synchronize()
    assert st == hlkv.OK
    return out.cpu().numpy().view(np.uint16)[out_off:out_off + n]


def test_fp8_all_codes_kernel_scales_against_reference_fixtures(hlkv_lib, golden, cuda_device):
    codes = np.arange(256, dtype=np.uint8)
    for fmt in (1, 2):
        for k, s in enumerate(golden["k_scales"]):
            params = np.array([[s, 0.0]], np.float32)
            want = golden[f"fp8_scales_{fmt}"][k]
            assert np.array_equal(_fp8_run(hlkv_lib, fmt, codes, params, 256), want), (fmt, s)
            assert np.array_equal(_fp8_run(hlkv_lib, fmt, codes, params, 256, 1, 1), want), (fmt, s)


def test_fp8_random_shapes_groups_alignments(hlkv_lib, oracle, cuda_device):
    rng = np.random.default_rng(11)
    for fmt in (1, 2):
        for n in (1, 7, 8, 9, 255, 4099, 65543):
            for g in (1, 24, 128, n):
                codes = rng.integers(0, 256, size=n, dtype=np.uint8)
                e = rng.integers(-24, 13, size=-(-n // g))
                m = 1 + rng.integers(0, 1024, size=e.size) / 1024.0
                sign = np.where(rng.integers(0, 2, size=e.size) == 1, -1.0, 1.0)
                params = np.stack([(sign * np.ldexp(m, e)).astype(np.float32),
                                   np.zeros(e.size, np.float32)], 1)
                st, want = oracle.dequantize_to_fp16(fmt, codes, n, params, g)
                assert st == 0
                for in_off, out_off in ((0, 0), (8, 8), (3, 0), (0, 1), (5, 3)):
                    got = _fp8_run(hlkv_lib, fmt, codes, params, g, in_off, out_off)
                    assert np.array_equal(got, want), (fmt, n, g, in_off, out_off)


def test_fp8_large_input_grid_stride(hlkv_lib, oracle, cuda_device):
    rng = np.random.default_rng(13)
    n = (1 << 25) + 13
    codes = rng.integers(0, 256, size=n, dtype=np.uint8)
    params = np.stack([rng.standard_normal(-(-n // 128)).astype(np.float32),
                       np.zeros(-(-n // 128), np.float32)], 1)
    st, want = oracle.dequantize_to_fp16(1, codes, n, params, 128)
    assert st == 0
    assert np.array_equal(_fp8_run(hlkv_lib, 1, codes, params, 128), want)


def test_fp8_runs_on_the_given_stream(hlkv_lib, oracle, cuda_device):
    import torch
    rng = np.random.default_rng(17)
    codes = rng.integers(0, 256, size=10000, dtype=np.uint8)
    params = np.stack([rng.standard_normal(157).astype(np.float32), np.zeros(157, np.float32)], 1)
    s = torch.cuda.Stream()
    keep_din, din = _dev(codes)
    keep_dp, dp = _dev(params)
    out = torch.zeros(10000, dtype=torch.int16, device="cuda")
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        assert hlkv_lib.dequantize_fp8_to_fp16(2, din, 10000, dp, 64, out.data_ptr(), stream=s) == 0
    s.synchronize()
    _, want = oracle.dequantize_to_fp16(2, codes, 10000, params, 64)
    assert np.array_equal(out.cpu().numpy().view(np.uint16), want)


def test_device_quantize_matches_reference_fixtures(hlkv_lib, golden, cuda_device):
    import torch
    for key in [k for k in golden.files if k.startswith("q_in_")]:
        _, _, fmt, gs = key.split("_")
        fmt, gs = int(fmt), int(gs)
        x = golden[key]
        n = x.size
        ng = 0 if gs == 0 else -(-n // gs)
        pb = 2 * n if fmt == 0 else (n // 2 + n % 2 if fmt == 3 else n)
        keep_dx, dx = _dev(x)
        params = torch.full((max(ng, 1), 2), 9.0, dtype=torch.float32, device="cuda")
        packed = torch.full((pb,), 0xAB, dtype=torch.int32, device="cuda").to(torch.uint8)
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        st = hlkv_lib.quantize(fmt, dx, n, gs, params.data_ptr(), ng, packed.data_ptr(), pb, err.data_ptr())
        torch.cuda.synchronize()
        assert st == 0 and int(err.item()) == 0
        assert np.array_equal(packed.cpu().numpy(), golden[f"q_packed_{fmt}_{gs}"]), key
        if ng:
            assert np.array_equal(params.cpu().numpy()[:ng].view(np.uint32),
                                  golden[f"q_params_{fmt}_{gs}"].view(np.uint32)), key
        out = torch.zeros(n, dtype=torch.int16, device="cuda")
        st = hlkv_lib.dequantize_to_fp16(fmt, packed.data_ptr(), pb, n, params.data_ptr(), ng, gs,
                                         out.data_ptr(), n, err.data_ptr())
        torch.cuda.synchronize()
        assert st == 0 and int(err.item()) == 0
        assert np.array_equal(out.cpu().numpy().view(np.uint16), golden[f"q_fp16_{fmt}_{gs}"]), key


def test_device_quantize_random_and_skips_nonfinite_groups(hlkv_lib, oracle, cuda_device):
    import torch
    rng = np.random.default_rng(23)
    for fmt in (1, 2, 3):
        for n, gs in ((4097, 16), (1000, 128), (129, 2), (2 ** 16, 4096), (33, 32)):
            x = (rng.standard_normal(n) * rng.choice([1e-3, 1, 1e3])).astype(np.float32)
            bad_group = 1 if n // gs > 2 else None
            if bad_group is not None:
                x[bad_group * gs + 1] = np.inf
            ng = -(-n // gs)
            pb = n // 2 + n % 2 if fmt == 3 else n
            keep_dx, dx = _dev(x)
            params = torch.full((ng, 2), 9.0, dtype=torch.float32, device="cuda")
            packed = torch.full((pb,), 0xAB, dtype=torch.int32, device="cuda").to(torch.uint8)
            err = torch.zeros(1, dtype=torch.int32, device="cuda")
            assert hlkv_lib.quantize(fmt, dx, n, gs, params.data_ptr(), ng, packed.data_ptr(), pb,
                                     err.data_ptr()) == 0
            torch.cuda.synchronize()
            got_p, got_c = params.cpu().numpy(), packed.cpu().numpy()
            for gi in range(ng):
                sl = slice(gi * gs, min(n, (gi + 1) * gs))
                st, p, c = oracle.quantize(fmt, x[sl], gs)
                cs = slice(sl.start // 2, (sl.stop + 1) // 2) if fmt == 3 else sl
                if gi == bad_group:
                    assert st == 1 and np.all(got_p[gi] == 9.0) and np.all(got_c[cs] == 0xAB)
                else:
                    assert st == 0
                    assert np.array_equal(got_p[gi].view(np.uint32), p[0].view(np.uint32)), (fmt, n, gi)
                    assert np.array_equal(got_c[cs], c), (fmt, n, gi)
            assert int(err.item()) == (512 if bad_group is not None else 0)


def test_device_dequantize_every_format_and_bad_params(hlkv_lib, oracle, cuda_device):
    import torch
    rng = np.random.default_rng(29)
    for fmt, gs in ((0, 0), (1, 32), (2, 8), (3, 64), (3, 2)):
        n = 3001 if fmt != 3 else 3000
        pb = 2 * n if fmt == 0 else (n // 2 if fmt == 3 else n)
        packed = rng.integers(0, 256, size=pb, dtype=np.uint8)
        ng = 0 if gs == 0 else -(-n // gs)
        params = np.stack([rng.standard_normal(max(ng, 1)).astype(np.float32),
                           (rng.standard_normal(max(ng, 1)) if fmt == 3 else np.zeros(max(ng, 1))).astype(np.float32)], 1)
        if ng > 3:
            params[2, 0] = np.nan  # group 2 must be skipped
        keep_dpk, dpk = _dev(packed)
        keep_dp, dp = _dev(params)
        out = torch.from_numpy(np.full(n, 0x5555, np.uint16).view(np.int16)).cuda()
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        assert hlkv_lib.dequantize_to_fp16(fmt, dpk, pb, n, dp, ng, gs, out.data_ptr(), n, err.data_ptr()) == 0
        torch.cuda.synchronize()
        got = out.cpu().numpy().view(np.uint16)
        if ng > 3:
            assert int(err.item()) == 512
            assert np.all(got[2 * gs:3 * gs] == 0x5555)
            params[2, 0] = 1.0  # compare the rest against the oracle
            st, want = oracle.dequantize_to_fp16(fmt, packed, n, params[:ng], gs)
            mask = np.ones(n, bool)
            mask[2 * gs:3 * gs] = False
            assert st == 0 and np.array_equal(got[mask], want[mask])
        else:
            st, want = oracle.dequantize_to_fp16(fmt, packed, n, params[:max(ng, 0)] if ng else np.zeros((0, 2), np.float32), gs)
            assert st == 0 and int(err.item()) == 0 and np.array_equal(got, want)


@pytest.fixture(scope="module")
def ref_cuda():
    from oracle.oracle import RefCuda, ref_cuda_available
    if not ref_cuda_available():
        pytest.skip("the reference's GPU kernel is not built (no reference tree)")
    return RefCuda()


def test_fp8_drop_in_equals_reference_gpu_kernel(hlkv_lib, ref_cuda, cuda_device):
    """The drop-in against the reference's own kernel (dequant_kernel.cu, compiled for
    sm_100a from its source): bit-identical outputs over every code, the kScales set, random
    group sizes and both kernels' vector and per-element paths (aligned and not)."""
    import torch
    rng = np.random.default_rng(41)
    cases = [(fmt, 256, 256, 0, 0) for fmt in (1, 2)]
    cases += [(int(rng.choice([1, 2])), int(n), int(g), int(a), int(b))
              for n, g, a, b in [(4096, 128, 0, 0), (4099, 24, 3, 1), (65543, 8, 0, 0),
                                 (1 << 20, 128, 0, 0), (1000, 1000, 5, 3), (77, 7, 1, 0)]]
    for fmt, n, g, in_off, out_off in cases:
        codes = np.arange(256, dtype=np.uint8) if n == 256 else rng.integers(0, 256, n, dtype=np.uint8)
        ng = -(-n // g)
        scales = (rng.choice([-1.0, 1.0], ng) * np.ldexp(1 + rng.integers(0, 1024, ng) / 1024.0,
                                                          rng.integers(-30, 20, ng))).astype(np.float32)
        params = np.stack([scales, np.zeros(ng, np.float32)], 1)
        keep_in, din = _dev(codes, in_off)
        keep_p, dp = _dev(params)
        outs = []
        for impl in ("ours", "ref"):
            out = torch.full((n + out_off + 8,), 0x3333, dtype=torch.int32, device="cuda").to(torch.int16)
            d_out = out.data_ptr() + 2 * out_off
            if impl == "ours":
                st = hlkv_lib.dequantize_fp8_to_fp16(fmt, din, n, dp, g, d_out)
            else:
                st = ref_cuda.dequantize_fp8_to_fp16(fmt, din, n, dp, g, d_out)
            torch.cuda.synchronize()
            assert st == 0, (impl, st)
            outs.append(out.cpu().numpy().view(np.uint16)[out_off:out_off + n])
        # NaN codes: both give a NaN (the reference test compares NaN by class,
        # test_dequant_cuda.cpp:81-86); every other output bit for bit.
        nan0, nan1 = fp16_nan(outs[0]), fp16_nan(outs[1])
        assert np.array_equal(nan0, nan1), (fmt, n, g)
        bad = np.nonzero((outs[0] != outs[1]) & ~nan0)[0]
        assert bad.size == 0, (fmt, n, g, in_off, out_off, bad[:4], outs[0][bad[:4]], outs[1][bad[:4]])

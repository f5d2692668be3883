"""The reference's CPU hl_quant API as libhlkv.so exports it.

tests/cpp/test_quant_api.cpp is written against include/hl_quant/cpu_quant.hpp,
cpu_dequant.hpp and cuda_dequant.hpp with the reference's own call forms and is
linked against libhlkv.so alone.  Its results must equal the golden fixtures
(tests/golden/golden.npz, made by the reference library) bit for bit, and -- where
the reference tree is present -- the reference library itself on seeded random
inputs, including non-finite values, zeros of both signs and group tails.
"""
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BUILD = os.path.join(ROOT, "tests", "_build")
GOLDEN = os.path.join(ROOT, "tests", "golden", "golden.npz")


@pytest.fixture(scope="module")
def quant_api(hlkv_lib):
    os.makedirs(BUILD, exist_ok=True)
    src = os.path.join(ROOT, "tests", "cpp", "test_quant_api.cpp")
    out = os.path.join(BUILD, "test_quant_api")
    hdrs = [os.path.join(ROOT, "include", "hl_quant", h) for h in
            ("cpu_quant.hpp", "cpu_dequant.hpp", "cuda_dequant.hpp", "quant_types.hpp")]
    deps = [src, hlkv_lib.LIB_PATH, *hdrs]
    if not os.path.exists(out) or os.path.getmtime(out) < max(os.path.getmtime(d) for d in deps):
        libdir = os.path.dirname(hlkv_lib.LIB_PATH)
        subprocess.run(["g++", "-std=c++20", "-O1", "-Wall", "-Wextra", "-Werror", "-I",
                        os.path.join(ROOT, "include"), "-I", "/usr/local/cuda/include", src,
                        "-o", out + ".tmp", "-L", libdir, "-l:libhlkv.so", f"-Wl,-rpath,{libdir}"],
                       check=True)
        os.replace(out + ".tmp", out)
    return out


def _run(exe, d, cases):
    with open(os.path.join(d, "q_cases.txt"), "w") as f:
        for fmt, gs, name, x in cases:
            x.astype(np.float32).tofile(os.path.join(d, name))
            f.write(f"{fmt} {gs} {name}\n")
    r = subprocess.run([exe, d], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
    assert " 0 failures" in r.stdout, r.stdout[-4000:]


def _load(d, name, dtype):
    return np.fromfile(os.path.join(d, name), dtype=dtype)


def test_links_libhlkv_alone(quant_api):
    r = subprocess.run(["ldd", quant_api], capture_output=True, text=True)
    libs = [l.split()[0] for l in r.stdout.splitlines() if "=>" in l]
    assert any(l == "libhlkv.so" for l in libs)
    assert not any("hlkv_ref" in l or "oracle" in l for l in r.stdout.splitlines())


def test_matches_golden_fixtures(quant_api, tmp_path):
    g = np.load(GOLDEN)
    d = str(tmp_path)
    g["encode_in"].tofile(os.path.join(d, "encode_in.bin"))
    g["k_scales"].astype(np.float32).tofile(os.path.join(d, "k_scales.bin"))
    cases = []
    for key in [k for k in g.files if k.startswith("q_in_")]:
        fmt, gs = (int(v) for v in key[5:].split("_"))
        cases.append((fmt, gs, key + ".bin", g[key]))
    _run(quant_api, d, cases)
    for f in (0, 1, 2):
        assert np.array_equal(_load(d, f"decode_{f}.bin", np.uint32), g[f"decode_{f}"]), f"decode {f}"
        assert np.array_equal(_load(d, f"encode_{f}.bin", np.uint16), g[f"encode_{f}"]), f"encode {f}"
    for f in (1, 2):
        want = g[f"fp8_scales_{f}"].reshape(-1)
        assert np.array_equal(_load(d, f"fp8_scales_{f}.bin", np.uint16), want), f"fp8 x scales {f}"
        for path in ("scalar", "vector"):
            assert np.array_equal(_load(d, f"emulate_{path}_{f}.bin", np.uint16), want), (f, path)
    for fmt, gs, _, _ in cases:
        tag = f"{fmt}_{gs}"
        assert np.array_equal(_load(d, f"q_params_{tag}.bin", np.uint32),
                              g[f"q_params_{tag}"].view(np.uint32).reshape(-1)), tag
        assert np.array_equal(_load(d, f"q_packed_{tag}.bin", np.uint8), g[f"q_packed_{tag}"]), tag
        assert np.array_equal(_load(d, f"q_fp16_{tag}.bin", np.uint16), g[f"q_fp16_{tag}"]), tag


def _random_cases(seed: int):
    rng = np.random.default_rng(seed)
    cases = []
    for fmt, gs in ((0, 0), (1, 1), (1, 7), (1, 128), (2, 16), (2, 129), (3, 2), (3, 18), (3, 128)):
        n = int(rng.integers(1, 3000))
        x = (rng.standard_normal(n) * rng.choice([1e-6, 1e-3, 1, 30, 5e3], size=n)).astype(np.float32)
        x[rng.integers(0, n, size=max(1, n // 50))] = 0.0
        x[rng.integers(0, n, size=max(1, n // 50))] = -0.0
        if fmt == 0:  # FP16 takes non-finite inputs, halfway cases and overflow
            x[rng.integers(0, n, size=4)] = [np.inf, -np.inf, np.nan, 65520.0]
        cases.append((fmt, gs, f"r{seed}_{fmt}_{gs}.bin", x))
    return cases


@pytest.mark.parametrize("seed", [1, 2, 3])
def test_matches_live_reference(quant_api, ref, tmp_path, seed):
    g = np.load(GOLDEN)
    d = str(tmp_path)
    rng = np.random.default_rng(100 + seed)
    scaled = (rng.standard_normal(20000) * 10.0 ** rng.integers(-8, 6, 20000)).astype(np.float32)
    patterns = rng.integers(0, 2 ** 32, 20000, dtype=np.uint64).astype(np.uint32).view(np.float32)
    enc = np.concatenate([scaled, patterns])
    enc.tofile(os.path.join(d, "encode_in.bin"))
    g["k_scales"].astype(np.float32).tofile(os.path.join(d, "k_scales.bin"))
    cases = _random_cases(seed)
    _run(quant_api, d, cases)
    for f in (0, 1, 2):
        assert np.array_equal(_load(d, f"encode_{f}.bin", np.uint16), ref.encode(f, enc)), f"encode {f}"
    for fmt, gs, _, x in cases:
        tag = f"{fmt}_{gs}"
        st, p, packed = ref.quantize(fmt, x, gs)
        assert st == 0
        assert np.array_equal(_load(d, f"q_params_{tag}.bin", np.uint32), p.view(np.uint32).reshape(-1)), tag
        assert np.array_equal(_load(d, f"q_packed_{tag}.bin", np.uint8), packed), tag
        st, h = ref.dequantize_to_fp16(fmt, packed, x.size, p, gs)
        assert st == 0 and np.array_equal(_load(d, f"q_fp16_{tag}.bin", np.uint16), h), tag

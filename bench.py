"""Benchmark of the heterogeneous KV gather-dequant path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl hlkv|reference]
                    [--workload llama8b|mixed|mixed_updates|homogeneous|fp16|e4m3|int4|llama70b|decode|...]

Default workload ("llama8b", the Llama-3-8B-shaped cache): 32 layers of 64
sequences x 8192 tokens, 16-token blocks, 8 KV heads x 128, K and V, age tiers
(newest 512 tokens FP16, the 2048 before them E4M3, the rest INT4), N(0,1)
values with 4 outlier channels per head x20, block ids and slots scattered by a
seeded scramble.  The sequences are sharded over the N GPUs (one process each,
torchrun for N > 1; strong scaling, no inter-GPU traffic): one step is one
hlkv_gather_dequant launch per layer into an FP16 scratch buffer of a layer's
size.  A step moves 95 GB at N=1, far more than the 126 MB L2, so no flush is
needed.  Ranks meet only at barriers and at the max-over-ranks reduction of the
timings.

Other workloads: "mixed" (one layer of 64 x 2048 tokens, per-block formats FP16
.25 / E4M3 .5 / INT4 .25, a cache per GPU: weak scaling), "homogeneous" (1
sequence x 4096 tokens of E4M3, L2-resident: flushed between steps),
single-format caches "fp16" / "e4m3" / "int4", "llama70b" (8 resident layers of
16 x 131072 tokens with 1000 descriptor updates per step), the decode-step
append ("decode"), decode attention ("attn_*") and the flat FP8 drop-in
("flat_*").

value = algorithmic bytes of all ranks / max-over-ranks device time, GB/s.
Algorithmic bytes per block = codes + row parameters read + 2*T*H*D*2 bytes
written + 20 bytes of descriptor and arena entry (131 092 / 99 348 / 83 988
bytes for FP16 / E4M3 / INT4 blocks).

Beside it the line carries: `e2e` (the same metric through the C ABI with host
buffers: segments up, every layer's FP16 output down), `parity` (the last
launch's output for a sample of sequences against the reference's CPU gather,
bit for bit), `roofline` and `cpu_baseline` (the reference's CPU gather of the
same sample on all host threads).

--impl reference times the reference's CPU path instead (its
dequantize_reference_to_fp16 per parameter group walked through its own
descriptor table, oracle/_ref), on all host threads, over a bounded sample of
the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "hl-kv_b200"))

METRIC = "hetero KV dequant GB/s per GPU (% of HBM peak) at 1/2/4/8 B200; CPU ref GB/s"
WORKLOADS = {
    # The reference's headline configuration (the default): one layer, per-GPU cache fixed.
    "mixed": dict(nseq=64, blocks=128, probs=(0.25, 0.5, 0.0, 0.25), scaling="weak",
                  name="mixed-format single layer: 64 seq x 2048 tok, 16-tok blocks, 8 KV heads x 128, "
                       "K+V, FP16 .25 / E4M3 .5 / INT4 .25, N(0,1) + 4 outlier channels x20"),
    # The headline cache with the allocator live: 1000 random descriptor updates (valid
    # tokens, format changes transcoded on the device) applied before every gather.
    "mixed_updates": dict(nseq=64, blocks=128, probs=(0.25, 0.5, 0.0, 0.25), scaling="weak",
                          updates=1000,
                          name="mixed-format single layer (as 'mixed') + 1000 random descriptor "
                               "updates per step (valid tokens; format changes transcoded on the device)"),
    "homogeneous": dict(nseq=1, blocks=256, probs=(0.0, 1.0, 0.0, 0.0), scaling="weak", flush=True,
                        l2="25 MB per step fits the L2: a 2x-L2 buffer is overwritten between steps, "
                           "value from the per-step events",
                        name="homogeneous E4M3: 1 seq x 4096 tok, 16-tok blocks, 8 KV heads x 128, K+V"),
    # Single-format caches of the mixed workload's size: per-format throughput.
    "fp16": dict(nseq=64, blocks=128, probs=(1.0, 0.0, 0.0, 0.0), scaling="weak",
                 name="FP16 only: 64 seq x 2048 tok, 16-tok blocks, 8 KV heads x 128, K+V"),
    "e4m3": dict(nseq=64, blocks=128, probs=(0.0, 1.0, 0.0, 0.0), scaling="weak",
                 name="E4M3 only: 64 seq x 2048 tok, 16-tok blocks, 8 KV heads x 128, K+V"),
    "int4": dict(nseq=64, blocks=128, probs=(0.0, 0.0, 0.0, 1.0), scaling="weak",
                 name="INT4 only: 64 seq x 2048 tok, 16-tok blocks, 8 KV heads x 128, K+V"),
    # Llama-3-8B-shaped cache sharded by sequence; a step dequantizes all 32 layers, one
    # launch per layer into one FP16 scratch buffer.
    "llama8b": dict(nseq=64, tokens=8192, tiers=(512, 2048), layers=32, scaling="strong", cpu_sample_seqs=2,
                    name="Llama-3-8B cache: 32 layers, 64 seq x 8192 tok sharded by sequence, "
                         "8 KV heads x 128, K+V; newest 512 tok FP16, previous 2048 E4M3, rest INT4"),
    # One layer of that cache (2.97 GB per launch): the same launch as each of llama8b's, small
    # enough (0.8 GB of pools + 2.1 GB of output) for a full ncu capture.
    "llama8b_layer": dict(nseq=64, tokens=8192, tiers=(512, 2048), layers=1, scaling="strong", cpu_sample_seqs=2,
                          name="one layer of the Llama-3-8B cache: 64 seq x 8192 tok sharded by sequence, "
                               "8 KV heads x 128, K+V; newest 512 tok FP16, previous 2048 E4M3, rest INT4"),
    # Llama-3-70B-shaped long context sharded by sequence; 8 resident layers per GPU (the
    # 80-layer payload of 234 GB does not fit one GPU), one launch per layer per step.
    "llama70b": dict(nseq=16, blocks=8192, probs=(0.05, 0.10, 0.0, 0.85), layers=8,
                     scaling="strong", updates=1000, cpu_sample_seqs=1,
                     name="Llama-3-70B long context: 16 seq x 131072 tok sharded by sequence, "
                          "8 resident layers, 8 KV heads x 128, K+V; INT4 .85 / E4M3 .10 / FP16 .05; "
                          "1000 random descriptor updates (valid_tokens changes and format "
                          "changes transcoded on the device) before each sweep"),
    # Decode attention straight from the quantized blocks of the mixed cache: 32 query
    # heads over the 8 KV heads (Llama-3-8B's GQA group of 4), one query per sequence.
    "attn_mixed": dict(nseq=64, blocks=128, probs=(0.25, 0.5, 0.0, 0.25), scaling="weak",
                       attn=True, q_heads=32, l2="L2 flushed between launches (313 MB read per step)",
                       name="decode attention fused with dequant over the mixed cache: 64 seq x 2048 "
                            "tok, 8 KV heads x 128, 32 query heads, FP16 .25 / E4M3 .5 / INT4 .25"),
    # Decode attention over one layer of the long-context cache (config 5's shape: 16 seq x
    # 131072 tokens, INT4 .85 / E4M3 .10 / FP16 .05) with Llama-3-70B's 64 query heads:
    # few sequences, so each (sequence, KV head) is split over many CTAs.
    "attn_long": dict(nseq=16, blocks=8192, probs=(0.05, 0.10, 0.0, 0.85), scaling="strong",
                      attn=True, q_heads=64,
                      name="decode attention fused with dequant, long context: 16 seq x 131072 tok "
                           "(one layer), 8 KV heads x 128, 64 query heads, INT4 .85 / E4M3 .10 / FP16 .05"),
    # Decode attention over a serving-like batch of mixed lengths: 8 sequences of 16,384
    # tokens among 56 of 512 (mixed formats as 'mixed'), where one CTA per (sequence, KV head)
    # leaves most SMs idle while the long sequences finish.
    "attn_varied": dict(nseq=64, blocks=[1024] * 8 + [32] * 56, probs=(0.25, 0.5, 0.0, 0.25), scaling="weak",
                        attn=True, q_heads=32, l2="L2 flushed between launches",
                        name="decode attention fused with dequant, mixed lengths: 8 seq x 16384 tok + 56 seq x "
                             "512 tok, 8 KV heads x 128, 32 query heads, FP16 .25 / E4M3 .5 / INT4 .25"),
    # Config 1's data as one contiguous E4M3 array (8,388,608 values, 128-value groups):
    # the drop-in hlkv_dequantize_fp8_to_fp16 against the reference's own GPU kernel.
    "flat_e4m3": dict(n=8_388_608, group=128, fmt=1, scaling="weak", flat=True,
                      l2="L2 flushed between launches",
                      name="contiguous E4M3 -> FP16: 8,388,608 values (1 seq x 4096 tok x K+V x 8 "
                           "heads x 128), scale per 128 values; drop-in vs the reference's kernel"),
    # The same conversion at 2^28 values (805 MB moved, over 6x L2): the drop-in against the
    # reference's own kernel where bandwidth rather than launch latency sets the time.
    "flat_e4m3_large": dict(n=268_435_456, group=128, fmt=1, scaling="weak", flat=True,
                            l2="L2 flushed between launches",
                            name="contiguous E4M3 -> FP16: 268,435,456 values, scale per 128 values; "
                                 "drop-in vs the reference's kernel at a bandwidth-bound size"),
    # Decode step: every (sequence, layer) stream appends one token, encoded into its tail
    # block (kernel 2), and the allocator's descriptor delta is applied on the device
    # (kernel 3).  Sequences sharded over the ranks.
    "decode": dict(nseq=256, min_len=512, max_len=8192, layers=32, scaling="strong", decode=True,
                   name="decode-step append: 256 seq (lengths U[512, 8192]) x 32 layers, 8 KV heads "
                        "x 128, K+V; one N(0,1) FP16 token per seq-layer per step encoded into its "
                        "tail block (E4M3 or INT4 .5/.5, a new block every 16 tokens) + descriptor "
                        "delta applied on the device"),
    # The same step on short sequences (1-48 tokens): the same 8192 appends per step on
    # a cache of a few hundred MB, the case small enough for a full ncu capture.
    "decode_small": dict(nseq=256, min_len=1, max_len=48, layers=32, scaling="strong", decode=True,
                         name="decode-step append, short sequences: 256 seq (lengths U[1, 48]) x 32 "
                              "layers, 8 KV heads x 128, K+V; E4M3 or INT4 .5/.5 tail blocks"),
}


def measured_peak_gbs() -> tuple[float, str]:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def dist_env() -> tuple[int, int, int]:
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous share [lo, hi) of n sequences for `rank` of `world` ranks; shares differ
    by at most one sequence and cover 0..n-1 exactly once."""
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def cpu_model() -> str:
    """The host CPU's model name (the first "model name" of /proc/cpuinfo), for the CPU
    baseline's record."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


def max_over_ranks(values, world: int, device) -> list[float]:
    """Element-wise maximum of per-rank timings (all ranks take part; a no-op at world 1)."""
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


_SAMPLER = r"""
import sys, time
import pynvml
pynvml.nvmlInit()
h = pynvml.nvmlDeviceGetHandleByIndex(int(sys.argv[1]))
period = float(sys.argv[2])
out = open(sys.argv[3], "w", buffering=1)
print("max", pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM), file=out)
while True:
    try:
        mhz = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
        reasons = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
        print(time.time(), mhz, reasons, file=out)
    except pynvml.NVMLError:
        pass
    time.sleep(period)
"""


class TimedRange:
    """An NVTX push/pop range named "timed" around a timed region, so that a profiler's
    launch list can be restricted to it (ncu --nvtx --nvtx-include timed/)."""

    def __enter__(self):
        import torch
        torch.cuda.nvtx.range_push("timed")
        return self

    def __exit__(self, *exc):
        import torch
        torch.cuda.nvtx.range_pop()
        return False


class ClockSampler:
    """Samples SM clock and throttle reasons of one GPU through NVML in a child process
    (NVML calls made from the benchmarked process contend with its CUDA calls).  The
    child appends to a temporary file, so a long run never blocks it on a full pipe;
    __enter__ returns once the first sample is in.  Sample times are time.time();
    summary() takes the same clock."""

    def __init__(self, index: int, period_s: float = 0.02):
        # NVML enumerates all GPUs; map the CUDA index through CUDA_VISIBLE_DEVICES.
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        self.index = int(vis.split(",")[index]) if vis and vis.split(",")[0].isdigit() else index
        self.period = period_s
        self.samples: list[tuple[float, int, int]] = []
        self.max_mhz = None
        self._p = None
        self._path = None

    def _read(self) -> list[list[str]]:
        try:
            with open(self._path) as f:
                return [line.split() for line in f.read().splitlines()]
        except OSError:
            return []

    def __enter__(self):
        import subprocess
        import tempfile
        try:
            fd, self._path = tempfile.mkstemp(prefix="hlkv_clocks_", suffix=".txt")
            os.close(fd)
            self._p = subprocess.Popen([sys.executable, "-c", _SAMPLER, str(self.index), str(self.period),
                                        self._path], stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
            deadline = time.time() + 20.0
            while time.time() < deadline and self._p.poll() is None:
                if any(len(f) == 3 for f in self._read()):
                    break
                time.sleep(0.02)
        except Exception:
            self._p = None
        return self

    def __exit__(self, *exc):
        if self._p is None:
            return
        time.sleep(max(0.1, 3 * self.period))
        self._p.terminate()  # this child only, by its own handle
        try:
            self._p.wait(timeout=30)
        except Exception:
            pass
        for f in self._read():
            if len(f) == 2 and f[0] == "max":
                self.max_mhz = int(f[1])
            elif len(f) == 3:
                self.samples.append((float(f[0]), int(f[1]), int(f[2])))
        try:
            os.unlink(self._path)
        except OSError:
            pass

    def summary(self, t0: float, t1: float) -> dict:
        """Samples inside [t0, t1] (the timed region); a region shorter than three sample
        periods is widened to the whole sampled window (warm-up included)."""
        names = {0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
                 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
                 0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}
        inside = [s for s in self.samples if t0 <= s[0] <= t1]
        window = "timed region"
        if len(inside) < 3:
            inside = list(self.samples)
            window = "whole bench window (timed region shorter than 3 samples)"
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        reasons = sorted({n for _, _, r in inside for b, n in names.items() if r & b})
        return {"sm_mhz": statistics.median(m for _, m, _ in inside), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(inside), "window": window}


def traffic_from_profile(summary: str) -> int | None:
    """DRAM bytes (read + write) per launch of a kernel, from the committed ncu summary
    profiles/<summary>.md, or None.  The summary's table row "traffic (read + write) per
    launch" lists one capture per column, the current kernel last."""
    import re
    try:
        with open(os.path.join(ROOT, "profiles", f"{summary}.md")) as f:
            row = re.search(r"^\| traffic \(read \+ write\) per launch \|(.*)$", f.read(), re.M)
        cells = re.findall(r"([0-9,]+) B", row.group(1)) if row else []
        return int(cells[-1].replace(",", "")) if cells else None
    except OSError:
        return None


def static_config(workload: str, world: int) -> dict:
    """The `config` object of the JSON line: a description of the workload that both arms
    print identically (no measured or device-dependent values)."""
    spec = WORKLOADS[workload]
    cfg = {"workload": spec["name"], "key": workload, "scaling": spec["scaling"]}
    for k in ("layers", "nseq", "tokens", "updates", "q_heads"):
        if k in spec:
            cfg[{"nseq": "sequences", "tokens": "tokens_per_sequence"}.get(k, k)] = spec[k]
    cfg["l2"] = spec.get("l2", "a step's inputs and outputs exceed 4x the 126 MB L2: no flush needed")
    cfg["parallelism"] = (f"sequences sharded over {world} GPU(s), one process each, no collective "
                          "on the data path" if spec["scaling"] == "strong" else
                          f"one cache per GPU x{world}, no collective on the data path")
    return cfg


def sample_inputs(wl, rows):
    """Host copies of what the gather reads for the table sequences `rows` (indices into
    wl.seqs): the device descriptor table and arena as the kernel sees them, the rows'
    segments, and compact pools holding only the slots those blocks reference (their
    descriptors' slots renumbered into the compact pools; the decode does not depend on the
    slot number).  Keeps host memory to the sample's size on caches of tens of GB."""
    import numpy as np
    import torch
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from helpers import device_arena, device_table_words
    table = device_table_words(wl).copy()
    arena = device_arena(wl)
    segs = np.ascontiguousarray(wl.segs_host[rows], dtype=np.uint32).reshape(-1, 2)
    ids = np.concatenate([arena[o:o + n] for o, n in segs]) if len(segs) else np.zeros(0, np.uint32)
    pools = {}
    for f, (buf, sb, _) in wl.pools.items():
        sel = ids[(table[ids, 1] & 0xF) == f]
        if sel.size == 0:
            continue
        uniq, inv = np.unique(table[sel, 0], return_inverse=True)
        host = buf[torch.from_numpy(uniq.astype(np.int64)).to(buf.device)].cpu().numpy().reshape(-1)
        table[sel, 0] = inv.astype(np.uint32)
        pools[f] = (host, sb, int(uniq.size))
    return pools, table, arena, segs


def cpu_gather_sample(wl, rows, out_dev, out_first_elem: int, timed: bool, min_wall_s: float = 10.0,
                      max_reps: int = 5000):
    """The reference's CPU path (oracle/_ref: its dequantize_reference_to_fp16 per parameter
    group, walked through the same descriptor table) -- or the C restatement when the
    reference library is absent -- on the table sequences `rows`.  Its output is compared
    bit for bit with the GPU's output for the same sequences (out_dev from element
    out_first_elem on: `parity`); with `timed`, the gather is repeated on all host threads for
    about min_wall_s seconds (`cpu_baseline`)."""
    import numpy as np
    from oracle.oracle import Oracle, Ref, ref_available
    from hlkv.workload import block_bytes
    kind = "reference" if ref_available() else "port"
    impl = Ref() if kind == "reference" else Oracle()
    pools, table, arena, segs = sample_inputs(wl, rows)
    nblocks = int(segs[:, 1].sum())
    out = np.empty(max(1, nblocks * wl.block_elems), dtype=np.uint16)
    threads = os.cpu_count() or 1
    ids = np.concatenate([arena[o:o + n] for o, n in segs])
    nbytes = sum(block_bytes(int(table[i][1] & 0xF), wl.T, wl.H, wl.D, int((table[i][1] >> 10) & 0x3FF))
                 for i in ids)
    err = impl.gather_dequant(pools, wl.T, wl.H, wl.D, wl.layout.layout_id, table, arena, segs, out,
                              threads=threads)
    got = out_dev[out_first_elem:out_first_elem + nblocks * wl.block_elems].cpu().numpy().view(np.uint16)
    parity = {"ok": bool(err == 0 and np.array_equal(got, out[:nblocks * wl.block_elems])),
              "checked": f"{len(rows)} sequences ({nblocks} blocks, {nblocks * wl.block_elems} fp16 values) "
                         f"of the last launch's output against the reference's CPU gather ({kind}), "
                         "bit for bit",
              "differing_values": int(np.count_nonzero(got != out[:nblocks * wl.block_elems]))}
    if not timed:
        return parity, None
    reps, t0 = 0, time.perf_counter()
    while True:
        err = impl.gather_dequant(pools, wl.T, wl.H, wl.D, wl.layout.layout_id, table, arena, segs,
                                  out, threads=threads)
        reps += 1
        wall = time.perf_counter() - t0
        if wall >= min_wall_s or reps >= max_reps:
            break
    assert err == 0
    gbs = nbytes * reps / wall / 1e9
    return parity, {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "cpu_model": cpu_model(), "kind": kind,
                    "sample": f"{len(rows)} sequences of one layer ({nblocks} blocks, {nbytes / 1e6:.1f} MB "
                              f"algorithmic) x {reps} passes, {wall:.2f} s wall"}


def build_bench_workload(spec: dict, rank: int, world: int, spare_slots: int = 0):
    """This rank's cache: all spec["nseq"] sequences (weak scaling) or its contiguous
    share of them (strong scaling), for every layer; table sequences are layer-major."""
    from hlkv.workload import build_workload, mixed_formats, tiered_formats
    lo, hi = (0, spec["nseq"]) if spec["scaling"] == "weak" else shard_range(spec["nseq"], world, rank)
    n = hi - lo
    rows = []
    for layer in range(spec.get("layers", 1)):
        if "tiers" in spec:
            rows += tiered_formats(n, spec["tokens"], fp16_tokens=spec["tiers"][0],
                                   fp8_tokens=spec["tiers"][1])
        else:
            rows += mixed_formats(n, spec["blocks"], probs=spec["probs"],
                                  seed=1000 + rank + 7919 * layer)
    return build_workload(rows, seed=1000 + rank, spare_slots=spare_slots), n


def run_hlkv(args) -> None:
    import numpy as np
    import torch
    import torch.distributed as dist
    import hlkv
    from hlkv.workload import UpdateStream

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    spec = WORKLOADS[args.workload]
    layers = spec.get("layers", 1)
    e2e_steps = max(1, min(args.steps, args.e2e_steps if layers == 1 else min(args.e2e_steps, 4)))
    # Format changes take a slot in the target pool before the commit frees the old one.
    spare = spec.get("updates", 0) * (args.steps + args.warmup + e2e_steps + 3)
    t_build = time.perf_counter()
    wl, nseq_rank = build_bench_workload(spec, rank, world, spare)
    build_s = time.perf_counter() - t_build
    pools = wl.hlkv_pools()
    # One launch per layer per step, all into one FP16 scratch buffer of a layer's size.
    layer_segs = [wl.segs[l * nseq_rank:(l + 1) * nseq_rank] for l in range(layers)]
    layer_blocks = [int(wl.segs_host[l * nseq_rank:(l + 1) * nseq_rank, 1].sum()) for l in range(layers)]
    n_out = max(1, max(layer_blocks)) * wl.block_elems
    out = torch.empty(n_out, dtype=torch.int16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream()

    updates = UpdateStream(wl, spec["updates"], 5000 + rank) if spec.get("updates") else None
    moved = [0]  # algorithmic bytes of the steps run so far (updates change the sweep's bytes)
    host_update_s = [0.0]
    launches = [0]

    def prepare():
        """Host work of a step (table updates), outside the device-timed window."""
        if updates is not None:
            t0 = time.perf_counter()
            moved[0] += updates.prepare()
            host_update_s[0] += time.perf_counter() - t0

    def step():
        if updates is not None:
            launches[0] += updates.launch(stream, err)
        moved[0] += updates.sweep_bytes if updates is not None else wl.algorithmic_bytes
        # Each layer's launch overlaps its prologue with the previous gather's tail
        # (HLKV_LAUNCH_OVERLAP_PREVIOUS), except right after kernel (3), which writes the
        # tables the prologue reads.
        for i, segs in enumerate(layer_segs):
            hlkv.gather_dequant(pools, wl.layout, wl.dt.table_ptr, wl.dt.table_size,
                                wl.dt.arena_ptr, wl.dt.arena_size, segs, out, err, stream=stream,
                                overlap_previous=not args.no_overlap and (updates is None or i > 0))
        launches[0] += len(layer_segs)

    def barrier():
        if world > 1:
            dist.barrier()

    # Inputs + outputs smaller than a few L2 capacities would be served from L2 on the
    # next step: then a buffer of twice the L2 size is overwritten between steps and the
    # value is taken from the per-step events (the flush is not timed).
    l2_bytes = torch.cuda.get_device_properties(torch.cuda.current_device()).L2_cache_size
    flush = None
    if spec.get("flush"):
        flush = torch.empty(2 * l2_bytes, dtype=torch.uint8, device="cuda")
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clocks:
        for _ in range(args.warmup):
            prepare()
            step()
        torch.cuda.synchronize()
        assert int(err.item()) == 0, f"error bits {int(err.item()):#x}"
        barrier()
        torch.cuda.synchronize()
        moved[0] = 0
        host_update_s[0] = 0.0
        launches[0] = 0
        h0 = time.time()
        with TimedRange():
            t_start.record(stream)
            for k in range(args.steps):
                if flush is not None:
                    flush.fill_(k & 0xFF)
                prepare()
                ev[k][0].record(stream)
                step()
                ev[k][1].record(stream)
            t_end.record(stream)
        torch.cuda.synchronize()
        h1 = time.time()
        barrier()
    total_ms = t_start.elapsed_time(t_end)
    step_ms = [a.elapsed_time(b) for a, b in ev]
    bytes_per_step = moved[0] / args.steps
    timed_launches = launches[0]
    assert int(err.item()) == 0
    if flush is not None or updates is not None:
        # the timed work is the launches, not the flushes or the host table updates between them
        total_ms = sum(step_ms)
    total_ms, mean_step_ms, median_step_ms = max_over_ranks(
        [total_ms, statistics.mean(step_ms), statistics.median(step_ms)], world, "cuda")

    if spec["scaling"] == "weak":
        job_bytes = world * bytes_per_step
    else:  # strong: the ranks' shares add up to the whole cache
        (job_bytes,) = [int(x) for x in _sum_over_ranks([bytes_per_step], world)]
    value = job_bytes * args.steps / (total_ms / 1e3) / 1e9
    per_gpu = value / world
    peak, peak_kind = measured_peak_gbs()
    achieved = bytes_per_step / (mean_step_ms / 1e3) / 1e9
    mean_launch_ms = mean_step_ms / layers

    # Parity and the CPU baseline, outside every timed region: the reference's CPU gather
    # of the first sequences of the last layer (the last launch, whose output is still in
    # `out`), compared bit for bit with the GPU output; timed on all host threads at N=1.
    parity, cpu = None, None
    if rank == 0:
        k = min(spec.get("cpu_sample_seqs", 16), nseq_rank)
        rows = list(range((layers - 1) * nseq_rank, (layers - 1) * nseq_rank + k))
        parity, cpu = cpu_gather_sample(wl, rows, out, 0, timed=world == 1 and not args.no_cpu_baseline)

    e2e = measure_e2e(args, wl, layer_segs, nseq_rank, out, err, stream, world, e2e_steps, updates,
                      barrier)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(total_ms / args.steps, 5), "median_ms_per_step": round(median_step_ms, 5),
            "higher_is_better": True,
            "scaling": spec["scaling"], "vs_baseline": None, "dtype": "fp16 out; fp16/e4m3/int4 in",
            "data": "synthetic (seeded N(0,1) + outlier channels, quantized on the GPU)",
            "config": static_config(args.workload, world),
            "work": {"layers": layers, "sequences_per_gpu": nseq_rank,
                     "blocks_per_gpu": wl.total_blocks,
                     "blocks_per_format": {"fp16": wl.blocks_per_format[0],
                                           "e4m3": wl.blocks_per_format[1],
                                           "int4": wl.blocks_per_format[3]},
                     "bytes_per_step_per_gpu": round(bytes_per_step),
                     "updates_applied": updates.counts if updates is not None else None,
                     "host_update_ms_per_step": round(1e3 * host_update_s[0] / args.steps, 3)
                     if updates is not None else None,
                     "l2": ("L2 flushed between steps (%.0f MB overwritten); value from the per-step "
                            "events" % (2 * l2_bytes / 1e6)) if flush is not None else
                           ("no flush: %.0f MB of inputs+outputs per step against a %.0f MB L2" % (
                               bytes_per_step / 1e6, l2_bytes / 1e6)),
                     "build_s": round(build_s, 1)},
            "per_gpu_gbs": round(per_gpu, 2),
            "pct_hbm_peak": round(100 * per_gpu / peak, 2),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs, copy bandwidth)",
                         "traffic": traffic_from_profile("gather_dequant_" + (
                             "llama8b_layer" if args.workload == "llama8b" else args.workload) + "_full"),
                         "kernel": "gather_dequant_kernel<128>",
                         "launch_ms": round(mean_launch_ms, 5)},
            "parity": parity["ok"] if parity is not None else None,
            "parity_detail": parity,
            "e2e": e2e,
            "gpu_launches": timed_launches,  # gathers (+ transcode and delta with updates)
            "clocks": clocks.summary(h0, h1),
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_decode(args) -> None:
    """Decode-append step (kernel 2 + kernel 3) on a resident multi-layer cache."""
    import numpy as np
    import torch
    import torch.distributed as dist
    import hlkv

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    spec = WORKLOADS[args.workload]
    T, H, D, layers = 16, 8, 128, spec["layers"]
    lo, hi = shard_range(spec["nseq"], world, rank)
    lengths = np.random.default_rng(3000).integers(spec["min_len"], spec["max_len"] + 1,
                                                   size=spec["nseq"])[lo:hi]
    n = len(lengths) * layers  # streams: one table sequence per (layer, sequence), layer-major
    stream_len = np.tile(lengths, layers)
    rng = np.random.default_rng(3001 + rank)
    quant = np.array([hlkv.FP8_E4M3, hlkv.INT4], dtype=np.uint32)
    steps_total = args.warmup + args.steps
    split_steps = 8  # after the timed steps: the two kernels timed apart (an event between them)
    all_steps = steps_total + split_steps + 1  # + the parity step
    nb = -(-stream_len // T)
    init_fmt = rng.choice(quant, size=int(nb.sum()))
    new_fmt = rng.choice(quant, size=(all_steps, n)).astype(np.uint32)
    layout = hlkv.Layout(T, H, D, 1)
    extra = n * (all_steps // T + 2)
    slots = {int(f): int((init_fmt == f).sum()) + extra for f in quant}
    sbytes = {f: (hlkv.layout_slot_bytes(f, layout) + 15) // 16 * 16 for f in slots}
    t_build = time.perf_counter()
    table = hlkv.Table(int(nb.sum()) + 2 * extra, [(f, sbytes[f], slots[f]) for f in slots],
                       block_tokens=T)
    seqs, k = [], 0
    for j in range(n):
        st, s = table.create_sequence()
        assert st == 0
        seqs.append(s)
        tail_tokens = int(stream_len[j]) - T * (int(nb[j]) - 1)
        for b in range(int(nb[j])):
            st, _ = table.append_block(s, int(init_fmt[k]), T if b + 1 < nb[j] else tail_tokens, 1)
            assert st == 0, st
            k += 1
    tail_fmt = init_fmt[np.cumsum(nb) - 1].astype(np.uint32)
    handles = (hlkv.Handle * n)(*seqs)
    dt = hlkv.DeviceTables()
    dt.sync(table)
    pools_t = {f: (torch.empty((slots[f], sbytes[f]), dtype=torch.uint8, device="cuda"), sbytes[f],
                   slots[f]) for f in slots}
    pools = hlkv.make_pools(pools_t)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(3002 + rank)
    tokens = [torch.randn((n, 2, H, D), generator=gen, device="cuda").to(torch.float16)
              for _ in range(4)]
    pinned = [torch.empty((n, 2), dtype=torch.int32).pin_memory() for _ in range(2)]
    pinned_np = [p.numpy().view(np.uint32) for p in pinned]
    d_targets = [torch.empty((n, 2), dtype=torch.int32, device="cuda") for _ in range(2)]
    copied = [torch.cuda.Event() for _ in range(2)]
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream()
    torch.cuda.synchronize()
    build_s = time.perf_counter() - t_build

    rows_in = 2 * H * D * 2
    enc_out = {int(hlkv.FP8_E4M3): 2 * H * D + 2 * H * 4, int(hlkv.INT4): 2 * H * D // 2 + 2 * H * 8}
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps_total + split_steps)]
    for e in ev:  # torch creates the CUDA event at its first record
        e[0].record(stream)
        e[1].record(stream)
    host = {"table_s": 0.0, "sync_s": 0.0}
    nbytes = {"encode": 0, "delta": 0, "h2d": 0}

    def step(k: int, timed: bool, split: bool = False) -> None:
        nonlocal tail_fmt
        b = k & 1
        if k >= 2:
            copied[b].synchronize()  # the upload two steps back has read pinned[b]
        h0 = time.perf_counter()
        st, tg, done = table.append_tokens(handles, new_fmt[k], 1, out=pinned_np[b])
        assert st == 0 and done == n, (st, done)
        nd, ni = table.pending()
        h1 = time.perf_counter()
        dt.collect(table)  # host half of the delta protocol: nothing queued on the GPU yet
        h2 = time.perf_counter()
        # ev[k][0], kernel (3) with the delta and the targets, kernel (2): one native call,
        # which records ev[k][0] just before its first launch.  Kernel (2) overlaps kernel (3)'s
        # tail (programmatic serialization) unless ev[k][1] is recorded between them (split).
        hlkv.decode_step_queue(dt, pools, layout, pinned[b], d_targets[b], tokens[k % 4], err,
                               start_event=ev[k][0], encode_event=ev[k][1] if split else None,
                               stream=stream)
        ev[k][2].record(stream)
        copied[b].record(stream)
        tail_fmt = np.where(tg[:, 1] == 0, new_fmt[k], tail_fmt)
        if timed:
            host["table_s"] += h1 - h0
            host["sync_s"] += h2 - h1
            n8 = int((tail_fmt == hlkv.FP8_E4M3).sum())
            nbytes["encode"] += n * (rows_in + 16) + n8 * enc_out[1] + (n - n8) * enc_out[3]
            nbytes["delta"] += nd * 32 + ni * 12
            nbytes["h2d"] += n * 8 + nd * 16 + ni * 8  # targets + staged delta, read in place

    for k in range(args.warmup):
        step(k, False)
    torch.cuda.synchronize()
    assert int(err.item()) == 0, f"error bits {int(err.item()):#x}"
    with ClockSampler(torch.cuda.current_device()) as clocks:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        w0, c0 = time.perf_counter(), time.time()
        with TimedRange():
            for k in range(args.warmup, steps_total):
                step(k, True)
        torch.cuda.synchronize()
        w1, c1 = time.perf_counter(), time.time()
    assert int(err.item()) == 0, f"error bits {int(err.item()):#x}"
    for k in range(steps_total, steps_total + split_steps):
        step(k, False, split=True)
    torch.cuda.synchronize()
    assert int(err.item()) == 0, f"error bits {int(err.item()):#x}"
    dev_ms = [e[0].elapsed_time(e[2]) for e in ev[args.warmup:steps_total]]
    enc_ms = [e[1].elapsed_time(e[2]) for e in ev[steps_total:]]
    delta_ms = [e[0].elapsed_time(e[1]) for e in ev[steps_total:]]
    wall_ms = 1e3 * (w1 - w0)
    dev_total, enc_mean, delta_mean, wall_ms = max_over_ranks(
        [sum(dev_ms), statistics.mean(enc_ms), statistics.mean(delta_ms), wall_ms], world, "cuda")
    step_bytes = (nbytes["encode"] + nbytes["delta"]) / args.steps
    (job_bytes,) = _sum_over_ranks([step_bytes], world)
    value = job_bytes * args.steps / (dev_total / 1e3) / 1e9
    peak, peak_kind = measured_peak_gbs()
    achieved = nbytes["encode"] / args.steps / (enc_mean / 1e3) / 1e9

    # Parity, outside the timed region: one more step; the rows it wrote for a sample of
    # its targets (codes and parameters in the pools) against the reference's own
    # quantize_reference of the same tokens, bit for bit.
    parity = None
    if rank == 0:
        k = steps_total + split_steps
        b = k & 1
        copied[b].synchronize()
        st, tg, done = table.append_tokens(handles, new_fmt[k], 1, out=pinned_np[b])
        assert st == 0 and done == n
        dt.collect(table)
        hlkv.decode_step_queue(dt, pools, layout, pinned[b], d_targets[b], tokens[k % 4], err, stream=stream)
        torch.cuda.synchronize()
        parity = decode_parity(table, pools_t, tokens[k % 4], tg, T, H, D, layout, int(err.item()))

    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cpu = cpu_encode_sample(tokens[0], tail_fmt, H, D, n)
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(dev_total / args.steps, 5), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "fp16 in; e4m3/int4 out",
            "data": "synthetic (seeded lengths, formats and N(0,1) tokens)",
            "config": static_config(args.workload, world),
            "work": {"streams_per_gpu": n, "sequences_per_gpu": len(lengths),
                     "blocks_at_start": int(nb.sum()), "bytes_per_step_per_gpu": round(step_bytes),
                     "build_s": round(build_s, 1)},
            "us_per_step": {"device": round(1e3 * dev_total / args.steps, 2),
                            "encode_kernel": round(1e3 * enc_mean, 2),
                            "delta_upload_and_apply": round(1e3 * delta_mean, 2),
                            "split": f"device: the timed steps, kernel (2) overlapping kernel (3); "
                                     f"encode_kernel and delta_upload_and_apply: {split_steps} further "
                                     f"steps with an event between the two kernels",
                            "host_table_ops": round(1e6 * host["table_s"] / args.steps, 2),
                            "host_collect_delta": round(1e6 * host["sync_s"] / args.steps, 2),
                            "wall": round(1e3 * wall_ms / args.steps, 2)},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4),
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                         # the profiled launch (decode_small) encodes the same 8192 appends
                         "traffic": traffic_from_profile("append_encode_decode_small_full"),
                         "kernel": "append_encode_kernel<128>",
                         "launch_ms": round(enc_mean, 5)},
            "e2e": {"value": round(job_bytes * args.steps / (wall_ms / 1e3) / 1e9, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": round(nbytes["h2d"] / args.steps), "d2h_bytes_per_step": 0,
                    "path": "host table ops + collect_delta -> hlkv_decode_step_queue (H2D of "
                            "targets and delta -> apply_delta -> append_encode), wall clock per step "
                            "(tokens resident)"},
            "parity": parity["ok"] if parity is not None else None,
            "parity_detail": parity,
            "gpu_launches": 2 * args.steps,  # apply_delta + append_encode per step
            "clocks": clocks.summary(c0, c1),
            "cpu_baseline": cpu,
        }), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def decode_parity(table, pools_t, tokens, targets, T: int, H: int, D: int, layout, err_bits: int,
                  sample_size: int = 256) -> dict:
    """The rows a decode step wrote for a sample of its targets -- codes and parameters as
    the pools hold them -- against the reference's quantize_reference (oracle/_ref; the C
    restatement when the reference library is absent) of the same FP16 tokens."""
    import numpy as np
    import torch
    import hlkv
    from oracle.oracle import Oracle, Ref, ref_available
    kind = "reference" if ref_available() else "port"
    impl = Ref() if kind == "reference" else Oracle()
    n = targets.shape[0]
    sample = np.unique(np.linspace(0, n - 1, num=min(n, sample_size)).astype(np.int64))
    ids = targets[sample, 0]
    desc = np.array([table.device_descriptor(int(i)) for i in ids], np.uint32).reshape(-1, 4)
    fmts = desc[:, 1] & 0xF
    x = tokens[torch.from_numpy(sample).to(tokens.device)].float().cpu().numpy().reshape(-1, D)
    rows = x.shape[0]
    params = np.zeros((rows, 2), np.float32)
    codes = np.zeros((rows, D), np.uint8)
    rejected = impl.quantize_rows(np.repeat(fmts.astype(np.uint8), 2 * H), np.ascontiguousarray(x), params, codes,
                                  os.cpu_count() or 1)
    differing = 0
    for f in np.unique(fmts):
        sel = np.nonzero(fmts == f)[0]
        buf, sb, _ = pools_t[int(f)]
        slots = buf[torch.from_numpy(desc[sel, 0].astype(np.int64)).to(buf.device)].cpu().numpy()
        cb = D if f == hlkv.FP8_E4M3 else D // 2           # code bytes per row
        code_region = 2 * T * H * cb
        pw = 1 if f == hlkv.FP8_E4M3 else 2                # parameter words per row
        for j, t in enumerate(sel):
            tok = int(targets[sample[t], 1])
            for rr in range(2 * H):
                kv, h = divmod(rr, H)
                row = (kv * T + tok) * H + h
                r = t * 2 * H + rr
                got_codes = slots[j, row * cb:(row + 1) * cb]
                got_prm = slots[j, code_region + row * 4 * pw:code_region + (row + 1) * 4 * pw].view(np.uint32)
                want_prm = params[r, :pw].view(np.uint32)
                differing += int(not np.array_equal(got_codes, codes[r, :cb])) + int(not np.array_equal(got_prm, want_prm))
    ok = err_bits == 0 and rejected == 0 and differing == 0
    return {"ok": bool(ok), "differing_rows": differing,
            "checked": f"{len(sample)} of {n} targets of one more decode step ({rows} rows: codes and "
                       f"parameters in the pools) against quantize_reference ({kind}), bit for bit"}


def cpu_encode_sample(tokens, tail_fmt, H: int, D: int, n: int, min_wall_s: float = 10.0):
    """The reference's quantize_reference per row (oracle/_ref), on all host threads, over
    one step's tokens: n targets x 2*H rows of D values, in the formats of their blocks."""
    import numpy as np
    from oracle.oracle import Oracle, Ref, ref_available
    kind = "reference" if ref_available() else "port"
    impl = Ref() if kind == "reference" else Oracle()
    x = tokens.float().cpu().numpy().reshape(n * 2 * H, D)
    fm = np.repeat(tail_fmt.astype(np.uint8), 2 * H)
    params = np.zeros((x.shape[0], 2), np.float32)
    codes = np.zeros(x.shape, np.uint8)
    threads = os.cpu_count() or 1
    impl.quantize_rows(fm, x, params, codes, threads)
    reps, t0 = 0, time.perf_counter()
    while True:
        bad = impl.quantize_rows(fm, x, params, codes, threads)
        reps += 1
        wall = time.perf_counter() - t0
        if wall >= min_wall_s or reps >= 2000:
            break
    assert bad == 0
    n8 = int((tail_fmt == 1).sum())
    nbytes = n * (2 * H * D * 2 + 16) + n8 * (2 * H * D + 2 * H * 4) + (n - n8) * (H * D + 2 * H * 8)
    return {"value": round(nbytes * reps / wall / 1e9, 3), "unit": "GB/s", "cores": threads,
            "cpu_model": cpu_model(), "kind": kind,
            "sample": f"one step's {n} appended tokens ({x.shape[0]} rows of {D}) "
                                    f"x {reps} passes, {wall:.2f} s wall"}


def run_attention(args) -> None:
    """Decode attention over a whole cache per step: one launch, or with a split the kernel
    and a merge, or in balanced mode a prefix pass, the kernel and a merge."""
    import numpy as np
    import torch
    import torch.distributed as dist
    import hlkv
    from hlkv.workload import code_bytes, param_bytes

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    spec = WORKLOADS[args.workload]
    wl, nseq = build_bench_workload(spec, rank, world)
    qh, D = spec["q_heads"], wl.D
    gen = torch.Generator(device="cuda")
    gen.manual_seed(9000 + rank)
    q = torch.randn((nseq, qh, D), generator=gen, device="cuda").to(torch.float16)
    out = torch.empty((nseq, qh, D), dtype=torch.float16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    pools = wl.hlkv_pools()
    stream = torch.cuda.current_stream()
    scale = 1.0 / float(np.sqrt(D))

    # With at least two (sequence, KV head) units per SM the grid already fills the GPU and a
    # split only adds the merge; with fewer, each unit is split so that about 32 CTAs per SM
    # are launched (long sequences, few of them).
    # Uneven lengths (the longest sequence at least 1.5x the mean): the balanced mode over one
    # CTA per resident slot (4 per SM), since per-unit CTAs would leave SMs idle while the
    # long sequences finish (measured 0.195 ms against 0.696 ms unsplit, 0.226 ms at 16 splits).
    sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    units = nseq * wl.H
    auto = 1 if units >= 2 * sms else max(1, -(-32 * sms // units))
    splits = args.splits if args.splits else auto
    lens = wl.segs_host[:, 1].astype(np.float64)
    uneven = lens.size > 0 and lens.max() >= 1.5 * lens.mean()
    ctas = args.ctas if args.ctas else (4 * sms if uneven and not args.splits else 0)
    ws = None
    if ctas:
        # balanced: the units' blocks cut into `ctas` equal ranges
        ws = torch.empty(hlkv.decode_attention_balanced_workspace_bytes(nseq, wl.H, D, ctas), dtype=torch.uint8,
                         device="cuda")
    elif splits > 1:
        ws = torch.empty(hlkv.decode_attention_workspace_bytes(nseq, wl.H, D, splits), dtype=torch.uint8,
                         device="cuda")

    def step():
        if ctas:
            hlkv.decode_attention_balanced(pools, wl.layout, wl.dt.table_ptr, wl.dt.table_size, wl.dt.arena_ptr,
                                           wl.dt.arena_size, wl.segs, q, qh, scale, ctas, ws, out, err,
                                           stream=stream)
        else:
            hlkv.decode_attention_split(pools, wl.layout, wl.dt.table_ptr, wl.dt.table_size, wl.dt.arena_ptr,
                                        wl.dt.arena_size, wl.segs, q, qh, scale, splits, ws, out, err,
                                        stream=stream)

    # Algorithmic bytes: codes + row parameters of the K and V rows read, 20 B of descriptor
    # and arena entry per block, the queries read and the outputs written.
    rows, elems = 2 * wl.T * wl.H, wl.block_elems
    per_fmt = {f: code_bytes(f, elems) + param_bytes(f, rows) + 20 for f in (0, 1, 2, 3)}
    nbytes = sum(per_fmt[f] * n for f, n in wl.blocks_per_format.items()) + 2 * 2 * nseq * qh * D
    l2_bytes = torch.cuda.get_device_properties(torch.cuda.current_device()).L2_cache_size
    flush = torch.empty(2 * l2_bytes, dtype=torch.uint8, device="cuda") if nbytes < 4 * l2_bytes else None
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    with ClockSampler(torch.cuda.current_device()) as clocks:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        c0 = time.time()
        with TimedRange():
            for k in range(args.steps):
                if flush is not None:
                    flush.fill_(k & 0xFF)
                ev[k][0].record(stream)
                step()
                ev[k][1].record(stream)
        torch.cuda.synchronize()
        c1 = time.time()
    ms = [a.elapsed_time(b) for a, b in ev]
    total_ms, mean_ms = max_over_ranks([sum(ms), statistics.mean(ms)], world, "cuda")
    value = world * nbytes * args.steps / (total_ms / 1e3) / 1e9
    peak, peak_kind = measured_peak_gbs()
    tokens = wl.valid_tokens_total
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "fp16/e4m3/int4 KV in; fp32 math; fp16 out",
            "data": "synthetic (seeded N(0,1) + outlier channels; N(0,1) queries)",
            "config": static_config(args.workload, world),
            "work": {"bytes_per_step_per_gpu": nbytes,
                     "kv_tokens_per_step_per_gpu": tokens, "query_heads": qh,
                     "splits_per_sequence_head": None if ctas else splits,
                     "balanced_ctas": ctas or None,
                     "l2": "L2 flushed between launches" if flush is not None else "no flush needed"},
            "kv_tokens_per_s": round(world * tokens * args.steps / (total_ms / 1e3), 1),
            "roofline": {"bound": "hbm", "achieved": round(nbytes / (mean_ms / 1e3) / 1e9, 2), "peak": peak,
                         "unit": "GB/s", "frac": round(nbytes / (mean_ms / 1e3) / 1e9 / peak, 4),
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)", "traffic": None,
                         "kernel": f"decode_attention_kernel<128,{qh // wl.H}> (+ merge)",
                         "launch_ms": round(mean_ms, 5)},
            "e2e": {"value": None, "unit": "GB/s", "h2d_bytes_per_step": None, "d2h_bytes_per_step": None,
                    "reason": "the cache is resident in HBM; end to end is measured on 'mixed'"},
            "gpu_launches": args.steps * (3 if ctas else (2 if splits > 1 else 1)),  # prefix, kernel, merge
            "clocks": clocks.summary(c0, c1),
            "cpu_baseline": None,
        }), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_flat(args) -> None:
    """The flat FP8 -> FP16 drop-in and the reference's own kernel, on one contiguous array."""
    import numpy as np
    import torch
    import torch.distributed as dist
    import hlkv

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    spec = WORKLOADS[args.workload]
    n, group, fmt = spec["n"], spec["group"], spec["fmt"]
    ng = -(-n // group)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(7000 + rank)
    x = torch.randn(n, generator=gen, device="cuda").to(torch.float16).to(torch.float32)
    codes = torch.empty(n, dtype=torch.uint8, device="cuda")
    params = torch.empty((ng, 2), dtype=torch.float32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    hlkv.check(hlkv.quantize(fmt, x.data_ptr(), n, group, params.data_ptr(), ng, codes.data_ptr(), n,
                             err.data_ptr()), "quantize")
    del x
    out = torch.empty(n, dtype=torch.int16, device="cuda")
    out_ref = torch.empty(n, dtype=torch.int16, device="cuda")
    stream = torch.cuda.current_stream()
    ref = None
    try:
        from oracle.oracle import RefCuda
        ref = RefCuda()
    except Exception:
        ref = None

    def ours():
        hlkv.check(hlkv.dequantize_fp8_to_fp16(fmt, codes.data_ptr(), n, params.data_ptr(), group,
                                                out.data_ptr(), stream=stream), "dequantize_fp8_to_fp16")

    def theirs():
        assert ref.dequantize_fp8_to_fp16(fmt, codes.data_ptr(), n, params.data_ptr(), group,
                                          out_ref.data_ptr(), stream.cuda_stream) == 0

    # codes + one scale per group read, FP16 written
    nbytes = n + 4 * ng + 2 * n
    l2_bytes = torch.cuda.get_device_properties(torch.cuda.current_device()).L2_cache_size
    flush = torch.empty(2 * l2_bytes, dtype=torch.uint8, device="cuda")

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(args.steps)]
        for k in range(args.steps):
            flush.fill_(k & 0xFF)  # inputs and outputs fit in L2: evict them between launches
            ev[k][0].record(stream)
            fn()
            ev[k][1].record(stream)
        torch.cuda.synchronize()
        return [a.elapsed_time(b) for a, b in ev]

    with ClockSampler(torch.cuda.current_device()) as clocks:
        if world > 1:
            dist.barrier()
        c0 = time.time()
        with TimedRange():
            ms = timed(ours)
        c1 = time.time()
    total_ms, mean_ms = max_over_ranks([sum(ms), statistics.mean(ms)], world, "cuda")
    value = world * nbytes * args.steps / (total_ms / 1e3) / 1e9
    peak, peak_kind = measured_peak_gbs()
    achieved = nbytes / (mean_ms / 1e3) / 1e9
    ref_line = None
    if ref is not None:
        rms = timed(theirs)
        torch.cuda.synchronize()
        a = out.cpu().numpy().view(np.uint16)
        b = out_ref.cpu().numpy().view(np.uint16)
        nan = ((a & 0x7C00) == 0x7C00) & ((a & 0x3FF) != 0)
        same = bool(np.array_equal(a[~nan], b[~nan]))
        rmean = statistics.mean(rms)
        ref_line = {"kernel": "reference dequant_kernel.cu (fp8_to_fp16_vec8), built from its "
                              "source for sm_100a", "value": round(nbytes / (rmean / 1e3) / 1e9, 2),
                    "unit": "GB/s", "launch_ms": round(rmean, 5), "outputs_equal": same,
                    "speedup_of_drop_in": round(rmean / mean_ms, 3)}

    # End to end through the C ABI: codes and scales from pinned host memory, the kernel,
    # the FP16 output back into pinned host memory.
    e2e_steps = max(1, min(args.steps, args.e2e_steps))
    h_codes = codes.cpu().pin_memory()
    h_params = params.cpu().pin_memory()
    h_out = torch.empty(n, dtype=torch.int16).pin_memory()
    for k in range(e2e_steps + 1):
        if k == 1:
            torch.cuda.synchronize()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
        codes.copy_(h_codes, non_blocking=True)
        params.copy_(h_params, non_blocking=True)
        ours()
        h_out.copy_(out, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    (e2e_ms,) = max_over_ranks([e0.elapsed_time(e1)], world, "cuda")

    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cpu = cpu_flat_sample(h_codes.numpy(), h_params.numpy(), fmt, group)
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "e4m3 in; fp16 out", "data": "synthetic (seeded N(0,1), quantized on the GPU)",
            "config": static_config(args.workload, world),
            "work": {"bytes_per_step_per_gpu": nbytes,
                     "l2": "L2 flushed between launches (%.0f MB overwritten); value from the "
                           "per-launch events" % (2 * l2_bytes / 1e6)},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4),
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)", "traffic": None,
                         "kernel": "fp8_vec8 (hlkv_dequantize_fp8_to_fp16)", "launch_ms": round(mean_ms, 5)},
            "reference_gpu_kernel": ref_line,
            "e2e": {"value": round(world * nbytes * e2e_steps / (e2e_ms / 1e3) / 1e9, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": n + 8 * ng, "d2h_bytes_per_step": 2 * n,
                    "path": "pinned host codes + params -> H2D -> hlkv_dequantize_fp8_to_fp16 -> D2H"},
            "gpu_launches": args.steps,
            "clocks": clocks.summary(c0, c1),
            "cpu_baseline": cpu,
        }), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def cpu_flat_sample(codes, params, fmt: int, group: int, min_wall_s: float = 10.0):
    """The reference's dequantize_reference_to_fp16 (oracle/_ref) on one thread, over the
    first 1,048,576 values of the same array."""
    import numpy as np
    from oracle.oracle import Oracle, Ref, ref_available
    kind = "reference" if ref_available() else "port"
    impl = Ref() if kind == "reference" else Oracle()
    m = min(codes.size, 1 << 20)
    c = codes[:m].view(np.uint8)
    p = params[: -(-m // group)].view(np.float32).reshape(-1, 2)
    reps, t0 = 0, time.perf_counter()
    while True:
        st, _ = impl.dequantize_to_fp16(fmt, c, m, p, group)
        reps += 1
        wall = time.perf_counter() - t0
        if wall >= min_wall_s or reps >= 2000:
            break
    assert st == 0
    nbytes = m + 4 * p.shape[0] + 2 * m
    return {"value": round(nbytes * reps / wall / 1e9, 3), "unit": "GB/s", "cores": 1, "cpu_model": cpu_model(), "kind": kind,
            "sample": f"{m} of {codes.size} values x {reps} passes, {wall:.2f} s wall"}


def _sum_over_ranks(values, world: int):
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return t.tolist()


def measure_e2e(args, wl, layer_segs, nseq_rank, out, err, stream, world, e2e_steps, updates,
                barrier) -> dict:
    """End to end through the C ABI with host buffers.  The pools are the resident KV cache
    (they stay in HBM, as in a serving engine); every step
      * (with updates) runs the host table updates and their collect into pinned staging,
        which kernel (3) reads in place, plus the transcode jobs' upload,
      * uploads the step's segments of every layer from pinned host memory,
      * runs one gather per layer into one of two FP16 scratch buffers, and
      * reads each layer's FP16 output back into pinned host memory on a second stream,
        overlapping the next layer's gather (a layer's scratch is reused two layers later,
        after its readback).
    Timed with CUDA events from before the first upload to after the last readback."""
    import numpy as np
    import torch
    import hlkv
    layers = len(layer_segs)
    host_segs = wl.segs.cpu().pin_memory()
    dev_segs = torch.empty_like(wl.segs)
    dev_out = [out, torch.empty_like(out)]
    host_out = [torch.empty(out.numel(), dtype=torch.int16).pin_memory() for _ in range(2)]
    layer_elems = [int(s[:, 1].sum().item()) * wl.block_elems for s in layer_segs]
    s_out = torch.cuda.Stream()
    gathered = [torch.cuda.Event() for _ in range(2)]
    read_back = [torch.cuda.Event() for _ in range(2)]
    used = [False, False]
    pools = wl.hlkv_pools()
    staged = [0]
    moved = [0]

    def e2e_step() -> None:
        if updates is not None:
            nd, ni = wl.table.pending()
            moved[0] += updates.prepare()
            staged[0] += 16 * nd + 8 * ni + 32 * updates.n_jobs
        dev_segs.copy_(host_segs, non_blocking=True)
        if updates is not None:
            updates.launch(stream, err)
        moved[0] += updates.sweep_bytes if updates is not None else wl.algorithmic_bytes
        for l in range(layers):
            b = l & 1
            if used[b]:
                stream.wait_event(read_back[b])  # the readback of this scratch is done
            hlkv.gather_dequant(pools, wl.layout, wl.dt.table_ptr, wl.dt.table_size, wl.dt.arena_ptr,
                                wl.dt.arena_size, dev_segs[l * nseq_rank:(l + 1) * nseq_rank], dev_out[b],
                                err, stream=stream)
            gathered[b].record(stream)
            with torch.cuda.stream(s_out):
                s_out.wait_event(gathered[b])
                host_out[b][:layer_elems[l]].copy_(dev_out[b][:layer_elems[l]], non_blocking=True)
                read_back[b].record(s_out)
            used[b] = True

    e2e_step()
    torch.cuda.synchronize()
    barrier()
    staged[0] = 0
    moved[0] = 0
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    w0 = time.perf_counter()
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    s_out.wait_stream(stream)
    e1.record(s_out)  # after the last readback, which follows every other operation
    torch.cuda.synchronize()
    wall_s = time.perf_counter() - w0
    e2e_ms, wall_ms = max_over_ranks([e0.elapsed_time(e1), 1e3 * wall_s], world, "cuda")
    bytes_per_step = moved[0] / e2e_steps
    if world > 1 and WORKLOADS[args.workload]["scaling"] == "strong":
        (job_bytes,) = _sum_over_ranks([bytes_per_step], world)
    else:
        job_bytes = world * bytes_per_step
    e2e_value = job_bytes * e2e_steps / (max(e2e_ms, wall_ms) / 1e3) / 1e9
    last = (layers - 1) & 1
    ok_bits = np.array_equal(host_out[last][:layer_elems[-1]].numpy().view(np.uint16),
                             dev_out[last][:layer_elems[-1]].cpu().numpy().view(np.uint16))
    assert int(err.item()) == 0
    h2d = host_segs.numel() * 4 + staged[0] // e2e_steps
    d2h = 2 * sum(layer_elems)

    # The ceiling: plain pinned device-to-host copies of one layer's output, nothing else
    # running, on every rank at once (the ranks share the host's memory and PCIe root).
    barrier()
    c0 = torch.cuda.Event(enable_timing=True)
    c1 = torch.cuda.Event(enable_timing=True)
    reps = 3
    with torch.cuda.stream(s_out):
        c0.record(s_out)
        for _ in range(reps):
            host_out[0][:layer_elems[0]].copy_(dev_out[0][:layer_elems[0]], non_blocking=True)
        c1.record(s_out)
    torch.cuda.synchronize()
    (copy_ms,) = max_over_ranks([c0.elapsed_time(c1)], world, "cuda")
    ceiling = 2 * layer_elems[0] * reps / (copy_ms / 1e3) / 1e9
    return {"value": round(e2e_value, 2), "unit": "GB/s", "steps": e2e_steps,
            "per_gpu": round(e2e_value / world, 2),
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "ms_per_step": round(max(e2e_ms, wall_ms) / e2e_steps, 3),
            "d2h_gbs_per_gpu": round(d2h / (max(e2e_ms, wall_ms) / e2e_steps / 1e3) / 1e9, 2),
            "d2h_ceiling_gbs_per_gpu": round(ceiling, 2),
            "limit": "the device-to-host copy of every layer's FP16 output: d2h_gbs_per_gpu against "
                     "d2h_ceiling_gbs_per_gpu, plain pinned copies of the same size on all ranks at once",
            "path": ("host table updates + collect_delta (pinned staging read in place by kernel 3) -> "
                     if updates is not None else "") +
                    "pinned host segments -> H2D -> hlkv_gather_dequant per layer (pools resident "
                    "in HBM) -> D2H of every layer's FP16 output into pinned host memory, "
                    "overlapped with the next layer's gather",
            "readback_ok": bool(ok_bits)}


def _cpu_formats(spec: dict, nseq: int, seed: int) -> list:
    """Per-block formats of nseq sequences of one layer of the workload: the age tiers
    (oldest blocks INT4, then E4M3, the newest FP16) or a seeded draw from the mix."""
    import numpy as np
    if "tiers" in spec:
        nb = spec["tokens"] // 16
        n16, n8 = spec["tiers"][0] // 16, spec["tiers"][1] // 16
        row = np.array([3] * (nb - n16 - n8) + [1] * n8 + [0] * n16, dtype=np.uint8)
        return [row.copy() for _ in range(nseq)]
    blocks = spec["blocks"] if np.isscalar(spec["blocks"]) else int(np.mean(spec["blocks"]))
    rng = np.random.default_rng(seed + 1)
    p = np.asarray(spec["probs"], dtype=np.float64)
    return [rng.choice(np.arange(4, dtype=np.uint8), size=blocks, p=p / p.sum()) for _ in range(nseq)]


def run_reference(args) -> None:
    """The reference's CPU path on the host cores (rank 0 only)."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    from oracle.oracle import ref_available
    from oracle.cpu_workload import build_cpu_workload, time_cpu_gather
    spec = WORKLOADS[args.workload]
    kind = "reference" if ref_available() else "port"
    threads = os.cpu_count() or 1
    if spec.get("decode"):
        run_reference_decode(args, spec, kind, threads)
        return
    if spec.get("flat"):
        run_reference_flat(args, spec, kind, threads)
        return
    # Size the per-step sample so that warm-up + steps stay within about two minutes.
    budget_s = 120.0 / max(1, args.steps + args.warmup)
    wl = build_cpu_workload(kind, formats=_cpu_formats(spec, 1, 1000), seed=1000)
    per_seq_s = time_cpu_gather(wl, threads)[0]
    nseq = int(max(1, min(spec["nseq"], budget_s / max(per_seq_s, 1e-6))))
    wl = build_cpu_workload(kind, formats=_cpu_formats(spec, nseq, 1000), seed=1000)
    for _ in range(args.warmup):
        time_cpu_gather(wl, threads)
    times = [time_cpu_gather(wl, threads)[0] for _ in range(args.steps)]
    total = sum(times)
    value = wl["bytes"] * args.steps / total / 1e9
    sample = (f"{nseq} of {spec['nseq']} sequences of one layer ({wl['blocks']} blocks, "
              f"{wl['bytes'] / 1e6:.1f} MB algorithmic) per step")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * total / args.steps, 3), "higher_is_better": True,
        "scaling": spec["scaling"], "vs_baseline": None, "dtype": "fp16 out; fp16/e4m3/int4 in",
        "data": "synthetic (seeded N(0,1) + outlier channels, quantize_reference)",
        "config": static_config(args.workload, world),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "cpu_model": cpu_model(), "kind": kind,
                         "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


def run_reference_flat(args, spec: dict, kind: str, threads: int) -> None:
    """The reference's CPU dequantize_reference_to_fp16 over the whole contiguous array, in
    equal slices (whole parameter groups) on all host threads."""
    import numpy as np
    from concurrent.futures import ThreadPoolExecutor
    from oracle.oracle import Oracle, Ref
    impl = Ref() if kind == "reference" else Oracle()
    n, group, fmt = spec["n"], spec["group"], spec["fmt"]
    ng = -(-n // group)
    rng = np.random.default_rng(7000)
    x = rng.standard_normal(n).astype(np.float16).astype(np.float32)
    st, params, codes = impl.quantize(fmt, x, group)
    assert st == 0
    per = -(-ng // threads) * group
    slices = [(lo, min(n, lo + per)) for lo in range(0, n, per)]

    def one(sl):
        lo, hi = sl
        st, _ = impl.dequantize_to_fp16(fmt, codes[lo:hi], hi - lo, params[lo // group:-(-hi // group)], group)
        return st

    with ThreadPoolExecutor(max_workers=threads) as ex:
        for _ in range(args.warmup):
            assert all(s == 0 for s in ex.map(one, slices))
        times = []
        for _ in range(args.steps):
            t0 = time.perf_counter()
            assert all(s == 0 for s in ex.map(one, slices))
            times.append(time.perf_counter() - t0)
    nbytes = n + 4 * ng + 2 * n
    total = sum(times)
    value = nbytes * args.steps / total / 1e9
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s",
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * total / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "e4m3 in; fp16 out",
        "data": "synthetic (seeded N(0,1), quantize_reference)",
        "config": static_config(args.workload, world),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "cpu_model": cpu_model(), "kind": kind,
                         "sample": f"the whole array ({n} values) per step"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


def run_reference_decode(args, spec: dict, kind: str, threads: int) -> None:
    """The reference's CPU encode of one decode step (quantize_reference per row of every
    appended token, formats E4M3/INT4 .5/.5) on all host threads."""
    import numpy as np
    from oracle.oracle import Oracle, Ref
    impl = Ref() if kind == "reference" else Oracle()
    H, D = 8, 128
    n = spec["nseq"] * spec["layers"]
    rng = np.random.default_rng(3001)
    fmt = rng.choice(np.array([1, 3], np.uint8), size=n)
    x = rng.standard_normal((n * 2 * H, D)).astype(np.float16).astype(np.float32)
    fm = np.repeat(fmt, 2 * H)
    params = np.zeros((x.shape[0], 2), np.float32)
    codes = np.zeros(x.shape, np.uint8)
    for _ in range(args.warmup):
        impl.quantize_rows(fm, x, params, codes, threads)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        assert impl.quantize_rows(fm, x, params, codes, threads) == 0
        times.append(time.perf_counter() - t0)
    n8 = int((fmt == 1).sum())
    nbytes = n * (2 * H * D * 2 + 16) + n8 * (2 * H * D + 2 * H * 4) + (n - n8) * (H * D + 2 * H * 8)
    total = sum(times)
    value = nbytes * args.steps / total / 1e9
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s",
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * total / args.steps, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "fp16 in; e4m3/int4 out",
        "data": "synthetic (seeded N(0,1) tokens, formats .5/.5)",
        "config": static_config(args.workload, world),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "cpu_model": cpu_model(), "kind": kind,
                         "sample": f"one full step: {n} appended tokens ({x.shape[0]} rows of {D})"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["hlkv", "reference"], default="hlkv")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="llama8b")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-overlap", action="store_true",
                    help="gather workloads: launch every layer without programmatic dependent launch")
    ap.add_argument("--ctas", type=int, default=0,
                    help="attention workloads: balanced mode over this many CTAs (0 = balanced over 4 per SM "
                         "when sequence lengths are uneven, else split mode)")
    ap.add_argument("--splits", type=int, default=0,
                    help="attention workloads: CTAs per (sequence, KV head); 0 = none with >= 2 units per SM, else about 32 CTAs per SM")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "hlkv" and WORKLOADS[args.workload].get("decode"):
        run_decode(args)
        return
    if args.impl == "hlkv" and WORKLOADS[args.workload].get("attn"):
        run_attention(args)
        return
    if args.impl == "hlkv" and WORKLOADS[args.workload].get("flat"):
        run_flat(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_hlkv(args)


if __name__ == "__main__":
    main()

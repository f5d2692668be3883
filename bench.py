"""Benchmark of the heterogeneous KV gather-dequant path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl hlkv|reference]
                    [--workload mixed|homogeneous]

One step = one hlkv_gather_dequant launch over the whole workload of a GPU:
the mixed single-layer cache (64 sequences x 2048 tokens, 16-token blocks,
8 KV heads x 128, K and V; per-block format FP16 0.25 / E4M3 0.5 / INT4 0.25;
N(0,1) values with 4 outlier channels per head x20; block ids and slots
scattered by a seeded scramble).  Inputs and outputs (about 850 MB) exceed the
126 MB L2, so no flush is needed between steps.  With N GPUs (torchrun), each
rank holds its own cache of that size (weak scaling, sequences sharded, no
inter-GPU traffic); ranks meet only at barriers and at the max-over-ranks
reduction of the timings.

value = algorithmic bytes of all ranks / max-over-ranks device time, GB/s.
Algorithmic bytes per block = codes + row parameters read + 2*T*H*D*2 bytes
written + 20 bytes of descriptor and arena entry (131 092 / 99 348 / 83 988
bytes for FP16 / E4M3 / INT4 blocks).

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
    "mixed": dict(nseq=64, blocks=128, probs=(0.25, 0.5, 0.0, 0.25),
                  name="mixed-format single layer: 64 seq x 2048 tok, 16-tok blocks, 8 KV heads x 128, "
                       "K+V, FP16 .25 / E4M3 .5 / INT4 .25, N(0,1) + 4 outlier channels x20"),
    "homogeneous": dict(nseq=1, blocks=256, probs=(0.0, 1.0, 0.0, 0.0),
                        name="homogeneous E4M3: 1 seq x 4096 tok, 16-tok blocks, 8 KV heads x 128, K+V"),
    # Single-format caches of the mixed workload's size: per-format throughput.
    "fp16": dict(nseq=64, blocks=128, probs=(1.0, 0.0, 0.0, 0.0),
                 name="FP16 only: 64 seq x 2048 tok, 16-tok blocks, 8 KV heads x 128, K+V"),
    "e4m3": dict(nseq=64, blocks=128, probs=(0.0, 1.0, 0.0, 0.0),
                 name="E4M3 only: 64 seq x 2048 tok, 16-tok blocks, 8 KV heads x 128, K+V"),
    "int4": dict(nseq=64, blocks=128, probs=(0.0, 0.0, 0.0, 1.0),
                 name="INT4 only: 64 seq x 2048 tok, 16-tok blocks, 8 KV heads x 128, K+V"),
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


def max_over_ranks(values, world: int, device) -> list[float]:
    """Element-wise maximum of per-rank timings (all ranks take part; a no-op at world 1)."""
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


class ClockSampler:
    """Samples SM clock and throttle reasons of one GPU through NVML in a thread."""

    def __init__(self, index: int, period_s: float = 0.002):
        self.index, self.period = index, period_s
        self.samples: list[tuple[float, int, int]] = []
        self._stop = threading.Event()
        self._t = None
        self.max_mhz = None

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nv = None
            return self
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.samples.append((time.perf_counter(), mhz, reasons))
            except Exception:
                pass
            time.sleep(self.period)

    def __exit__(self, *exc):
        self._stop.set()
        if self._t is not None:
            self._t.join()

    def summary(self, t0: float, t1: float) -> dict:
        names = {0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
                 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
                 0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}
        inside = [s for s in self.samples if t0 <= s[0] <= t1]
        window = "timed"
        if len(inside) < 3:  # very short timed regions: widen to the neighbouring samples
            inside = [s for s in self.samples if t0 - 0.25 <= s[0] <= t1 + 0.25]
            window = "timed +-0.25 s"
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        reasons = sorted({n for _, _, r in inside for b, n in names.items() if r & b})
        return {"sm_mhz": statistics.median(m for _, m, _ in inside), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(inside), "window": window}


def traffic_from_profile(workload: str) -> int | None:
    """DRAM bytes (read + write) per launch of the gather kernel, from the committed ncu
    summary of the same workload (profiles/gather_dequant_<workload>_full.md), or None."""
    import re
    try:
        with open(os.path.join(ROOT, "profiles", f"gather_dequant_{workload}_full.md")) as f:
            m = re.search(r"traffic \(read \+ write\) per launch \| ([0-9,]+) B", f.read())
        return int(m.group(1).replace(",", "")) if m else None
    except OSError:
        return None


def cpu_gather_sample(wl, nseq_sample: int, min_wall_s: float = 2.0, max_reps: int = 20):
    """Times the reference's CPU path (oracle/_ref) -- or the C restatement when the reference
    library is absent -- on host copies of the first nseq_sample sequences."""
    import numpy as np
    from oracle.oracle import Oracle, Ref, ref_available
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from helpers import device_arena, device_table_words, host_pools
    kind = "reference" if ref_available() else "port"
    impl = Ref() if kind == "reference" else Oracle()
    segs = wl.segs_host[:nseq_sample]
    nblocks = int(segs[:, 1].sum())
    out = np.empty(nblocks * wl.block_elems, dtype=np.uint16)
    pools, table, arena = host_pools(wl), device_table_words(wl), device_arena(wl)
    threads = os.cpu_count() or 1
    from hlkv.workload import block_bytes
    ids = [arena[o:o + n] for o, n in segs]
    nbytes = sum(block_bytes(int(table[i][1] & 0xF), wl.T, wl.H, wl.D, int((table[i][1] >> 10) & 0x3FF))
                 for row in ids for i in row)
    impl.gather_dequant(pools, wl.T, wl.H, wl.D, wl.layout.layout_id, table, arena, segs, out,
                        threads=threads)  # warm-up
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
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": kind,
            "sample": f"{nseq_sample} of {len(wl.segs_host)} sequences ({nblocks} blocks, "
                      f"{nbytes / 1e6:.1f} MB algorithmic) x {reps} passes, {wall:.2f} s wall"}


def run_hlkv(args) -> None:
    import numpy as np
    import torch
    import torch.distributed as dist
    import hlkv
    from hlkv.workload import build_workload, mixed_formats

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    spec = WORKLOADS[args.workload]
    fm = mixed_formats(spec["nseq"], spec["blocks"], probs=spec["probs"], seed=1000 + rank)
    wl = build_workload(fm, seed=1000 + rank)
    pools = wl.hlkv_pools()
    n_out = wl.total_blocks * wl.block_elems
    out = torch.empty(n_out, dtype=torch.int16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream()

    def step():
        hlkv.gather_dequant(pools, wl.layout, wl.dt.table_ptr, wl.dt.table_size, wl.dt.arena_ptr,
                            wl.dt.arena_size, wl.segs, out, err, stream=stream)

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    assert int(err.item()) == 0, f"error bits {int(err.item()):#x}"

    # Inputs + outputs smaller than a few L2 capacities would be served from L2 on the
    # next step: then a buffer of twice the L2 size is overwritten between steps and the
    # value is taken from the per-launch events (the flush is not timed).
    l2_bytes = torch.cuda.get_device_properties(torch.cuda.current_device()).L2_cache_size
    flush = None
    if wl.algorithmic_bytes < 4 * l2_bytes:
        flush = torch.empty(2 * l2_bytes, dtype=torch.uint8, device="cuda")
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clocks:
        barrier()
        torch.cuda.synchronize()
        h0 = time.perf_counter()
        t_start.record(stream)
        for k in range(args.steps):
            if flush is not None:
                flush.fill_(k & 0xFF)
            ev[k][0].record(stream)
            step()
            ev[k][1].record(stream)
        t_end.record(stream)
        torch.cuda.synchronize()
        h1 = time.perf_counter()
        barrier()
    total_ms = t_start.elapsed_time(t_end)
    launch_ms = [a.elapsed_time(b) for a, b in ev]
    assert int(err.item()) == 0
    if flush is not None:  # the timed work is the launches, not the flushes between them
        total_ms = sum(launch_ms)
    total_ms, mean_launch_ms = max_over_ranks([total_ms, statistics.mean(launch_ms)], world, "cuda")

    bytes_per_step = wl.algorithmic_bytes
    value = world * bytes_per_step * args.steps / (total_ms / 1e3) / 1e9
    per_gpu = value / world
    peak, peak_kind = measured_peak_gbs()
    achieved = bytes_per_step / (mean_launch_ms / 1e3) / 1e9

    # End to end through the C ABI with host buffers: every step uploads the pools and
    # segments from pinned host memory, syncs the (unchanged) device tables, runs the
    # gather and reads the FP16 output back into pinned host memory.  Steps alternate
    # between two sets of device buffers on an upload stream and a readback stream, so
    # that one step's upload overlaps the previous step's readback (PCIe is full
    # duplex); every step still moves all of its bytes in both directions.
    e2e_steps = max(1, min(args.steps, args.e2e_steps))
    host_pools = {f: buf.cpu().pin_memory() for f, (buf, _, _) in wl.pools.items()}
    host_segs = wl.segs.cpu().pin_memory()
    host_out = [torch.empty(n_out, dtype=torch.int16).pin_memory() for _ in range(2)]
    h2d = sum(p.numel() for p in host_pools.values()) + host_segs.numel() * 4
    d2h = n_out * 2
    dev_pools = [wl.pools, {f: (torch.empty_like(buf), sb, ns) for f, (buf, sb, ns) in wl.pools.items()}]
    dev_segs = [wl.segs, torch.empty_like(wl.segs)]
    dev_out = [out, torch.empty_like(out)]
    hl_pools = [hlkv.make_pools(dp) for dp in dev_pools]
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    uploaded = [torch.cuda.Event() for _ in range(2)]
    gathered = [torch.cuda.Event() for _ in range(2)]
    read_back = [torch.cuda.Event() for _ in range(2)]
    used = [False, False]

    def e2e_step(k: int) -> None:
        b = k & 1
        with torch.cuda.stream(s_in):
            if used[b]:
                s_in.wait_event(gathered[b])  # the gather two steps back has read pools[b]
            for f, (buf, _, _) in dev_pools[b].items():
                buf.copy_(host_pools[f], non_blocking=True)
            dev_segs[b].copy_(host_segs, non_blocking=True)
            uploaded[b].record(s_in)
        stream.wait_event(uploaded[b])
        if used[b]:
            stream.wait_event(read_back[b])  # out[b] of two steps back has been read back
        wl.dt.sync(wl.table, stream)
        hlkv.gather_dequant(hl_pools[b], wl.layout, wl.dt.table_ptr, wl.dt.table_size,
                            wl.dt.arena_ptr, wl.dt.arena_size, dev_segs[b], dev_out[b], err,
                            stream=stream)
        gathered[b].record(stream)
        with torch.cuda.stream(s_out):
            s_out.wait_event(gathered[b])
            host_out[b].copy_(dev_out[b], non_blocking=True)
            read_back[b].record(s_out)
        used[b] = True

    e2e_step(0)
    e2e_step(1)
    torch.cuda.synchronize()
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    s_in.wait_event(e0)
    s_out.wait_event(e0)
    for k in range(e2e_steps):
        e2e_step(k)
    e1.record(s_out)  # after the last readback, which follows every other operation
    torch.cuda.synchronize()
    (e2e_ms,) = max_over_ranks([e0.elapsed_time(e1)], world, "cuda")
    e2e_value = world * bytes_per_step * e2e_steps / (e2e_ms / 1e3) / 1e9
    last = (e2e_steps - 1) & 1
    ok_bits = np.array_equal(host_out[last].numpy().view(np.uint16),
                             dev_out[last].cpu().numpy().view(np.uint16))
    assert int(err.item()) == 0

    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cpu = cpu_gather_sample(wl, nseq_sample=min(16, len(wl.segs_host)))

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(total_ms / args.steps, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp16 out; fp16/e4m3/int4 in",
            "data": "synthetic (seeded N(0,1) + outlier channels, quantized on the GPU)",
            "config": {"workload": spec["name"], "blocks_per_gpu": wl.total_blocks,
                       "blocks_per_format": {"fp16": wl.blocks_per_format[0],
                                             "e4m3": wl.blocks_per_format[1],
                                             "int4": wl.blocks_per_format[3]},
                       "bytes_per_step_per_gpu": bytes_per_step,
                       "l2": ("inputs+outputs (%.0f MB) exceed 4x the %.0f MB L2; no flush" % (
                           bytes_per_step / 1e6, l2_bytes / 1e6)) if flush is None else
                             ("L2 flushed between steps (%.0f MB overwritten); value from the "
                              "per-launch events" % (2 * l2_bytes / 1e6)),
                       "parallelism": f"sequence-sharded x{world}, no collective on the data path"},
            "per_gpu_gbs": round(per_gpu, 2),
            "pct_hbm_peak": round(100 * per_gpu / peak, 2),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak,
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                         "traffic": traffic_from_profile(args.workload),
                         "kernel": "gather_dequant_kernel<128>", "launch_ms": round(mean_launch_ms, 5)},
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "steps": e2e_steps,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "path": "pinned host pools+segments -> H2D -> device-table sync -> "
                            "hlkv_gather_dequant -> D2H of the FP16 output; two buffer sets, "
                            "upload of step k overlaps readback of step k-1", "readback_ok": ok_bits},
            "gpu_launches": args.steps,  # gather launches in the timed region
            "clocks": clocks.summary(h0, h1),
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


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
    # Size the per-step sample so that warm-up + steps stay within about two minutes.
    budget_s = 120.0 / max(1, args.steps + args.warmup)
    wl = build_cpu_workload(kind, nseq=1, blocks=spec["blocks"], probs=spec["probs"], seed=1000)
    per_seq_s = time_cpu_gather(wl, threads)[0]
    nseq = int(max(1, min(spec["nseq"], budget_s / max(per_seq_s, 1e-6))))
    wl = build_cpu_workload(kind, nseq=nseq, blocks=spec["blocks"], probs=spec["probs"], seed=1000)
    for _ in range(args.warmup):
        time_cpu_gather(wl, threads)
    times = [time_cpu_gather(wl, threads)[0] for _ in range(args.steps)]
    total = sum(times)
    value = wl["bytes"] * args.steps / total / 1e9
    sample = (f"{nseq} of {spec['nseq']} sequences ({wl['blocks']} blocks, "
              f"{wl['bytes'] / 1e6:.1f} MB algorithmic) per step")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * total / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp16 out; fp16/e4m3/int4 in",
        "data": "synthetic (seeded N(0,1) + outlier channels, quantize_reference)",
        "config": {"workload": spec["name"], "parallelism": f"{threads} host threads"},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": kind,
                         "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["hlkv", "reference"], default="hlkv")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="mixed")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_hlkv(args)


if __name__ == "__main__":
    main()

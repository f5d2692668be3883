"""Multi-rank host logic on CPU (gloo, world size 2): the sequence sharding and the
max-over-ranks timing that bench.py uses on N GPUs.  Sequences are independent units
of the gather, so the ranks' shards gathered separately must equal the unsharded
gather byte for byte (checked with the oracle; no GPU involved)."""
import os
import socket
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_shard_range_covers_every_sequence_once():
    sys.path.insert(0, ROOT)
    from bench import shard_range
    for n in (0, 1, 2, 7, 16, 64, 255):
        for world in (1, 2, 3, 4, 8):
            ranges = [shard_range(n, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == n
            for (lo, hi), (lo2, _) in zip(ranges, ranges[1:]):
                assert hi == lo2 and lo <= hi
            sizes = [hi - lo for lo, hi in ranges]
            assert max(sizes) - min(sizes) <= 1


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, q) -> None:
    import torch
    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    from bench import max_over_ranks, shard_range
    from oracle.cpu_workload import build_cpu_workload
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        # Every rank builds the same seeded cache and gathers only its own sequences.
        wl = build_cpu_workload("port", nseq=7, blocks=5, probs=(0.25, 0.5, 0.0, 0.25), seed=5,
                                T=4, H=2, D=64)
        lo, hi = shard_range(wl["segs"].shape[0], world, rank)
        elems = 2 * wl["T"] * wl["H"] * wl["D"]
        n_out = int(wl["segs"][lo:hi, 1].sum()) * elems
        out = np.full(max(1, n_out), 0xAAAA, dtype=np.uint16)
        err = wl["oracle"].gather_dequant(wl["pools"], wl["T"], wl["H"], wl["D"], 1, wl["table"],
                                          wl["arena"], wl["segs"][lo:hi], out)
        parts = [None] * world
        dist.all_gather_object(parts, (lo, hi, int(err), out[:n_out].tobytes()))
        # Timings: each rank reports its own; every rank must see the maximum.
        mx = max_over_ranks([1.0 + rank, 10.0 - rank], world, "cpu")
        if rank == 0:
            full = np.full(wl["blocks"] * elems, 0x5555, dtype=np.uint16)
            ferr = wl["oracle"].gather_dequant(wl["pools"], wl["T"], wl["H"], wl["D"], 1,
                                               wl["table"], wl["arena"], wl["segs"], full)
            joined = b"".join(p[3] for p in sorted(parts))
            q.put((ferr, [p[2] for p in parts], joined == full.tobytes(),
                   [p[:2] for p in sorted(parts)], mx))
        else:
            q.put(("rank", rank, mx))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_sharded_gather_equals_unsharded_gloo_two_ranks(oracle):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = [q.get(timeout=240) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    main = next(g for g in got if g[0] != "rank")
    other = next(g for g in got if g[0] == "rank")
    ferr, errs, equal, ranges, mx = main
    assert ferr == 0 and errs == [0, 0]
    assert ranges == [(0, 4), (4, 7)]
    assert equal, "sharded gather differs from the unsharded gather"
    assert mx == [2.0, 10.0] and other[2] == [2.0, 10.0]

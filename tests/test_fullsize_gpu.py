"""Full-size parity on the three large configurations, every byte against the oracle.

* Decode-step append (256 sequences of U[512, 8192] tokens x 32 layers = 8192 streams,
  E4M3/INT4 tail blocks, N(0,1) tokens): three steps through hlkv_decode_step_queue
  (kernel 3 with the step's delta and targets, then kernel 2).  After each step the
  targets' slots equal the oracle's append (orc_append_encode, the reference's
  quantize_reference per row) of the same tokens into the same bytes, and the device
  descriptors of every target block equal the host table's device_descriptor.  At the
  end every slot no step wrote is still all zeros, so every pool byte is accounted for.
* One layer of the Llama-3-8B-shaped cache (64 x 8192 tokens, newest 512 FP16, the
  previous 2048 E4M3, the rest INT4): the gather equals the oracle's on all
  1,073,741,824 values.
* One layer of the long-context cache (16 x 131072 tokens, INT4 .85 / E4M3 .10 / FP16
  .05) after two batches of 1000 random descriptor updates (valid tokens and format
  changes transcoded on the device): after each batch every pool byte equals the oracle's
  transcode of the bytes before it and the device tables equal the host table; the final
  gather equals the oracle's, compared in chunks of sequences.

Each test frees its device memory before the next one starts (the decode cache alone
holds about 57 GB).
"""
import gc

import numpy as np
import pytest

from helpers import assert_bits_equal, d2h, device_arena, device_table_words

pytestmark = pytest.mark.gpu


def _free():
    import torch
    gc.collect()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


def _host_descriptors(table, ids) -> np.ndarray:
    return np.array([table.device_descriptor(int(i)) for i in ids], dtype=np.uint32).reshape(-1, 4)


def _slot_rows(pool_t, slots) -> np.ndarray:
    """Host copy of the given slots of a device pool tensor [num_slots, slot_bytes]."""
    import torch
    idx = torch.from_numpy(np.asarray(slots, dtype=np.int64)).to(pool_t.device)
    return pool_t[idx].cpu().numpy()


def test_decode_step_full_size(hlkv_lib, oracle, cuda_device):
    """Three decode steps on the full decode-append workload: 256 sequences with seeded
    lengths U[512, 8192] x 32 layers, 8 KV heads x 128, K and V."""
    import torch
    hlkv = hlkv_lib
    T, H, D, layers, nseq_total = 16, 8, 128, 32, 256
    lengths = np.random.default_rng(3000).integers(512, 8193, size=nseq_total)
    stream_len = np.tile(lengths, layers)
    n = stream_len.size
    rng = np.random.default_rng(3001)
    quant = np.array([hlkv.FP8_E4M3, hlkv.INT4], dtype=np.uint32)
    steps = 3
    nb = -(-stream_len // T)
    init_fmt = rng.choice(quant, size=int(nb.sum()))
    layout = hlkv.Layout(T, H, D, 1)
    extra = n * (steps // T + 2)
    slots = {int(f): int((init_fmt == f).sum()) + extra for f in quant}
    sbytes = {f: (hlkv.layout_slot_bytes(f, layout) + 15) // 16 * 16 for f in slots}
    table = hlkv.Table(int(nb.sum()) + 2 * extra, [(f, sbytes[f], slots[f]) for f in slots], block_tokens=T)
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
    handles = (hlkv.Handle * n)(*seqs)
    dt = hlkv.DeviceTables()
    dt.sync(table)
    pools_t = {f: torch.zeros((slots[f], sbytes[f]), dtype=torch.uint8, device="cuda") for f in slots}
    pools = hlkv.make_pools({f: (pools_t[f], sbytes[f], slots[f]) for f in slots})
    h_targets = torch.empty((n, 2), dtype=torch.int32).pin_memory()
    d_targets = torch.empty((n, 2), dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    touched = {f: set() for f in slots}
    for step in range(steps):
        new_fmt = rng.choice(quant, size=n).astype(np.uint32)
        st, tg, done = table.append_tokens(handles, new_fmt, 1, out=h_targets.numpy().view(np.uint32))
        assert st == 0 and done == n
        targets = tg.copy()
        desc = _host_descriptors(table, targets[:, 0])  # the step's descriptors, slots included
        tokens = np.random.default_rng(4000 + step).standard_normal((n, 2, H, D)).astype(np.float16)
        # The targets' slots before the step, compacted: slot numbers renumbered per format.
        before, tab = {}, np.zeros((table.max_blocks(), 4), np.uint32)
        tab[targets[:, 0]] = desc
        used_slots = {}
        for f in slots:
            sel = np.nonzero((desc[:, 1] & 0xF) == f)[0]
            uniq, inv = np.unique(desc[sel, 0], return_inverse=True)
            used_slots[f] = uniq
            touched[f].update(int(s) for s in uniq)
            tab[targets[sel, 0], 0] = inv
            before[f] = (np.ascontiguousarray(_slot_rows(pools_t[f], uniq)).reshape(-1), sbytes[f], uniq.size)
        dt.collect(table)
        hlkv.decode_step_queue(dt, pools, layout, h_targets, d_targets,
                               torch.from_numpy(tokens.view(np.int16)).cuda(), err)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        assert np.array_equal(d_targets.cpu().numpy().view(np.uint32), targets)
        dev_tab = d2h(dt.table_ptr, dt.table_size * 16).view(np.uint32).reshape(-1, 4)
        assert np.array_equal(dev_tab[targets[:, 0]], desc), f"step {step}: device descriptors"
        oerr = oracle.append_encode(before, T, H, D, 1, tab, targets, tokens.view(np.uint16))
        assert oerr == 0
        for f in slots:
            after = _slot_rows(pools_t[f], used_slots[f]).reshape(-1)
            bad = np.nonzero(after != before[f][0])[0]
            assert bad.size == 0, f"step {step} format {f}: {bad.size} bytes differ, first at {bad[:4]}"
    # Every slot no step wrote is untouched (all zeros).
    for f in slots:
        written = torch.zeros(slots[f], dtype=torch.bool)
        written[torch.tensor(sorted(touched[f]), dtype=torch.int64)] = True
        nonzero = torch.zeros(slots[f], dtype=torch.bool)
        for s0 in range(0, slots[f], 1 << 16):
            nonzero[s0:s0 + (1 << 16)] = (pools_t[f][s0:s0 + (1 << 16)] != 0).any(dim=1).cpu()
        stray = torch.nonzero(nonzero & ~written).flatten()
        assert stray.numel() == 0, f"format {f}: {stray.numel()} untouched slots were written"
    dt.close()
    del pools_t, pools, table
    _free()


def _gather_layer(hlkv, wl, out):
    import torch
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    hlkv.gather_dequant(wl.hlkv_pools(), wl.layout, wl.dt.table_ptr, wl.dt.table_size,
                        wl.dt.arena_ptr, wl.dt.arena_size, wl.segs, out, err)
    torch.cuda.synchronize()
    return int(err.item())


def _compare_in_chunks(oracle, wl, out, chunk_seqs: int, pools_host=None):
    """The oracle's gather of chunk_seqs sequences at a time against the matching slice of
    the device output (packed, in sequence order)."""
    from helpers import host_pools
    import os
    pools = host_pools(wl) if pools_host is None else pools_host
    table, arena = device_table_words(wl), device_arena(wl)
    first = 0
    for s0 in range(0, len(wl.segs_host), chunk_seqs):
        segs = np.ascontiguousarray(wl.segs_host[s0:s0 + chunk_seqs])
        n = int(segs[:, 1].sum()) * wl.block_elems
        want = np.empty(max(n, 1), np.uint16)
        oerr = oracle.gather_dequant(pools, wl.T, wl.H, wl.D, wl.layout.layout_id, table, arena, segs,
                                     want, threads=os.cpu_count() or 8)
        assert oerr == 0
        got = out[first:first + n].cpu().numpy().view(np.uint16)
        assert_bits_equal(got, want[:n], f"sequences {s0}..{s0 + len(segs) - 1}")
        first += n
    assert first == wl.total_blocks * wl.block_elems


def test_llama8b_layer_full_size(hlkv_lib, oracle, cuda_device):
    """One layer of the Llama-3-8B-shaped cache: 64 sequences x 8192 tokens, age tiers."""
    import torch
    from hlkv.workload import build_workload, tiered_formats
    wl = build_workload(tiered_formats(64, 8192, fp16_tokens=512, fp8_tokens=2048), seed=1000)
    assert wl.blocks_per_format[0] == 64 * 32 and wl.blocks_per_format[1] == 64 * 128
    assert wl.blocks_per_format[3] == 64 * 352
    out = torch.empty(wl.total_blocks * wl.block_elems, dtype=torch.int16, device="cuda")
    assert _gather_layer(hlkv_lib, wl, out) == 0
    _compare_in_chunks(oracle, wl, out, chunk_seqs=16)
    wl.dt.close()
    del out, wl
    _free()


def test_long_context_layer_after_updates(hlkv_lib, oracle, cuda_device):
    """One layer of the long-context cache (16 x 131072 tokens, INT4 .85 / E4M3 .10 / FP16
    .05) after two batches of 1000 random descriptor updates."""
    import torch
    from helpers import host_pools
    from hlkv.workload import UpdateStream, build_workload, host_table, mixed_formats
    fm = mixed_formats(16, 8192, probs=(0.05, 0.10, 0.0, 0.85), seed=1000)
    wl = build_workload(fm, seed=1000, spare_slots=2 * 1000 + 8)
    up = UpdateStream(wl, 1000, seed=5000)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream()
    for batch in range(2):
        before = host_pools(wl)
        up.prepare()
        jobs = up.jobs_np[:up.n_jobs].copy()
        assert up.n_jobs > 300  # about half the updates change a format
        up.launch(stream, err)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        oerr = oracle.transcode(before, wl.T, wl.H, wl.D, jobs)
        assert oerr == 0
        after = host_pools(wl)
        for f in before:
            bad = np.nonzero(after[f][0] != before[f][0])[0]
            assert bad.size == 0, f"batch {batch} format {f}: {bad.size} bytes differ, first at {bad[:4]}"
        del before
        assert np.array_equal(device_table_words(wl), host_table(wl)), f"batch {batch}: device table"
    out = torch.empty(wl.total_blocks * wl.block_elems, dtype=torch.int16, device="cuda")
    assert _gather_layer(hlkv_lib, wl, out) == 0
    _compare_in_chunks(oracle, wl, out, chunk_seqs=2, pools_host=after)
    wl.dt.close()
    del out, wl, up
    _free()

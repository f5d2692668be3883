"""Seeded synthetic heterogeneous KV caches: table + device pools + device tables.

Builds the inputs of the gather-dequant path the way a serving engine would
hold them: a HeteroBlockTable whose sequences reference blocks of mixed
formats, block ids and slots scattered by a seeded scramble of the LIFO free
lists, the persistent device tables brought up to date through the delta
protocol (kernel 3), and every payload slot filled with FP16 values
N(0, 1) (optionally with outlier channels) quantized per row on the GPU by
hlkv_quantize (the device quantize_reference).

Payload layout (the descriptor's layout tag ``layout_id``): 2 (K,V) x T tokens
x H heads rows of D elements, codes then per-row parameters -- see
include/hlkv.h.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from . import (FP16, FP8_E4M3, FP8_E5M2, INT4, DeviceTables, Handle, Layout, Status, Table,
               check, layout_slot_bytes, make_pools, quantize)

FORMATS = (FP16, FP8_E4M3, FP8_E5M2, INT4)


def code_bytes(fmt: int, elems: int) -> int:
    return 2 * elems if fmt == FP16 else (elems // 2 if fmt == INT4 else elems)


def param_bytes(fmt: int, rows: int) -> int:
    return 0 if fmt == FP16 else (8 * rows if fmt == INT4 else 4 * rows)


def block_bytes(fmt: int, T: int, H: int, D: int, valid_tokens: int | None = None) -> int:
    """Algorithmic bytes of one block: codes + parameters of the valid rows read,
    2*T*H*D binary16 values written, 16-byte descriptor + 4-byte arena entry read."""
    rows = 2 * T * H
    elems = rows * D
    vt = T if valid_tokens is None else valid_tokens
    frac_rows = 2 * vt * H
    read = (code_bytes(fmt, elems) + param_bytes(fmt, rows)) * frac_rows // rows
    return read + 2 * elems + 20


@dataclass
class KVWorkload:
    T: int
    H: int
    D: int
    layout: Layout
    table: Table
    dt: DeviceTables
    pools: dict                      # fmt -> (torch uint8 [num_slots, slot_bytes], slot_bytes, num_slots)
    seqs: list                       # sequence handles
    segs: object                     # torch int32 [nseq, 2] on the device
    segs_host: np.ndarray            # uint32 [nseq, 2]
    blocks_per_format: dict = field(default_factory=dict)
    valid_tokens_total: int = 0
    algorithmic_bytes: int = 0

    @property
    def block_elems(self) -> int:
        return 2 * self.T * self.H * self.D

    @property
    def total_blocks(self) -> int:
        return int(self.segs_host[:, 1].sum()) if len(self.segs_host) else 0

    def hlkv_pools(self):
        return make_pools(self.pools)


def _fill_pool(buf, fmt: int, num_slots: int, T: int, H: int, D: int, gen, outlier_channels: int,
               outlier_scale: float, chunk_slots: int = 2048) -> None:
    """Fills every slot of one pool with quantized N(0,1) FP16 data (device work)."""
    import torch
    rows = 2 * T * H
    elems = rows * D
    cb = code_bytes(fmt, elems)
    pb = param_bytes(fmt, rows)
    err = torch.zeros(1, dtype=torch.int32, device=buf.device)
    for s0 in range(0, num_slots, chunk_slots):
        n = min(chunk_slots, num_slots - s0)
        x = torch.randn((n, 2, T, H, D), generator=gen, device=buf.device, dtype=torch.float32)
        if outlier_channels > 0:
            for h in range(H):
                ch = torch.randperm(D, generator=gen, device=buf.device)[:outlier_channels]
                x[:, :, :, h, ch] *= outlier_scale
        x16 = x.to(torch.float16)
        dst = buf[s0:s0 + n]
        if fmt == FP16:
            dst[:, :cb] = x16.view(torch.uint8).reshape(n, cb)
            continue
        xf = x16.to(torch.float32).contiguous()
        codes = torch.empty(n * cb, dtype=torch.uint8, device=buf.device)
        params = torch.empty((n * rows, 2), dtype=torch.float32, device=buf.device)
        check(quantize(fmt, xf.data_ptr(), n * elems, D, params.data_ptr(), n * rows,
                       codes.data_ptr(), codes.numel(), err.data_ptr()), "quantize")
        dst[:, :cb] = codes.view(n, cb)
        if fmt == INT4:
            dst[:, cb:cb + pb] = params.view(torch.uint8).reshape(n, pb)
        else:
            dst[:, cb:cb + pb] = params[:, 0].contiguous().view(torch.uint8).reshape(n, pb)
    torch.cuda.current_stream().synchronize()
    if int(err.item()) != 0:
        raise RuntimeError(f"payload quantization flagged error bits {int(err.item()):#x}")


def build_workload(seq_formats: list, T: int = 16, H: int = 8, D: int = 128, seed: int = 0,
                   valid_tokens: list | None = None, outlier_channels: int = 4,
                   outlier_scale: float = 20.0, layout_id: int = 1, spare_slots: int = 0,
                   scramble: bool = True, device: str = "cuda") -> KVWorkload:
    """seq_formats[i][j] = format of block j of sequence i; valid_tokens likewise (default T)."""
    import torch
    rng = np.random.default_rng(seed)
    counts = {f: 0 for f in FORMATS}
    for fl in seq_formats:
        for f in fl:
            counts[int(f)] += 1
    layout = Layout(T, H, D, layout_id)
    used = [f for f in FORMATS if counts[f] > 0] or [FP16]
    slots = {f: counts[f] + spare_slots for f in used}
    slot_bytes = {}
    for f in used:
        sb = layout_slot_bytes(f, layout)
        slot_bytes[f] = (sb + 15) // 16 * 16
    max_blocks = max(1, sum(slots.values()))
    table = Table(max_blocks, [(f, slot_bytes[f], slots[f]) for f in used], block_tokens=T)

    if scramble:  # allocate everything, release in a seeded order: ids and slots come out shuffled
        handles = []
        for f in used:
            for _ in range(slots[f]):
                st, h = table.allocate(f, 0, layout_id)
                if st != Status.OK:
                    raise RuntimeError(f"scramble allocate failed: {st}")
                handles.append(h)
        for i in rng.permutation(len(handles)):
            if table.release(handles[i]) != Status.OK:
                raise RuntimeError("scramble release failed")

    seqs = []
    vt_total = 0
    algo = 0
    for i, fl in enumerate(seq_formats):
        st, s = table.create_sequence()
        if st != Status.OK:
            raise RuntimeError(f"create_sequence: {st}")
        seqs.append(s)
        for j, f in enumerate(fl):
            vt = T if valid_tokens is None else int(valid_tokens[i][j])
            st, _ = table.append_block(s, int(f), vt, layout_id)
            if st != Status.OK:
                raise RuntimeError(f"append_block: {st}")
            vt_total += vt
            algo += block_bytes(int(f), T, H, D, vt)
    st, segs_host = table.batch_segments(seqs)
    if st != Status.OK:
        raise RuntimeError(f"batch_segments: {st}")

    dt = DeviceTables()
    dt.sync(table)
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    pools = {}
    for f in used:
        buf = torch.zeros((slots[f], slot_bytes[f]), dtype=torch.uint8, device=device)
        _fill_pool(buf, f, slots[f], T, H, D, gen, outlier_channels, outlier_scale)
        pools[f] = (buf, slot_bytes[f], slots[f])
    segs = torch.from_numpy(segs_host.astype(np.int32).reshape(-1, 2)).to(device)
    torch.cuda.current_stream().synchronize()
    return KVWorkload(T, H, D, layout, table, dt, pools, seqs, segs, segs_host,
                      {f: counts[f] for f in FORMATS}, vt_total, algo)


def mixed_formats(nseq: int, blocks_per_seq, probs=(0.25, 0.5, 0.0, 0.25), seed: int = 0) -> list:
    """Per-block formats drawn from {FP16, E4M3, E5M2, INT4} with the given probabilities."""
    rng = np.random.default_rng(seed + 1)
    per = [blocks_per_seq] * nseq if np.isscalar(blocks_per_seq) else list(blocks_per_seq)
    p = np.asarray(probs, dtype=np.float64)
    return [list(rng.choice(FORMATS, size=int(n), p=p / p.sum())) for n in per]


def tiered_formats(nseq: int, tokens: int, T: int = 16, fp16_tokens: int = 512,
                   fp8_tokens: int = 2048) -> list:
    """Age tiers: the newest fp16_tokens in FP16, the fp8_tokens before them in E4M3, older INT4."""
    nb = tokens // T
    n16, n8 = fp16_tokens // T, fp8_tokens // T
    row = [INT4] * max(nb - n16 - n8, 0) + [FP8_E4M3] * min(n8, max(nb - n16, 0)) + [FP16] * min(n16, nb)
    return [list(row) for _ in range(nseq)]


def host_arena(wl: KVWorkload) -> np.ndarray:
    """The arena entries the segments reference, rebuilt from the host table."""
    size = wl.dt.arena_size
    arena = np.full(max(size, 1), 0xFFFFFFFF, dtype=np.uint32)
    for s, (off, ln) in zip(wl.seqs, wl.segs_host):
        st, ids = wl.table.sequence_block_ids(s)
        if st != Status.OK:
            raise RuntimeError("sequence_block_ids")
        arena[off:off + ln] = ids
    return arena[:size]


def host_table(wl: KVWorkload) -> np.ndarray:
    """device_descriptor(id) for every id, uint32 [max_blocks, 4]."""
    n = wl.table.max_blocks()
    return np.array([wl.table.device_descriptor(i) for i in range(n)], dtype=np.uint32).reshape(n, 4)


class UpdateStream:
    """Seeded stream of descriptor updates for a resident cache, as a serving engine makes
    them between sweeps: each batch takes `n` distinct blocks of the workload's sequences;
    half get set_valid_tokens (1..T) while unsealed, the rest a format change to the next
    age tier (seal, begin_format_change, a transcode job, commit).  prepare() is the host
    half (table calls, then collect() into the device tables' pinned staging); launch()
    queues the device half (job upload, hlkv_transcode, then the delta flush = kernel 3).

    `sweep_bytes` tracks the algorithmic bytes of one gather over all the workload's
    sequences as valid tokens and formats change.  The pools need `n` spare slots per
    batch in every target format (a format change takes its new slot before the commit
    frees the old one)."""

    NEXT = {FP16: FP8_E4M3, FP8_E4M3: INT4, INT4: FP8_E4M3}  # FP16 -> E4M3 -> INT4 -> E4M3

    def __init__(self, wl: KVWorkload, n: int, seed: int):
        import torch
        self.wl, self.n = wl, n
        self.rng = np.random.default_rng(seed)
        ids = []
        for s in wl.seqs:
            st, row = wl.table.sequence_block_ids(s)
            if st != Status.OK:
                raise RuntimeError("sequence_block_ids")
            ids.extend(row)
        self.ids = np.array(ids, dtype=np.uint32)
        m = wl.table.max_blocks()
        self.sealed = np.zeros(m, bool)
        self.fmt = np.zeros(m, np.uint8)
        self.vt = np.zeros(m, np.uint32)
        for bid in self.ids:
            info = wl.table.device_descriptor(int(bid))[1]
            self.fmt[bid], self.vt[bid] = info & 0xF, (info >> 10) & 0x3FF
        self.sweep_bytes = wl.algorithmic_bytes
        self.jobs_host = torch.empty((n, 8), dtype=torch.int32).pin_memory()
        self.jobs_dev = torch.empty((n, 8), dtype=torch.int32, device="cuda")
        self.jobs_np = self.jobs_host.numpy().view(np.uint32)
        self.uploaded = torch.cuda.Event()
        self.first = True
        self.n_jobs = 0
        self.counts = {"valid_tokens": 0, "format_changes": 0}

    def _bytes(self, f: int, vt: int) -> int:
        w = self.wl
        return block_bytes(f, w.T, w.H, w.D, vt)

    def prepare(self) -> int:
        """Host half of one batch; returns the bytes the batch moves on the device
        (descriptor patches, transcode reads and writes)."""
        w, t, rng = self.wl, self.wl.table, self.rng
        if not self.first:
            self.uploaded.synchronize()  # the previous upload has read jobs_host
        self.first = False
        picks = rng.choice(self.ids.size, size=self.n, replace=False)
        kinds = rng.integers(0, 2, size=self.n)
        out_bytes = 2 * 2 * w.T * w.H * w.D + 20  # FP16 written + descriptor per block
        nj, moved, changed = 0, 0, []
        for i, kind in zip(picks, kinds):
            bid = int(self.ids[i])
            h = t.handle_of(bid)
            f, vt = int(self.fmt[bid]), int(self.vt[bid])
            if kind == 0 and not self.sealed[bid]:
                nvt = int(rng.integers(1, w.T + 1))
                if t.set_valid_tokens(h, nvt) != Status.OK:
                    raise RuntimeError("set_valid_tokens")
                self.sweep_bytes += self._bytes(f, nvt) - self._bytes(f, vt)
                self.vt[bid] = nvt
                self.counts["valid_tokens"] += 1
                moved += 32  # one descriptor patch read and written
                continue
            target = self.NEXT[f]
            if not self.sealed[bid]:
                if t.seal(h) != Status.OK:
                    raise RuntimeError("seal")
                self.sealed[bid] = True
            st, fc = t.begin_format_change(h, target)
            if st != Status.OK:
                raise RuntimeError(f"begin_format_change: {st}")
            self.jobs_np[nj] = (fc[0], fc[1], fc[2], fc[3], vt, 0, 0, 0)
            nj += 1
            changed.append(h)
            # source codes + params of the valid rows read, all destination rows written
            moved += (self._bytes(f, vt) - out_bytes) + (self._bytes(target, w.T) - out_bytes) + 64
            self.sweep_bytes += self._bytes(target, vt) - self._bytes(f, vt)
            self.fmt[bid] = target
        # The commits only change host state; the device sees them through the delta,
        # which launch() queues after the transcode.
        for h in changed:
            if t.commit_format_change(h, 0, 0) != Status.OK:
                raise RuntimeError("commit_format_change")
        self.counts["format_changes"] += nj
        self.n_jobs = nj
        w.dt.collect(t)
        return moved

    def launch(self, stream, err) -> int:
        """Device half, in stream order: job upload, transcode, delta flush (kernel 3).
        Returns the number of kernels queued."""
        from . import transcode
        w, nj = self.wl, self.n_jobs
        launches = 0
        if nj:
            self.jobs_dev[:nj].copy_(self.jobs_host[:nj], non_blocking=True)
            self.uploaded.record(stream)
            check(transcode(w.hlkv_pools(), w.layout, self.jobs_dev[:nj], err, stream=stream), "transcode")
            launches += 1
        w.dt.flush(stream)
        return launches + 1

"""Work assignment of the gather-dequant kernel (gather_dequant_kernel, gather_dequant.cu),
restated on the CPU and checked over random batches.

Sequences are taken in chunks of 256.  A chunk's blocks are numbered in sequence order;
when the chunk has fewer than 2 blocks per CTA, every block is cut into `parts` tile ranges
(parts doubles while parts < 8, total * parts < 2 G and ntiles >= 16 * parts, so that a
part keeps at least 8 tiles, one per warp).  Piece q (numbered across chunks) belongs to CTA q mod G, which takes its pieces
256 at a time, one per thread, and finds each piece's sequence by a binary search of the
chunk's exclusive prefix.  Checked: every tile of every block of every sequence is streamed
by exactly one CTA, and each batch's item count (n_items) equals the number of threads that
wrote an item."""
import numpy as np
import pytest

K_THREADS = 256
K_TILE_CHUNKS = 32 * 4  # 8-element chunks per warp tile


def parts_for(total, G, ntiles):
    parts = 1
    while parts < 8 and total * parts < 2 * G and ntiles >= 16 * parts:
        parts *= 2
    return parts


def cta_items(c, G, lengths, ntiles):
    """The (seq, block, tile_begin, tile_end) items CTA c streams, in the kernel's order."""
    items = []
    pbase = 0
    nseq = len(lengths)
    for chunk in range(0, nseq, K_THREADS):
        cnt = min(nseq - chunk, K_THREADS)
        lens = lengths[chunk:chunk + cnt]
        prefix = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)  # exclusive prefix
        total = int(prefix[-1])
        parts = parts_for(total, G, ntiles)
        pend = pbase + total * parts
        first = pbase + (c + G - pbase % G) % G
        while first < pend:
            batch = []
            for t in range(K_THREADS):
                q = first + t * G
                if q >= pend:
                    continue
                lq = q - pbase
                local = lq // parts
                lo, hi = 0, cnt  # last s with prefix[s] <= local
                while hi - lo > 1:
                    mid = (lo + hi) >> 1
                    if prefix[mid] <= local:
                        lo = mid
                    else:
                        hi = mid
                j = local - int(prefix[lo])
                assert 0 <= j < lens[lo], "the piece lies in a non-empty sequence"
                per_part = (ntiles + parts - 1) // parts
                tb = (lq % parts) * per_part
                batch.append((chunk + lo, j, tb, min(ntiles, tb + per_part)))
            n_items = min(K_THREADS, (pend - first + G - 1) // G)
            assert n_items == len(batch)
            items += batch
            first += K_THREADS * G
        pbase = pend
    return items


def check(lengths, G, ntiles):
    seen = {}
    for c in range(G):
        for seq, j, tb, te in cta_items(c, G, lengths, ntiles):
            for t in range(tb, te):
                key = (seq, j, t)
                assert key not in seen, "tile streamed twice"
                seen[key] = c
    assert len(seen) == sum(lengths) * ntiles, "a tile is never streamed"


def ntiles_for(T, H, D):
    return (2 * T * H * D // 8 + K_TILE_CHUNKS - 1) // K_TILE_CHUNKS


def test_config_shapes():
    # config 1: one sequence of 256 blocks, 16 tokens x 8 KV heads x 128: 4 parts of 8 tiles
    # (one per warp), 1,024 pieces on 592 CTAs
    nt = ntiles_for(16, 8, 128)
    assert nt == 32 and parts_for(256, 592, nt) == 4
    check([256], 592, nt)
    # config 2: 64 x 128 blocks, no split
    assert parts_for(64 * 128, 592, nt) == 1
    check([128] * 64, 592, nt)


@pytest.mark.parametrize("seed", range(4))
def test_random_batches(seed):
    rng = np.random.default_rng(seed)
    for _ in range(40):
        nseq = int(rng.choice([1, 3, 40, 255, 256, 257, 600]))
        lengths = [int(v) for v in rng.integers(0, 6, nseq)]
        if rng.random() < 0.3:
            lengths = [0] * nseq
            lengths[int(rng.integers(0, nseq))] = int(rng.integers(1, 50))
        T, H, D = [(16, 8, 128), (4, 2, 64), (16, 1, 64), (32, 8, 256)][int(rng.integers(0, 4))]
        G = int(rng.choice([1, 5, 148, 592]))
        check(lengths, G, ntiles_for(T, H, D))


def test_all_empty():
    for G in (1, 592):
        assert all(cta_items(c, G, [0] * 300, 32) == [] for c in range(G))

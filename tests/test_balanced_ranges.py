"""Index arithmetic of the balanced decode attention (hlkv_decode_attention_balanced,
decode_attention.cu), restated on the CPU and checked over random batches of sequence
lengths, empty sequences and CTA counts above and below the block count included:

* the prefix pass: prefix[0] = 0, prefix[i + 1] = prefix[i] + H * n_i (attention_prefix);
* CTA c of G takes blocks [floor(c W / G), floor((c + 1) W / G)) of all (sequence, KV head)
  units laid end to end, cut into one piece per unit its range meets, and writes piece
  (c, u) to partial slot c + u (decode_attention_kernel, balanced branch);
* the merge of unit u reads the slots c + u of the non-empty CTAs from the one holding the
  unit's first block to the one holding its last (decode_attention_merge_balanced).

Checked: every block lies in exactly one piece, no two pieces share a slot, every slot is
below ctas + nseq * H (the workspace's slot count,
hlkv_decode_attention_balanced_workspace_bytes), and each unit's merge reads exactly the
slots its pieces wrote."""
import numpy as np
import pytest


def prefix_sums(lengths, H):
    p = [0]
    for n in lengths:
        p.append(p[-1] + H * n)
    return p


def balanced_cta(x, W, G):
    """The CTA whose range holds block x: the largest c with floor(c W / G) <= x."""
    return ((x + 1) * G - 1) // W


def pieces_of_cta(c, G, prefix, lengths, H):
    """The pieces (seq, h, b0, b1, slot) that CTA c of G processes, as the kernel walks them."""
    nseq = len(lengths)
    W = prefix[nseq]
    x, x_end = c * W // G, (c + 1) * W // G
    out = []
    while x < x_end:
        lo, hi = 0, nseq  # the largest s with prefix[s] <= x
        while hi - lo > 1:
            mid = (lo + hi) >> 1
            if prefix[mid] <= x:
                lo = mid
            else:
                hi = mid
        seq = lo
        n = lengths[seq]
        assert n > 0, "x lies inside a non-empty sequence's range"
        local = x - prefix[seq]
        h = local // n
        b0 = local - h * n
        b1 = min(n, b0 + (x_end - x))
        x += b1 - b0
        out.append((seq, h, b0, b1, c + seq * H + h))
    return out


def merged_slots(seq, h, G, prefix, lengths, H):
    """The slots the merge reads for unit (seq, h)."""
    n = lengths[seq]
    if n == 0:
        return []
    W = prefix[len(lengths)]
    u = seq * H + h
    start = prefix[seq] + h * n
    c0, c1 = balanced_cta(start, W, G), balanced_cta(start + n - 1, W, G)
    sparse = G > W

    def empty(c):
        return sparse and c * W // G == (c + 1) * W // G

    return [c + u for c in range(c0, c1 + 1) if not empty(c)]


def check_batch(lengths, H, G):
    prefix = prefix_sums(lengths, H)
    W = prefix[-1]
    covered = {}
    written = {}
    for c in range(G):
        for seq, h, b0, b1, slot in pieces_of_cta(c, G, prefix, lengths, H):
            assert 0 <= h < H and 0 <= b0 < b1 <= lengths[seq]
            assert slot not in written, "two pieces share a slot"
            assert slot < G + len(lengths) * H, "slot beyond the workspace"
            written[slot] = (seq, h)
            for b in range(b0, b1):
                key = (seq, h, b)
                assert key not in covered, "block in two pieces"
                covered[key] = c
    assert len(covered) == W
    for seq, n in enumerate(lengths):
        for h in range(H):
            want = sorted(s for s, unit in written.items() if unit == (seq, h))
            assert merged_slots(seq, h, G, prefix, lengths, H) == want


def test_balanced_worked_example():
    # 3 sequences of 5, 0 and 3 blocks, 2 KV heads: W = 16 blocks over 3 CTAs
    lengths, H, G = [5, 0, 3], 2, 3
    prefix = prefix_sums(lengths, H)
    assert prefix == [0, 10, 10, 16]
    assert pieces_of_cta(0, G, prefix, lengths, H) == [(0, 0, 0, 5, 0)]
    assert pieces_of_cta(1, G, prefix, lengths, H) == [(0, 1, 0, 5, 2)]
    assert pieces_of_cta(2, G, prefix, lengths, H) == [(2, 0, 0, 3, 6), (2, 1, 0, 3, 7)]
    check_batch(lengths, H, G)


@pytest.mark.parametrize("seed", range(6))
def test_balanced_ranges_random_batches(seed):
    rng = np.random.default_rng(seed)
    for _ in range(150):
        nseq = int(rng.integers(1, 12))
        lengths = [int(v) for v in rng.integers(0, 40, nseq)]
        if rng.random() < 0.3:
            lengths[int(rng.integers(0, nseq))] = int(rng.integers(100, 600))  # one long sequence
        if sum(lengths) == 0:
            lengths[0] = 1
        H = int(rng.choice([1, 2, 4, 8]))
        W = H * sum(lengths)
        G = int(rng.choice([1, 2, 7, max(1, W // 3), W, W + 5, 592]))
        check_batch(lengths, H, G)

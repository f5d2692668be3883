"""The checks bench.py prints beside its numbers, on CPU: the decode workload's parity
check (bench.decode_parity) accepts pools that hold exactly the oracle's append of the
step's tokens and reports a single flipped byte in one of them; the roofline's traffic
figure is read from the current-kernel column of the committed ncu summary.  No GPU: the
pools are numpy arrays written by the oracle, the table is the host library's."""
import numpy as np
import pytest


def _decode_step(hlkv_lib, oracle, n=40, seed=1):
    import torch
    T, H, D = 16, 8, 128
    layout = hlkv_lib.Layout(T, H, D, 1)
    quant = [hlkv_lib.FP8_E4M3, hlkv_lib.INT4]
    sb = {int(f): (oracle.slot_bytes_needed(int(f), T, H, D) + 15) // 16 * 16 for f in quant}
    table = hlkv_lib.Table(4 * n, [(f, sb[f], 2 * n) for f in sb], block_tokens=T)
    rng = np.random.default_rng(seed)
    seqs = []
    for _ in range(n):
        st, s = table.create_sequence()
        assert st == 0
        seqs.append(s)
        st, _ = table.append_block(s, int(rng.choice(quant)), int(rng.integers(1, T)), 1)
        assert st == 0
    st, targets, done = table.append_tokens(seqs, rng.choice(quant, size=n).astype(np.uint32), 1)
    assert st == 0 and done == n
    desc = np.array([table.device_descriptor(i) for i in range(4 * n)], np.uint32)
    pools = {f: (np.zeros((2 * n, sb[f]), np.uint8), sb[f], 2 * n) for f in sb}
    tokens = torch.from_numpy(rng.standard_normal((n, 2, H, D)).astype(np.float16))
    assert oracle.append_encode(pools, T, H, D, 1, desc, targets, tokens.numpy().view(np.uint16)) == 0
    pools_t = {f: (torch.from_numpy(v[0]), v[1], v[2]) for f, v in pools.items()}
    return table, pools, pools_t, tokens, targets, desc, (T, H, D, layout)


def test_decode_parity_accepts_the_oracle_append(hlkv_lib, oracle):
    from bench import decode_parity
    table, _, pools_t, tokens, targets, _, (T, H, D, layout) = _decode_step(hlkv_lib, oracle)
    for sample in (8, 40):
        res = decode_parity(table, pools_t, tokens, targets, T, H, D, layout, 0, sample_size=sample)
        assert res["ok"] and res["differing_rows"] == 0, res


def test_decode_parity_reports_one_flipped_byte(hlkv_lib, oracle):
    from bench import decode_parity
    table, pools, pools_t, tokens, targets, desc, (T, H, D, layout) = _decode_step(hlkv_lib, oracle)
    d = desc[targets[0, 0]]
    f = int(d[1] & 0xF)
    cb = D if f == hlkv_lib.FP8_E4M3 else D // 2
    row = (1 * T + int(targets[0, 1])) * H + 3  # V half, head 3 of target 0
    pools[f][0][d[0], row * cb + 7] ^= 1
    res = decode_parity(table, pools_t, tokens, targets, T, H, D, layout, 0, sample_size=40)
    assert not res["ok"] and res["differing_rows"] == 1, res
    # error bits reported by the kernel fail the check as well
    pools[f][0][d[0], row * cb + 7] ^= 1
    assert not decode_parity(table, pools_t, tokens, targets, T, H, D, layout, 1)["ok"]


def test_traffic_is_read_from_the_current_kernel_column():
    from bench import traffic_from_profile
    # one config-4 layer: the per-format kernel's capture is the last column
    assert traffic_from_profile("gather_dequant_llama8b_layer_full") == 2_915_823_616
    # the decode step's encoder, captured on the same 8192 appends
    assert traffic_from_profile("append_encode_decode_small_full") == 34_006_528
    assert traffic_from_profile("no_such_summary") is None


if __name__ == "__main__":
    pytest.main([__file__, "-q"])

"""bench.py's workload definitions and algorithmic byte counts, on the CPU.

The headline number is bytes / time, so the byte counts are pinned here against the
per-call figures of the measurement plan: config 1 moves 2*1024*12*64*4 bytes of K/V plus
Q, O, the 64-entry block table and the length (6,297,860 B); config 3 with seed 42 has
sum(ctx) = 147,397 over 9,230 blocks, 1,208,589,056 B in fp32; a GPT-2 Small step at batch
64 and mean context 192.5 reads ~1.15 GB (int8 weights, fp32 tied embedding, fp32 KV)."""
import numpy as np
import pytest


def test_config3_workload_is_seeded_and_ragged():
    import bench

    lens, bt, P = bench.workload_meta()
    lens2, bt2, P2 = bench.workload_meta()
    assert np.array_equal(lens, lens2) and np.array_equal(bt, bt2) and P == P2
    assert lens.shape == (bench.B,) and lens.min() >= bench.CTX_LO and lens.max() <= bench.CTX_HI
    assert int(lens.sum()) == 147397 and P == 9230
    nb = (lens + bench.BS - 1) // bench.BS
    used = np.concatenate([bt[b, :nb[b]] for b in range(bench.B)])
    assert np.array_equal(np.sort(used), np.arange(P))  # a permutation of the pool


def test_algorithmic_bytes():
    import bench

    lens, bt, P = bench.workload_meta()
    assert bench.attn_alg_bytes(lens, 8, 32, 128, 4, bt.shape[1]) == 1208589056
    assert bench.attn_alg_bytes(np.array([1024]), 12, 12, 64, 4, 64) == 6297860
    # bf16 halves only the K/V term
    kv32 = int(lens.sum()) * 2 * 8 * 128 * 4
    assert bench.attn_alg_bytes(lens, 8, 32, 128, 2, bt.shape[1]) == 1208589056 - kv32 // 2
    assert bench.gpt2_step_bytes(bench.GPT2_SMALL, 64, 192.5) == pytest.approx(1.148e9, rel=1e-3)


def test_profile_report_parsing():
    import bench

    text = "step_us 700.5 launches 99\nattention 12 210.0 30.0\ngemm_fc2 12 100.25 14.3\n"
    r = bench.parse_profile(text)
    assert r["step_us"] == pytest.approx(700.5)
    assert r["us"]["attention"] == pytest.approx(210.0) and r["us"]["gemm_fc2"] == pytest.approx(100.25)

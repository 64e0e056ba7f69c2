"""Pins the CPU oracle (oracle/oracle.c) to the reference's own code.

- Quantiser: bit-exact against fixtures produced by the reference's numpy quantize_per_row
  (python/export_gpt2.py:10-40; tests/golden/make_golden.py).
- Attention: bit-exact against fixtures produced by the reference harness's CPU attention
  gqa_cpu_reference (tests/test_paged_attention.cu:138-179), paged through random block
  tables, and live against the same function compiled from the reference sources when
  oracle/_ref/libref.so is present.
- int32 GEMM: exact against an int64 numpy contraction.
"""
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _cases(npz, suffix):
    names = sorted({k.split("__")[0] for k in npz.files})
    return [(n, {k.split("__")[1]: npz[k] for k in npz.files if k.startswith(n + "__")}) for n in names]


def test_quantize_matches_reference_numpy(oracle):
    z = np.load(os.path.join(GOLDEN, "quantize_golden.npz"))
    cases = _cases(z, "")
    assert len(cases) >= 7
    for name, c in cases:
        packed, scales = oracle.quantize(c["x"])
        np.testing.assert_array_equal(scales.view(np.uint32), c["scales"].view(np.uint32), err_msg=name)
        np.testing.assert_array_equal(packed, c["packed"], err_msg=name)


def page(K, V, block_size, rng, extra_blocks=3):
    """Scatter contiguous K/V [B,H_kv,N,d] into a paged cache with a random block table."""
    B, H_kv, N, d = K.shape
    nbps = (N + block_size - 1) // block_size
    P = B * nbps + extra_blocks
    perm = rng.permutation(P)[: B * nbps].reshape(B, nbps).astype(np.int32)
    kc = rng.standard_normal((P, block_size, H_kv, d)).astype(np.float32)  # garbage elsewhere
    vc = rng.standard_normal((P, block_size, H_kv, d)).astype(np.float32)
    for b in range(B):
        for t in range(N):
            kc[perm[b, t // block_size], t % block_size] = K[b, :, t]
            vc[perm[b, t // block_size], t % block_size] = V[b, :, t]
    return kc, vc, perm


def test_decode_attention_matches_reference_harness_fixtures(oracle):
    z = np.load(os.path.join(GOLDEN, "attention_golden.npz"))
    rng = np.random.default_rng(7)
    cases = _cases(z, "")
    assert len(cases) >= 5
    for name, c in cases:
        B, H_kv, N, d = c["K"].shape
        for bs in (16, 5):
            kc, vc, bt = page(c["K"], c["V"], bs, rng)
            O = oracle.decode_attn(c["q"], kc, vc, bt, np.full(B, N, np.int32))
            np.testing.assert_array_equal(O.view(np.uint32), c["O"].view(np.uint32), err_msg=f"{name} bs={bs}")


@pytest.mark.parametrize("B,H_q,H_kv,N,d", [(1, 12, 12, 64, 64), (2, 8, 2, 33, 128), (1, 8, 1, 100, 64)])
def test_decode_attention_matches_live_reference_harness(oracle, B, H_q, H_kv, N, d):
    if not oracle.ref_available():
        pytest.skip("oracle/_ref/libref.so not built")
    rng = np.random.default_rng(B * 1000 + N)
    Q = rng.standard_normal((B, H_q, N, d)).astype(np.float32)
    K = rng.standard_normal((B, H_kv, N, d)).astype(np.float32)
    V = rng.standard_normal((B, H_kv, N, d)).astype(np.float32)
    ref = oracle.ref_gqa_cpu(Q, K, V, causal=False)[:, :, N - 1]
    kc, vc, bt = page(K, V, 16, rng)
    O = oracle.decode_attn(Q[:, :, N - 1], kc, vc, bt, np.full(B, N, np.int32))
    np.testing.assert_array_equal(O.view(np.uint32), ref.view(np.uint32))


def test_decode_attention_ragged_and_empty(oracle):
    """Ragged lengths (incl. 0 and 1) equal per-sequence dense computations."""
    rng = np.random.default_rng(3)
    B, H_q, H_kv, d, bs = 4, 4, 2, 64, 16
    lens = np.array([0, 1, 17, 40], np.int32)
    N = int(lens.max())
    K = rng.standard_normal((B, H_kv, N, d)).astype(np.float32)
    V = rng.standard_normal((B, H_kv, N, d)).astype(np.float32)
    q = rng.standard_normal((B, H_q, d)).astype(np.float32)
    kc, vc, bt = page(K, V, bs, rng)
    O = oracle.decode_attn(q, kc, vc, bt, lens)
    assert np.all(O[0] == 0)
    for b in range(1, B):
        n = int(lens[b])
        Ob = oracle.decode_attn(q[b:b + 1], *page(K[b:b + 1, :, :n], V[b:b + 1, :, :n], bs, rng), np.array([n], np.int32))
        np.testing.assert_array_equal(O[b], Ob[0])


def test_decode_attention_bf16_upcast(oracle):
    rng = np.random.default_rng(4)
    P, bs, H_kv, d = 6, 16, 2, 64
    kf = rng.standard_normal((P, bs, H_kv, d)).astype(np.float32)
    vf = rng.standard_normal((P, bs, H_kv, d)).astype(np.float32)
    # truncate to bf16-representable values so both paths see identical numbers
    kb = (kf.view(np.uint32) >> 16).astype(np.uint16)
    vb = (vf.view(np.uint32) >> 16).astype(np.uint16)
    k32 = (kb.astype(np.uint32) << 16).view(np.float32)
    v32 = (vb.astype(np.uint32) << 16).view(np.float32)
    q = rng.standard_normal((1, 4, d)).astype(np.float32)
    bt = np.array([[3, 1, 5, 0]], np.int32)
    lens = np.array([55], np.int32)
    a = oracle.decode_attn(q, kb, vb, bt, lens)
    b = oracle.decode_attn(q, k32, v32, bt, lens)
    np.testing.assert_array_equal(a, b)


def test_int8_gemm_s32_exact(oracle):
    rng = np.random.default_rng(5)
    M, N, K = 17, 23, 36
    A = rng.integers(-128, 128, (M, K), dtype=np.int8)
    Bm = rng.integers(-128, 128, (N, K), dtype=np.int8)
    C = oracle.int8_gemm_s32(A.view(np.int32), Bm.view(np.int32))
    np.testing.assert_array_equal(C, A.astype(np.int64) @ Bm.astype(np.int64).T)


def test_epilogue_order(oracle):
    """(float(acc)*sA)*sB, bias by fused multiply-add, then residual (14_int8_gemm.cu:154-167)."""
    acc = np.array([[1000, -7]], np.int32)
    sA = np.array([0.1], np.float32)
    sB = np.array([0.3, 3.0], np.float32)
    bias = np.array([0.25, -1.0], np.float32)
    res = np.array([[1.0, 2.0]], np.float32)
    t = (acc.astype(np.float32) * sA[:, None]).astype(np.float32)
    plain = (t * sB).astype(np.float32)
    np.testing.assert_array_equal(oracle.epilogue(acc, sA, sB, epi=0), plain)
    fused = (t.astype(np.float64) * sB + bias).astype(np.float32)  # one rounding, like fmaf
    np.testing.assert_array_equal(oracle.epilogue(acc, sA, sB, bias, epi=1), fused)
    np.testing.assert_array_equal(oracle.epilogue(acc, sA, sB, bias, res, epi=3), (fused + res).astype(np.float32))

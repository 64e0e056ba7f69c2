"""K13 decode attention on the GPU vs the oracle and vs the reference's own K13.

Tolerances: fp32 KV within rtol 1e-4 / atol 1e-5 of the oracle (the reference's K13 test
uses 1e-5 abs, tests/test_decode_attention.cu:132); bf16 KV within rtol 2e-2 / atol 2e-3.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

F32_TOL = dict(rtol=1e-4, atol=1e-5)
BF16_TOL = dict(rtol=2e-2, atol=2e-3)


def _libc_uniform(n_list):
    """The reference harness's generator: srand(42); rand()/RAND_MAX*2-1, drawn in its order."""
    libc = ctypes.CDLL("libc.so.6")
    libc.rand.restype = ctypes.c_int
    libc.srand(42)
    RAND_MAX = 2147483647
    out = []
    for n in n_list:
        out.append(np.array([libc.rand() for _ in range(n)], np.float64))
    return out, RAND_MAX


def reference_inputs(B, H_q, H_kv, ctx, d, block_size):
    """Inputs exactly as tests/test_decode_attention.cu:60-76 builds them (srand(42),
    K and V interleaved draws, contiguous physical blocks per sequence)."""
    libc = ctypes.CDLL("libc.so.6")
    libc.rand.restype = ctypes.c_int
    libc.srand(42)
    RM = np.float32(2147483647)
    q = np.array([libc.rand() for _ in range(B * H_q * d)], np.float32)
    q = q / RM * np.float32(2.0) - np.float32(1.0)
    kv = np.array([libc.rand() for _ in range(2 * B * H_kv * ctx * d)], np.float32)
    kv = kv / RM * np.float32(2.0) - np.float32(1.0)
    K = kv[0::2].reshape(B, H_kv, ctx, d)
    V = kv[1::2].reshape(B, H_kv, ctx, d)
    bps = (ctx + block_size - 1) // block_size
    kc = np.zeros((B * bps, block_size, H_kv, d), np.float32)
    vc = np.zeros_like(kc)
    bt = np.arange(B * bps, dtype=np.int32).reshape(B, bps)
    for b in range(B):
        for t in range(ctx):
            kc[bt[b, t // block_size], t % block_size] = K[b, :, t]
            vc[bt[b, t // block_size], t % block_size] = V[b, :, t]
    return q.reshape(B, H_q, d), kc, vc, bt, np.full(B, ctx, np.int32)


def random_paged(rng, B, H_q, H_kv, d, lens, block_size=16, extra=5, dtype="f32"):
    lens = np.asarray(lens, np.int32)
    nbps = max(1, int((lens.max() + block_size - 1) // block_size))
    need = int(sum((int(l) + block_size - 1) // block_size for l in lens))
    P = need + extra
    perm = rng.permutation(P).astype(np.int32)
    bt = np.full((B, nbps), -1, np.int32)  # unused entries are garbage the kernel must not read
    i = 0
    for b in range(B):
        nb = (int(lens[b]) + block_size - 1) // block_size
        bt[b, :nb] = perm[i:i + nb]
        i += nb
    kc = rng.standard_normal((P, block_size, H_kv, d)).astype(np.float32)
    vc = rng.standard_normal((P, block_size, H_kv, d)).astype(np.float32)
    q = rng.standard_normal((B, H_q, d)).astype(np.float32)
    if dtype == "bf16":
        kc = (kc.view(np.uint32) >> 16).astype(np.uint16)
        vc = (vc.view(np.uint32) >> 16).astype(np.uint16)
    return q, kc, vc, bt, lens


def to_dev(torch, a, device):
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).to(device).view(torch.bfloat16)
    return torch.from_numpy(a).to(device)


def run_b2(b2, torch, device, q, kc, vc, bt, lens, max_ctx=None):
    tq, tk, tv, tbt, tl = (to_dev(torch, a, device) for a in (q, kc, vc, bt, lens))
    O = b2.decode_attn(tq, tk, tv, tbt, tl, int(max_ctx if max_ctx is not None else max(1, lens.max())))
    torch.cuda.synchronize()
    assert b2.device_error() == 0
    return O.cpu().numpy()


# The reference's own K13 cases (tests/test_decode_attention.cu:144-151), same generator.
REF_CASES = [(1, 8, 8, 128, 64), (1, 16, 16, 512, 64), (4, 8, 8, 256, 64), (1, 8, 8, 1024, 64),
             (1, 16, 4, 256, 64), (8, 32, 8, 1024, 64)]


@pytest.mark.parametrize("B,H_q,H_kv,ctx,d", REF_CASES)
def test_reference_cases_vs_oracle_and_reference_k13(b2, oracle, cuda, B, H_q, H_kv, ctx, d):
    import torch

    q, kc, vc, bt, lens = reference_inputs(B, H_q, H_kv, ctx, d, 16)
    want = oracle.decode_attn(q, kc, vc, bt, lens)
    got = run_b2(b2, torch, cuda, q, kc, vc, bt, lens, ctx)
    np.testing.assert_allclose(got, want, **F32_TOL)
    # drop-in entry point with the reference's signature and workspace size
    tq, tk, tv, tbt, tl = (torch.from_numpy(a).to(cuda) for a in (q, kc, vc, bt, lens))
    O2 = torch.empty_like(tq)
    ws = torch.empty(B * H_q * b2.DA_MAX_SPLITS * (d + 2), dtype=torch.float32, device=cuda)
    b2.run_decode_attn(B, H_q, H_kv, d, tq, tk, tv, tbt, tl, ctx, 16, bt.shape[1], O2, ws)
    torch.cuda.synchronize()
    np.testing.assert_allclose(O2.cpu().numpy(), want, **F32_TOL)
    if oracle.ref_available():
        O3 = torch.zeros_like(tq)
        oracle.ref().ref_run_decode_attn(B, H_q, H_kv, d, tq.data_ptr(), tk.data_ptr(), tv.data_ptr(),
                                         tbt.data_ptr(), tl.data_ptr(), ctx, 16, bt.shape[1], O3.data_ptr(),
                                         ws.data_ptr())
        assert oracle.ref().ref_sync() == 0
        np.testing.assert_allclose(O3.cpu().numpy(), got, rtol=0, atol=1e-5)


@pytest.mark.parametrize("G", [1, 2, 4, 8])
@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_gqa_head_dims_dtypes_ragged(b2, oracle, cuda, G, d, dtype):
    import torch

    rng = np.random.default_rng(100 * G + d + (7 if dtype == "bf16" else 0))
    H_kv = 2
    lens = [1, 15, 16, 17, 100, 333, 700]
    q, kc, vc, bt, lens = random_paged(rng, len(lens), G * H_kv, H_kv, d, lens, dtype=dtype)
    want = oracle.decode_attn(q, kc, vc, bt, lens)
    got = run_b2(b2, torch, cuda, q, kc, vc, bt, lens)
    np.testing.assert_allclose(got, want, **(F32_TOL if dtype == "f32" else BF16_TOL))


def test_config1_mha_random_permutation(b2, oracle, cuda):
    """B1 H12 d64 ctx1024, block table = seeded permutation of 64 blocks."""
    import torch

    rng = np.random.default_rng(42)
    B, H, d, ctx, bs = 1, 12, 64, 1024, 16
    bt = rng.permutation(64).astype(np.int32).reshape(1, 64)
    kc = rng.standard_normal((64, bs, H, d)).astype(np.float32)
    vc = rng.standard_normal((64, bs, H, d)).astype(np.float32)
    q = rng.standard_normal((B, H, d)).astype(np.float32)
    lens = np.array([ctx], np.int32)
    want = oracle.decode_attn(q, kc, vc, bt, lens)
    got = run_b2(b2, torch, cuda, q, kc, vc, bt, lens)
    np.testing.assert_allclose(got, want, **F32_TOL)


def test_empty_contexts_and_empty_splits(b2, oracle, cuda):
    """Zero-length sequences give 0; short sequences in a long batch leave splits empty
    (the case the reference reads stale workspace for, 13_decode_attn.cuh:56)."""
    import torch

    rng = np.random.default_rng(11)
    lens = [0, 3, 4000, 0, 63 * 16, 17]
    q, kc, vc, bt, lens = random_paged(rng, len(lens), 8, 2, 128, lens)
    want = oracle.decode_attn(q, kc, vc, bt, lens)
    got = run_b2(b2, torch, cuda, q, kc, vc, bt, lens)
    assert np.all(got[0] == 0) and np.all(got[3] == 0)
    np.testing.assert_allclose(got, want, **F32_TOL)
    # repeated calls reuse the workspace counters (they must come back to zero)
    got2 = run_b2(b2, torch, cuda, q, kc, vc, bt, lens)
    np.testing.assert_array_equal(got, got2)


def test_block_size_not_16(b2, oracle, cuda):
    import torch

    rng = np.random.default_rng(12)
    for bs in (1, 8, 32, 48):
        q, kc, vc, bt, lens = random_paged(rng, 3, 4, 4, 64, [5, 77, 200], block_size=bs)
        want = oracle.decode_attn(q, kc, vc, bt, lens)
        got = run_b2(b2, torch, cuda, q, kc, vc, bt, lens)
        np.testing.assert_allclose(got, want, **F32_TOL, err_msg=f"block_size={bs}")


def test_block_size_not_16_bf16(b2, oracle, cuda):
    """bf16 caches at block sizes other than 16: those whose blocks divide the tiles (1, 8,
    32) take the TMA producer, 48 the cp.async gather; G 4, head_dim 128 and 64."""
    import torch

    rng = np.random.default_rng(13)
    for d in (128, 64):
        for bs in (1, 8, 32, 48):
            q, kc, vc, bt, lens = random_paged(rng, 3, 16, 4, d, [5, 77, 1000], block_size=bs, dtype="bf16")
            want = oracle.decode_attn(q, kc, vc, bt, lens)
            got = run_b2(b2, torch, cuda, q, kc, vc, bt, lens)
            np.testing.assert_allclose(got, want, **BF16_TOL, err_msg=f"d={d} block_size={bs}")


def test_config3_scaled_ragged(b2, oracle, cuda):
    """BASELINE config 3 shape (B32, H32/8, d128) at lengths the oracle finishes quickly."""
    import torch

    rng = np.random.default_rng(2024)
    lens = rng.integers(64, 1024, 32)
    for dtype in ("f32", "bf16"):
        q, kc, vc, bt, ln = random_paged(rng, 32, 32, 8, 128, lens, dtype=dtype)
        want = oracle.decode_attn(q, kc, vc, bt, ln, nthreads=0)
        got = run_b2(b2, torch, cuda, q, kc, vc, bt, ln)
        np.testing.assert_allclose(got, want, **(F32_TOL if dtype == "f32" else BF16_TOL))


def test_config3_full_size_properties(b2, cuda):
    """Full config 3 (ctx U[512,8192]): size-independent checks on the GPU result —
    permuting the physical blocks (and the table with them) leaves O unchanged, bf16 output
    agrees with fp32 on the same bf16 values, a sampled subset of sequences matches a
    torch fp64 reference."""
    import torch

    g = torch.Generator(device="cpu").manual_seed(7)
    B, H_q, H_kv, d, bs = 32, 32, 8, 128, 16
    lens = torch.randint(512, 8193, (B,), generator=g, dtype=torch.int32)
    nb = (lens + bs - 1) // bs
    P = int(nb.sum())
    nbps = int(nb.max())
    perm = torch.randperm(P, generator=g).to(torch.int32)
    bt = torch.zeros(B, nbps, dtype=torch.int32)
    off = 0
    for b in range(B):
        bt[b, : nb[b]] = perm[off: off + nb[b]]
        off += int(nb[b])
    dev = cuda
    kc = torch.randn(P, bs, H_kv, d, device=dev).to(torch.bfloat16)
    vc = torch.randn(P, bs, H_kv, d, device=dev).to(torch.bfloat16)
    q = torch.randn(B, H_q, d, device=dev)
    btd, lensd = bt.to(dev), lens.to(dev)
    o16 = b2.decode_attn(q, kc, vc, btd, lensd, int(lens.max()))
    o32 = b2.decode_attn(q, kc.float(), vc.float(), btd, lensd, int(lens.max()))
    torch.cuda.synchronize()
    assert b2.device_error() == 0
    torch.testing.assert_close(o16, o32, rtol=1e-5, atol=1e-6)
    # physical permutation invariance
    sigma = torch.randperm(P, generator=g).to(dev)
    inv = torch.empty_like(sigma)
    inv[sigma] = torch.arange(P, device=dev)
    kc2 = torch.empty_like(kc)
    vc2 = torch.empty_like(vc)
    kc2[sigma] = kc
    vc2[sigma] = vc
    bt2 = sigma[btd.long()].to(torch.int32)
    o16b = b2.decode_attn(q, kc2, vc2, bt2, lensd, int(lens.max()))
    torch.testing.assert_close(o16b, o16, rtol=0, atol=0)
    # fp64 reference on a few sequences
    for b in (0, 13, 31):
        n = int(lens[b])
        rows = bt[b, : nb[b]].to(dev).long()
        K = kc[rows].reshape(-1, H_kv, d)[:n].double()
        V = vc[rows].reshape(-1, H_kv, d)[:n].double()
        qq = q[b].double().view(H_kv, H_q // H_kv, d)
        s = torch.einsum("hgd,nhd->hgn", qq, K) / d ** 0.5
        p = torch.softmax(s, dim=-1)
        o = torch.einsum("hgn,nhd->hgd", p, V).reshape(H_q, d)
        torch.testing.assert_close(o16[b].double(), o, rtol=1e-4, atol=1e-5)


def test_unsupported_and_invalid_shapes_raise(b2, cuda):
    import torch

    q = torch.zeros(1, 3, 64, device=cuda)
    kc = torch.zeros(2, 16, 1, 64, device=cuda)
    bt = torch.zeros(1, 2, dtype=torch.int32, device=cuda)
    ln = torch.ones(1, dtype=torch.int32, device=cuda)
    with pytest.raises(b2.B2Error, match="unsupported"):
        b2.decode_attn(q, kc, kc, bt, ln, 16)  # GQA group 3: the reference silently does nothing
    q = torch.zeros(1, 1, 96, device=cuda)
    kc = torch.zeros(2, 16, 1, 96, device=cuda)
    with pytest.raises(b2.B2Error, match="unsupported"):
        b2.decode_attn(q, kc, kc, bt, ln, 16)
    ws = torch.zeros(4, dtype=torch.float32, device=cuda)
    q = torch.zeros(1, 1, 64, device=cuda)
    kc = torch.zeros(2, 16, 1, 64, device=cuda)
    with pytest.raises(b2.B2Error, match="unsupported"):
        b2.run_decode_attn(1, 3, 1, 64, q, kc, kc, bt, ln, 16, 16, 2, q, ws)


def test_device_bounds_checks_flag_errors(b2, cuda):
    """A block-table entry outside the pool and a context longer than its table row are
    reported in the device error word (host-side fault injection; nothing faults)."""
    import torch

    rng = np.random.default_rng(5)
    q, kc, vc, bt, lens = random_paged(rng, 2, 4, 4, 64, [40, 40])
    bt[1, 1] = 10_000
    tq, tk, tv, tbt, tl = (to_dev(torch, a, cuda) for a in (q, kc, vc, bt, lens))
    b2.device_error(clear=True)
    b2.decode_attn(tq, tk, tv, tbt, tl, 40)
    assert b2.device_error() & b2.B2_DEVERR_BLOCK_RANGE
    bt[1, 1] = 0
    tbt = to_dev(torch, bt, cuda)
    tl = torch.tensor([40, 40 + 16 * 8], dtype=torch.int32, device=cuda)
    b2.decode_attn(tq, tk, tv, tbt, tl, 40 + 16 * 8)
    assert b2.device_error() & b2.B2_DEVERR_CTX_RANGE
    assert b2.device_error() == 0  # cleared


@pytest.mark.parametrize("kv", ["f32", "bf16"])
def test_bench_workload_full_size_against_oracle(b2, oracle, cuda, kv):
    """The exact inputs the bench's headline line times (config 3: seed 42, B32, H 32/8,
    d128, Σctx 147,397, 16-token blocks behind the seeded shuffled table), every sequence
    and head, against the oracle run on all host threads; then the same through the
    allocation-free entry point. fp32 within rtol 1e-4 / atol 1e-5, bf16 within 2e-2."""
    import torch

    import bench

    lens, bt, P = bench.workload_meta()
    kc, vc = bench.make_kv_shard(torch, P, 0, bench.H_KV, torch.float32, cuda)
    gq = torch.Generator(device=cuda).manual_seed(bench.SEED + 1)
    q = torch.randn(bench.B, bench.H_Q, bench.D, generator=gq, device=cuda)
    if kv == "bf16":
        kc, vc = kc.to(torch.bfloat16), vc.to(torch.bfloat16)
    btd, lensd = torch.from_numpy(bt).to(cuda), torch.from_numpy(lens).to(cuda)
    max_ctx = int(lens.max())
    got = b2.decode_attn(q, kc, vc, btd, lensd, max_ctx).cpu().numpy()
    O = torch.empty_like(q)
    b2.decode_attn_noalloc(q, kc, vc, btd, lensd, max_ctx, O)
    got_na = O.cpu().numpy()
    assert b2.device_error() == 0

    def host(t):
        if t.dtype == torch.bfloat16:
            return t.view(torch.int16).cpu().numpy().view(np.uint16)
        return t.cpu().numpy()

    kh, vh = host(kc), host(vc)
    del kc, vc
    want = oracle.decode_attn(q.cpu().numpy(), kh, vh, bt, lens, nthreads=0)
    tol = F32_TOL if kv == "f32" else BF16_TOL
    np.testing.assert_allclose(got, want, **tol)
    np.testing.assert_allclose(got_na, want, **tol)


def _run_abi(b2, torch, device, q, kc, vc, bt, lens, max_ctx, ws_bytes):
    """b2_decode_attn through the C ABI with a caller workspace of ws_bytes (0: none)."""
    tq, tk, tv, tbt, tl = (to_dev(torch, a, device) for a in (q, kc, vc, bt, lens))
    O = torch.full_like(tq, float("nan"))
    ws = torch.zeros(max(256, ws_bytes), dtype=torch.uint8, device=device)
    kvt = b2.B2_KV_BF16 if tk.dtype == torch.bfloat16 else b2.B2_KV_F32
    B, H_q, d = tq.shape
    a = b2.DecodeAttnArgs(B, H_q, tk.shape[2], d, tq.data_ptr(), tk.data_ptr(), tv.data_ptr(), kvt,
                          tbt.data_ptr(), tl.data_ptr(), int(max_ctx), tk.shape[1], tbt.shape[1], tk.shape[0],
                          0.0, O.data_ptr(), ws.data_ptr() if ws_bytes else None, ws_bytes)
    assert b2.load_library().b2_decode_attn(ctypes.byref(a), None) == b2.B2_OK
    torch.cuda.synchronize()
    assert b2.device_error() == 0
    return O.cpu().numpy()


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_balanced_schedule_cuts_and_groups_units(b2, oracle, cuda, dtype):
    """Config-4 shape (B64, 12 heads, d64, contexts 100-260 with some empty): the balanced
    schedule gives each CTA an equal share of the blocks, so CTAs hold several short
    (sequence, head) units and units are cut across CTAs; every result matches the oracle,
    equals the one-CTA-per-unit schedule (no workspace) within rounding, and a second call
    reproduces the first bit for bit (counters back at zero)."""
    import torch

    rng = np.random.default_rng(64)
    lens = rng.integers(100, 261, 64)
    lens[[3, 17, 40]] = 0
    q, kc, vc, bt, lens = random_paged(rng, 64, 12, 12, 64, lens, dtype=dtype)
    want = oracle.decode_attn(q, kc, vc, bt, lens, nthreads=0)
    tol = F32_TOL if dtype == "f32" else BF16_TOL
    max_ctx = 2048  # long enough a bound that the balanced schedule is planned
    need = b2.decode_attn_workspace_size(64, 12, 12, 64, max_ctx)
    got = _run_abi(b2, torch, cuda, q, kc, vc, bt, lens, max_ctx, need)
    np.testing.assert_allclose(got, want, **tol)
    assert np.all(got[[3, 17, 40]] == 0)
    again = _run_abi(b2, torch, cuda, q, kc, vc, bt, lens, max_ctx, need)
    np.testing.assert_array_equal(got, again)
    whole = _run_abi(b2, torch, cuda, q, kc, vc, bt, lens, max_ctx, 0)
    np.testing.assert_allclose(whole, want, **tol)
    np.testing.assert_allclose(whole, got, rtol=1e-5, atol=1e-6)


def test_balanced_schedule_few_long_sequences(b2, oracle, cuda):
    """Two long sequences and one short, one KV head of G 4 (a head shard): each long unit is
    cut into many equal pieces merged through the workspace; matches the oracle."""
    import torch

    rng = np.random.default_rng(8)
    lens = [6000, 33, 8192]
    q, kc, vc, bt, lens = random_paged(rng, 3, 4, 1, 128, lens)
    want = oracle.decode_attn(q, kc, vc, bt, lens, nthreads=0)
    need = b2.decode_attn_workspace_size(3, 4, 1, 128, 8192)
    got = _run_abi(b2, torch, cuda, q, kc, vc, bt, lens, 8192, need)
    np.testing.assert_allclose(got, want, **F32_TOL)


def test_batch_above_one_launch(b2, oracle, cuda):
    """300 sequences run as two launches (256 + 44) that reuse one workspace; empty and
    one-token contexts included."""
    import torch

    rng = np.random.default_rng(300)
    lens = rng.integers(0, 90, 300)
    lens[[0, 255, 256, 299]] = [0, 1, 0, 89]
    q, kc, vc, bt, lens = random_paged(rng, 300, 4, 2, 64, lens)
    want = oracle.decode_attn(q, kc, vc, bt, lens, nthreads=0)
    got = run_b2(b2, torch, cuda, q, kc, vc, bt, lens)
    np.testing.assert_allclose(got, want, **F32_TOL)


@pytest.mark.parametrize("G,dtype", [(1, "f32"), (2, "f32"), (1, "bf16")])
def test_two_units_per_cta(b2, oracle, cuda, G, dtype):
    """Short units that fill the GPU 1.5 times (max_context_len <= 1024, head_dim 64) run two
    per CTA: an odd unit count (61 x 11 KV heads), empty and one-token contexts, blocks not
    filling the last tile; matches the oracle."""
    import torch

    rng = np.random.default_rng(61 + G)
    B, H_kv = 61, 11
    lens = rng.integers(1, 300, B)
    lens[[0, 30]] = 0
    lens[5] = 1
    q, kc, vc, bt, lens = random_paged(rng, B, G * H_kv, H_kv, 64, lens, dtype=dtype)
    want = oracle.decode_attn(q, kc, vc, bt, lens, nthreads=0)
    tol = F32_TOL if dtype == "f32" else BF16_TOL
    need = b2.decode_attn_workspace_size(B, G * H_kv, H_kv, 64, 1024)
    got = _run_abi(b2, torch, cuda, q, kc, vc, bt, lens, 1024, need)
    np.testing.assert_allclose(got, want, **tol)
    assert np.all(got[[0, 30]] == 0)

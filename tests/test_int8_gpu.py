"""K14 quantiser and INT8 GEMM on the GPU vs the oracle and vs the reference's own K14.

Bars: quantised bytes and scales bit-exact; int32 accumulators bit-exact; dequantised
outputs bit-exact for the plain / bias / residual epilogues (same operations, same
rounding) and within rtol 1e-4 for bias+GELU (host tanhf differs from CUDA's by ulps);
against the reference's K14 built for sm_100a, every epilogue bit-exact.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def quantized_pair(rng, M, N, K):
    A = rng.standard_normal((M, K)).astype(np.float32)
    Bt = rng.standard_normal((N, K)).astype(np.float32)
    return A, Bt


def dev(torch, a, d):
    return torch.from_numpy(np.ascontiguousarray(a)).to(d)


@pytest.mark.parametrize("rows,cols", [(1, 4), (7, 64), (64, 768), (128, 3072), (3, 16384), (2048, 2048)])
def test_quantizer_bit_exact(b2, oracle, cuda, rows, cols):
    import torch

    rng = np.random.default_rng(rows * 7 + cols)
    x = rng.standard_normal((rows, cols)).astype(np.float32)
    if rows > 2:
        x[1] = 0.0                     # all-zero row: scale 1
        x[2, : cols // 2] *= 1e-30     # tiny values
    want_q, want_s = oracle.quantize(x)
    tx = dev(torch, x, cuda)
    q, s = b2.quantize_fp32_to_int8(tx)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), want_s.view(np.uint32))
    np.testing.assert_array_equal(q.cpu().numpy(), want_q)
    # the reference-named entry point
    q2 = torch.empty_like(q)
    s2 = torch.empty_like(s)
    b2.run_quantize_fp32_to_int8(rows, cols, tx, q2, s2)
    torch.cuda.synchronize()
    assert torch.equal(q, q2) and torch.equal(s, s2)
    if oracle.ref_available():
        q3 = torch.empty_like(q)
        s3 = torch.empty_like(s)
        oracle.ref().ref_run_quantize_fp32_to_int8(rows, cols, tx.data_ptr(), q3.data_ptr(), s3.data_ptr())
        assert oracle.ref().ref_sync() == 0
        assert torch.equal(q, q3) and torch.equal(s, s3)


GEMM_SHAPES = [
    (256, 256, 256), (512, 512, 512), (1024, 1024, 1024), (512, 1024, 256),  # reference test shapes
    (2048, 2048, 2048),
    (2000, 2100, 272), (4096, 1024, 512),                                     # CTA-pair path, ragged
    (64, 3072, 768),                                                          # config 2 rectangular
    (64, 2304, 768), (128, 768, 3072),                                        # decode-step linears
    (100, 200, 48), (1, 16, 16), (130, 17, 4096), (129, 300, 144),            # ragged edges
    (5, 7, 20), (3, 9, 4),                                                    # K % 16 != 0
]


@pytest.mark.parametrize("M,N,K", GEMM_SHAPES)
def test_gemm_s32_bit_exact(b2, oracle, cuda, M, N, K):
    import torch

    rng = np.random.default_rng(M + 3 * N + 7 * K)
    A8 = rng.integers(-128, 128, (M, K), dtype=np.int8)
    B8 = rng.integers(-128, 128, (N, K), dtype=np.int8)
    A8[0, :] = -128  # extremes: |acc| up to K * 128^2
    B8[0, :] = -128
    Ap, Bp = A8.view(np.int32), B8.view(np.int32)
    want = oracle.int8_gemm_s32(Ap, Bp, nthreads=0)
    got = b2.int8_gemm_s32(dev(torch, Ap, cuda), dev(torch, Bp, cuda))
    torch.cuda.synchronize()
    assert b2.device_error() == 0
    np.testing.assert_array_equal(got.cpu().numpy(), want)


@pytest.mark.parametrize("M,N,K", [(256, 256, 256), (2048, 2048, 2048), (2000, 2100, 272), (64, 3072, 768),
                                   (100, 200, 48), (5, 7, 20)])
@pytest.mark.parametrize("epi", [0, 1, 2, 3])
def test_gemm_epilogues(b2, oracle, cuda, M, N, K, epi):
    import torch

    rng = np.random.default_rng(M * 31 + N + K + epi)
    A, Bt = quantized_pair(rng, M, N, K)
    Ap, sA = oracle.quantize(A)
    Bp, sB = oracle.quantize(Bt)
    bias = rng.standard_normal(N).astype(np.float32)
    res = rng.standard_normal((M, N)).astype(np.float32)
    acc = oracle.int8_gemm_s32(Ap, Bp, nthreads=0)
    want = oracle.epilogue(acc, sA, sB, bias, res, epi)
    t = {k: dev(torch, v, cuda) for k, v in dict(Ap=Ap, Bp=Bp, sA=sA, sB=sB, bias=bias, res=res).items()}
    got = b2.int8_gemm(t["Ap"], t["Bp"], t["sA"], t["sB"], t["bias"] if epi else None,
                       t["res"] if epi == 3 else None, epilogue=epi)
    torch.cuda.synchronize()
    g = got.cpu().numpy()
    if epi == 2:
        np.testing.assert_allclose(g, want, rtol=1e-4, atol=1e-6)
    else:
        np.testing.assert_array_equal(g.view(np.uint32), want.view(np.uint32))
    # reference-named entry points give the same bits
    C2 = torch.empty_like(got)
    if epi == 0:
        b2.run_int8_gemm(M, N, K, t["Ap"], t["Bp"], t["sA"], t["sB"], C2)
    elif epi == 1:
        b2.run_int8_gemm_bias(M, N, K, t["Ap"], t["Bp"], t["sA"], t["sB"], t["bias"], C2)
    elif epi == 2:
        b2.run_int8_gemm_bias_gelu(M, N, K, t["Ap"], t["Bp"], t["sA"], t["sB"], t["bias"], C2)
    else:
        b2.run_int8_gemm_bias_residual(M, N, K, t["Ap"], t["Bp"], t["sA"], t["sB"], t["bias"], t["res"], C2)
    torch.cuda.synchronize()
    assert torch.equal(C2, got)
    if oracle.ref_available():
        C3 = torch.zeros_like(got)
        oracle.ref().ref_run_int8_gemm(M, N, K, t["Ap"].data_ptr(), t["Bp"].data_ptr(), t["sA"].data_ptr(),
                                       t["sB"].data_ptr(), t["bias"].data_ptr(), t["res"].data_ptr(),
                                       C3.data_ptr(), epi)
        assert oracle.ref().ref_sync() == 0
        diff = (C3 != got).sum().item()
        assert diff == 0, f"{diff} outputs differ from the reference K14 (max |d| {(C3 - got).abs().max().item()})"


def test_gemm_8192_properties(b2, cuda):
    """North-star size M=N=K=8192: exact row-sum identity sum_n C[m,n] = A[m,:] . colsum(B)
    (fp64 is exact at these magnitudes) plus exact sampled entries."""
    import torch

    n = 8192
    g = torch.Generator(device=cuda).manual_seed(9)
    A8 = torch.randint(-127, 128, (n, n), dtype=torch.int8, device=cuda, generator=g)
    B8 = torch.randint(-127, 128, (n, n), dtype=torch.int8, device=cuda, generator=g)
    C = b2.int8_gemm_s32(A8.view(torch.int32), B8.view(torch.int32))
    torch.cuda.synchronize()
    assert b2.device_error() == 0
    rs = C.double().sum(dim=1)
    want = A8.double() @ B8.double().sum(dim=0)
    assert torch.equal(rs, want)
    idx_m = torch.randint(0, n, (2048,), device=cuda, generator=g)
    idx_n = torch.randint(0, n, (2048,), device=cuda, generator=g)
    exact = (A8[idx_m].double() * B8[idx_n].double()).sum(dim=1)
    assert torch.equal(C[idx_m, idx_n].double(), exact)


def test_gemm_invalid_args(b2, cuda):
    import torch

    A = torch.zeros(4, 2, dtype=torch.int32, device=cuda)
    s = torch.ones(4, device=cuda)
    with pytest.raises(b2.B2Error, match="invalid"):
        b2.int8_gemm(A, A, s, s, epilogue=b2.EPI_BIAS)  # bias missing
    with pytest.raises(b2.B2Error, match="invalid"):
        b2.int8_gemm(A, A, s, s, torch.zeros(4, device=cuda), epilogue=b2.EPI_BIAS_RESIDUAL)


SPLIT_SHAPES = [(64, 768, 3072), (64, 2304, 768), (64, 3072, 768), (1, 768, 3072), (128, 768, 1536),
                (100, 200, 1024), (3, 50, 2048)]


@pytest.mark.parametrize("M,N,K", SPLIT_SHAPES)
@pytest.mark.parametrize("epi", [0, 1, 2, 3])
def test_gemm_split_k_bit_exact(b2, oracle, cuda, M, N, K, epi):
    """Split-K (workspace) path: int32 partials summed exactly, so the output equals the
    unsplit kernel bit for bit and the oracle as in test_gemm_epilogues; repeated calls reuse
    the workspace (its tickets return to zero)."""
    import torch

    assert b2.int8_gemm_workspace_size(M, N, K) > 0
    rng = np.random.default_rng(M * 7 + N + K + epi)
    A, Bt = quantized_pair(rng, M, N, K)
    Ap, sA = oracle.quantize(A)
    Bp, sB = oracle.quantize(Bt)
    bias = rng.standard_normal(N).astype(np.float32)
    res = rng.standard_normal((M, N)).astype(np.float32)
    want = oracle.epilogue(oracle.int8_gemm_s32(Ap, Bp, nthreads=0), sA, sB, bias, res, epi)
    t = {k: dev(torch, v, cuda) for k, v in dict(Ap=Ap, Bp=Bp, sA=sA, sB=sB, bias=bias, res=res).items()}
    ws = b2.make_gemm_workspace(M, N, K, device=cuda)
    args = (t["Ap"], t["Bp"], t["sA"], t["sB"], t["bias"] if epi else None, t["res"] if epi == 3 else None)
    plain = b2.int8_gemm(*args, epilogue=epi)
    for _ in range(2):
        got = b2.int8_gemm(*args, epilogue=epi, workspace=ws)
        torch.cuda.synchronize()
        assert b2.device_error() == 0
        assert torch.equal(got, plain)
    g = got.cpu().numpy()
    if epi == 2:
        np.testing.assert_allclose(g, want, rtol=1e-4, atol=1e-6)
    else:
        np.testing.assert_array_equal(g.view(np.uint32), want.view(np.uint32))
    assert int(ws[:256].view(torch.int32).abs().sum()) == 0  # tickets back to zero


# Reduce-scatter split (workspace given, activation >= 256 KB): 128-column tiles whose K range
# is split over a cluster of 2, 4 or 8 CTAs, int32 partial slices exchanged through the
# workspace; exact, so equal to the oracle bit for bit.
RS_SHAPES = [
    (128, 4096, 4096),   # 4-CTA clusters, 32-column slices
    (128, 2048, 4096),   # 8 or 4 CTAs (as many as stay resident)
    (128, 6144, 4096),   # 2-CTA clusters, 64-column slices
    (128, 768, 4096),    # 8-CTA clusters over 6 tiles
    (100, 1000, 8192),   # ragged rows and a ragged last tile
    (64, 1536, 4096),    # 64 rows (A = 256 KB)
    (128, 3072, 2064),   # K tail past the last full k-block
]


@pytest.mark.parametrize("M,N,K", RS_SHAPES)
@pytest.mark.parametrize("epi", [0, 1, 2, 3, "s32"])
def test_gemm_reduce_scatter_bit_exact(b2, oracle, cuda, M, N, K, epi):
    import torch

    assert b2.int8_gemm_workspace_size(M, N, K) > 0
    rng = np.random.default_rng(M * 11 + N * 3 + K)
    A, Bt = quantized_pair(rng, M, N, K)
    Ap, sA = oracle.quantize(A)
    Bp, sB = oracle.quantize(Bt)
    acc = oracle.int8_gemm_s32(Ap, Bp, nthreads=0)
    t = {k: dev(torch, v, cuda) for k, v in dict(Ap=Ap, Bp=Bp, sA=sA, sB=sB).items()}
    ws = b2.make_gemm_workspace(M, N, K, device=cuda)
    if epi == "s32":
        for _ in range(2):  # repeated launches reuse the exchange rows
            got = b2.int8_gemm_s32(t["Ap"], t["Bp"], workspace=ws)
            torch.cuda.synchronize()
            assert b2.device_error() == 0
            np.testing.assert_array_equal(got.cpu().numpy(), acc)
        return
    bias = rng.standard_normal(N).astype(np.float32)
    res = rng.standard_normal((M, N)).astype(np.float32)
    want = oracle.epilogue(acc, sA, sB, bias, res, epi)
    for _ in range(2):
        got = b2.int8_gemm(t["Ap"], t["Bp"], t["sA"], t["sB"], dev(torch, bias, cuda) if epi else None,
                           dev(torch, res, cuda) if epi == 3 else None, epilogue=epi, workspace=ws)
        torch.cuda.synchronize()
        assert b2.device_error() == 0
        g = got.cpu().numpy()
        if epi == 2:
            np.testing.assert_allclose(g, want, rtol=1e-4, atol=1e-6)
        else:
            np.testing.assert_array_equal(g.view(np.uint32), want.view(np.uint32))


# Decode-size GEMMs (M <= 128: one row tile, skinny 32-column tiles, A boxes trimmed to the
# batch rows): every epilogue and the raw int32 view, ragged M and N, K tails.
DECODE_SHAPES = [
    (64, 768, 3072),     # GPT-2 FC2 (K split over a cluster of 4 CTAs per tile)
    (64, 768, 1536),     # K split over a cluster of 2
    (100, 800, 3072),    # cluster split with ragged rows and columns
    (128, 768, 4096),    # cluster split, full 128-row tile
    (64, 2304, 768),     # GPT-2 QKV
    (1, 768, 768),       # one sequence
    (33, 1000, 640),     # ragged last tile
    (7, 130, 1040),      # N % 4 != 0 (scalar stores), K tail of 16 past the last full k-block
    (128, 2048, 4096),   # config-5 shard: 128-column tiles, K reduce-scattered over 8 CTAs
    (128, 4096, 4096),   # reduce-scatter over 4 CTAs (32-column slices)
    (128, 6144, 4096),   # reduce-scatter over 2 CTAs (64-column slices)
    (100, 1000, 8192),   # reduce-scatter with ragged rows and a ragged last tile
    (64, 1536, 4096),    # reduce-scatter at 64 rows (A = 256 KB)
    (100, 200, 48),      # one k-block
    (120, 4100, 272),    # wide N, 3 k-blocks
]


@pytest.mark.parametrize("M,N,K", DECODE_SHAPES)
@pytest.mark.parametrize("epi", [0, 1, 2, 3, "s32"])
def test_gemm_decode_shapes_bit_exact(b2, oracle, cuda, M, N, K, epi):
    import torch

    rng = np.random.default_rng(M * 13 + N * 5 + K)
    A, Bt = quantized_pair(rng, M, N, K)
    Ap, sA = oracle.quantize(A)
    Bp, sB = oracle.quantize(Bt)
    acc = oracle.int8_gemm_s32(Ap, Bp, nthreads=0)
    t = {k: dev(torch, v, cuda) for k, v in dict(Ap=Ap, Bp=Bp, sA=sA, sB=sB).items()}
    if epi == "s32":
        for _ in range(2):  # repeated launches: nothing is left behind between calls
            got = b2.int8_gemm_s32(t["Ap"], t["Bp"])
            torch.cuda.synchronize()
            assert b2.device_error() == 0
            np.testing.assert_array_equal(got.cpu().numpy(), acc)
        return
    bias = rng.standard_normal(N).astype(np.float32)
    res = rng.standard_normal((M, N)).astype(np.float32)
    want = oracle.epilogue(acc, sA, sB, bias, res, epi)
    got = b2.int8_gemm(t["Ap"], t["Bp"], t["sA"], t["sB"], dev(torch, bias, cuda) if epi else None,
                       dev(torch, res, cuda) if epi == 3 else None, epilogue=epi)
    torch.cuda.synchronize()
    assert b2.device_error() == 0
    g = got.cpu().numpy()
    if epi == 2:
        np.testing.assert_allclose(g, want, rtol=1e-4, atol=1e-6)
    else:
        np.testing.assert_array_equal(g.view(np.uint32), want.view(np.uint32))

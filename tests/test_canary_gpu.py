"""Guard bytes around every output and workspace: the kernels write inside their buffers only.

compute-sanitizer is closed on this pool, so out-of-bounds stores are caught this way: each
output (and the caller-owned workspaces) is carved out of a larger allocation whose other bytes
hold a fixed pattern, the call runs on ragged and edge-case shapes (empty contexts, empty
splits, partial tiles, K not a multiple of 16, split-K), and afterwards every guard byte must
still hold the pattern and the output must match the oracle."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GUARD = 4096
PATTERN = 0xA5


class Guarded:
    """A region of `nbytes` (256-byte aligned) inside a buffer of guard bytes."""

    def __init__(self, torch, device, nbytes, zero=False):
        self.n = int(nbytes)
        self.buf = torch.full((GUARD + self.n + GUARD,), PATTERN, dtype=torch.uint8, device=device)
        if zero:
            self.buf[GUARD:GUARD + self.n].zero_()

    def view(self, dtype, shape):
        import math

        t = self.buf[GUARD:GUARD + self.n].view(dtype)
        return t[: math.prod(shape)].view(*shape)

    def check(self, what):
        b = self.buf.cpu().numpy()
        assert np.all(b[:GUARD] == PATTERN), f"{what}: bytes written before the buffer"
        assert np.all(b[GUARD + self.n:] == PATTERN), f"{what}: bytes written past the end"


def _nbytes(torch, dtype, shape):
    import math

    return math.prod(shape) * torch.tensor([], dtype=dtype).element_size()


@pytest.mark.parametrize("d,kv,G", [(128, "f32", 4), (64, "bf16", 8), (128, "bf16", 1)])
def test_decode_attention_stays_in_its_buffers(b2, oracle, cuda, d, kv, G):
    import torch

    from test_decode_attn_gpu import BF16_TOL, F32_TOL, random_paged, to_dev

    rng = np.random.default_rng(31 + d + G)
    lens = [0, 3, 4000, 0, 63 * 16, 17]
    H_kv = 2
    q, kc, vc, bt, lens = random_paged(rng, len(lens), G * H_kv, H_kv, d, lens, dtype=kv)
    tq, tk, tv, tbt, tl = (to_dev(torch, a, cuda) for a in (q, kc, vc, bt, lens))
    max_ctx = int(lens.max())
    ws = Guarded(torch, cuda, b2.decode_attn_workspace_size(len(lens), G * H_kv, H_kv, d, max_ctx), zero=True)
    o = Guarded(torch, cuda, _nbytes(torch, torch.float32, tq.shape))
    O = o.view(torch.float32, tq.shape)
    W = ws.view(torch.uint8, (ws.n,))
    for _ in range(2):  # the second call reuses the workspace counters
        b2.decode_attn(tq, tk, tv, tbt, tl, max_ctx, O=O, workspace=W)
    torch.cuda.synchronize()
    assert b2.device_error() == 0
    o.check("O")
    ws.check("workspace")
    np.testing.assert_allclose(O.cpu().numpy(), oracle.decode_attn(q, kc, vc, bt, lens),
                               **(F32_TOL if kv == "f32" else BF16_TOL))
    # the allocation-free entry point writes O only
    o2 = Guarded(torch, cuda, _nbytes(torch, torch.float32, tq.shape))
    O2 = o2.view(torch.float32, tq.shape)
    b2.decode_attn_noalloc(tq, tk, tv, tbt, tl, max_ctx, O2)
    torch.cuda.synchronize()
    o2.check("O (noalloc)")
    np.testing.assert_allclose(O2.cpu().numpy(), O.cpu().numpy(), **(F32_TOL if kv == "f32" else BF16_TOL))


def test_quantiser_stays_in_its_buffers(b2, oracle, cuda):
    import torch

    rng = np.random.default_rng(32)
    x = rng.standard_normal((7, 100)).astype(np.float32)
    q = Guarded(torch, cuda, 7 * 25 * 4)
    s = Guarded(torch, cuda, 7 * 4)
    b2.quantize_fp32_to_int8(torch.from_numpy(x).to(cuda), out=q.view(torch.int32, (7, 25)),
                             scales=s.view(torch.float32, (7,)))
    torch.cuda.synchronize()
    q.check("packed int8")
    s.check("scales")
    qw, sw = oracle.quantize(x)
    np.testing.assert_array_equal(q.view(torch.int32, (7, 25)).cpu().numpy(), qw)
    np.testing.assert_array_equal(s.view(torch.float32, (7,)).cpu().numpy(), sw)


@pytest.mark.parametrize("M,N,K,split", [(77, 130, 96, False),    # partial tiles, tensor-core path
                                         (5, 40, 100, False),     # K % 16 != 0: SIMT path
                                         (64, 2304, 768, True),   # decode shape, split-K workspace
                                         (100, 1000, 8192, True),  # reduce-scatter exchange rows, ragged
                                         (1800, 2100, 256, False)])  # CTA-pair path (72 tiles), ragged edges
def test_int8_gemm_stays_in_its_buffers(b2, oracle, cuda, M, N, K, split):
    import torch

    rng = np.random.default_rng(M + N + K)
    A = rng.integers(-127, 128, (M, K), dtype=np.int8).view(np.int32)
    Bt = rng.integers(-127, 128, (N, K), dtype=np.int8).view(np.int32)
    sA = rng.random(M).astype(np.float32)
    sB = rng.random(N).astype(np.float32)
    bias = rng.standard_normal(N).astype(np.float32)
    res = rng.standard_normal((M, N)).astype(np.float32)
    dev = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    c = Guarded(torch, cuda, M * N * 4)
    C = c.view(torch.float32, (M, N))
    ws = None
    if split:
        ws = Guarded(torch, cuda, max(256, b2.int8_gemm_workspace_size(M, N, K)), zero=True)
    b2.int8_gemm(dev(A), dev(Bt), dev(sA), dev(sB), bias=dev(bias), residual=dev(res),
                 epilogue=b2.EPI_BIAS_RESIDUAL, C=C, workspace=None if ws is None else ws.view(torch.uint8, (ws.n,)))
    torch.cuda.synchronize()
    assert b2.device_error() == 0
    c.check("C")
    if ws is not None:
        ws.check("split-K workspace")
    want = oracle.int8_gemm(A, Bt, sA, sB, bias=bias, residual=res, epi=b2.EPI_BIAS_RESIDUAL)
    np.testing.assert_array_equal(C.cpu().numpy(), want)
    c32 = Guarded(torch, cuda, M * N * 4)
    C32 = c32.view(torch.int32, (M, N))
    b2.int8_gemm_s32(dev(A), dev(Bt), C=C32)
    torch.cuda.synchronize()
    c32.check("C (int32)")
    np.testing.assert_array_equal(C32.cpu().numpy(), oracle.int8_gemm_s32(A, Bt))

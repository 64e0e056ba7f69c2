"""b2_decode_attn_noalloc: decode attention for callers that cannot allocate device memory.

Some hosts of this library cannot call cudaMalloc at the point where they run decode
attention (code inside someone else's stream capture, plugin hosts that own the
allocator, loops that forbid allocation after start-up) and cannot pass a workspace
either. This entry point uses the library's fixed per-GPU scratch array instead. These
checks call it through the C ABI and compare it with b2_decode_attn (which takes a caller
workspace) on the same inputs, twice in a row, because the shared scratch keeps the
previous call's contents. Tolerance: the same bar as the other fp32 decode tests
(rtol 1e-4, atol 1e-5); in practice the two paths run the same kernel on the same plan.
"""
import ctypes

import pytest

pytestmark = pytest.mark.gpu


def _inputs(torch, dev, seed, B, H_q, H_kv, d, lens, dtype=None, bs=16):
    g = torch.Generator(device="cpu").manual_seed(seed)
    lens = torch.tensor(lens, dtype=torch.int32)
    nb = (lens + bs - 1) // bs
    P = int(nb.sum()) + 3
    perm = torch.randperm(P, generator=g).to(torch.int32)
    bt = torch.zeros(B, int(nb.max()), dtype=torch.int32)
    off = 0
    for b in range(B):
        bt[b, : nb[b]] = perm[off: off + nb[b]]
        off += int(nb[b])
    kc = torch.randn(P, bs, H_kv, d, generator=g)
    vc = torch.randn(P, bs, H_kv, d, generator=g)
    q = torch.randn(B, H_q, d, generator=g)
    if dtype is not None:
        kc, vc = kc.to(dtype), vc.to(dtype)
    return [t.to(dev) for t in (q, kc, vc, bt, lens)]


@pytest.mark.parametrize("case", [
    dict(B=32, H_q=32, H_kv=8, d=128, lens=list(range(256, 256 + 32 * 61, 61))),   # config-3 shape, ragged
    dict(B=1, H_q=12, H_kv=12, d=64, lens=[1024]),                                 # config 1
    dict(B=5, H_q=8, H_kv=1, d=64, lens=[0, 1, 17, 600, 2000], dtype="bf16"),      # empty splits, bf16
])
def test_noalloc_matches_workspace_entry_point(b2, cuda, case):
    import torch

    dtype = torch.bfloat16 if case.get("dtype") == "bf16" else None
    q, kc, vc, bt, lens = _inputs(torch, cuda, 1234, case["B"], case["H_q"], case["H_kv"], case["d"], case["lens"],
                                  dtype)
    max_ctx = max(1, max(case["lens"]))
    need = b2.decode_attn_workspace_size(case["B"], case["H_q"], case["H_kv"], case["d"], max_ctx)
    assert need <= b2.DECODE_NOALLOC_SCRATCH_BYTES
    want = b2.decode_attn(q, kc, vc, bt, lens, max_ctx)
    outs = []
    for call in range(2):
        O = torch.full_like(q, float("nan"))
        if call == 1:
            torch.cuda.synchronize()
            free_before = torch.cuda.mem_get_info()[0]
        b2.decode_attn_noalloc(q, kc, vc, bt, lens, max_ctx, O)
        torch.cuda.synchronize()
        if call == 1:
            assert torch.cuda.mem_get_info()[0] == free_before  # nothing was allocated
        assert b2.device_error() == 0
        torch.testing.assert_close(O, want, rtol=1e-4, atol=1e-5)
        outs.append(O)
    torch.testing.assert_close(outs[0], outs[1], rtol=0, atol=0)


def test_noalloc_rejects_shapes_beyond_the_scratch(b2, cuda):
    """A batch whose split workspace exceeds the fixed array is refused with a clear status."""
    import torch

    B, H_q, H_kv, d, max_ctx = 256, 64, 8, 128, 32768
    assert b2.decode_attn_workspace_size(B, H_q, H_kv, d, max_ctx) > b2.DECODE_NOALLOC_SCRATCH_BYTES
    q = torch.zeros(B, H_q, d, device=cuda)
    kc = torch.zeros(4, 16, H_kv, d, device=cuda)
    bt = torch.zeros(B, max_ctx // 16, dtype=torch.int32, device=cuda)
    lens = torch.zeros(B, dtype=torch.int32, device=cuda)
    O = torch.zeros_like(q)
    a = b2.DecodeAttnArgs(B, H_q, H_kv, d, q.data_ptr(), kc.data_ptr(), kc.data_ptr(), b2.B2_KV_F32,
                          bt.data_ptr(), lens.data_ptr(), max_ctx, 16, bt.shape[1], 4, 0.0, O.data_ptr(), None, 0)
    st = b2.load_library().b2_decode_attn_noalloc(ctypes.byref(a), None)
    assert st == b2.B2_ERR_WORKSPACE
    with pytest.raises(b2.B2Error, match="workspace"):
        b2.decode_attn_noalloc(q, kc, kc, bt, lens, max_ctx, O)

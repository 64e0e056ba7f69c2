"""b2_decode_attn_noalloc: decode attention for callers that cannot allocate device memory.

Some hosts of this library cannot call cudaMalloc at the point where they run decode
attention (code inside someone else's stream capture, plugin hosts that own the
allocator, loops that forbid allocation after start-up) and cannot pass a workspace
either. This entry point uses the library's fixed per-GPU scratch array instead. These
checks call it through the C ABI, twice in a row (the shared scratch keeps the previous
call's contents), and compare every result with the CPU oracle and with b2_decode_attn
(which takes a caller workspace) on the same inputs. Tolerances are those of the other
decode tests: fp32 KV rtol 1e-4 / atol 1e-5, bf16 KV rtol 2e-2 / atol 2e-3 against the
oracle; against b2_decode_attn rtol 1e-4 / atol 1e-5 (the same kernel; a capped split
count only reorders the fp32 merge).
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

F32_TOL = dict(rtol=1e-4, atol=1e-5)
BF16_TOL = dict(rtol=2e-2, atol=2e-3)


def _inputs(seed, B, H_q, H_kv, d, lens, bf16=False, bs=16):
    """Seeded paged inputs (numpy): a shuffled pool with three spare blocks; bf16 caches are
    returned as their uint16 bit patterns, as the oracle takes them."""
    rng = np.random.default_rng(seed)
    lens = np.asarray(lens, np.int32)
    nb = (lens + bs - 1) // bs
    P = int(nb.sum()) + 3
    perm = rng.permutation(P).astype(np.int32)
    bt = np.zeros((B, max(1, int(nb.max()))), np.int32)
    off = 0
    for b in range(B):
        bt[b, : nb[b]] = perm[off: off + nb[b]]
        off += int(nb[b])
    kc = rng.standard_normal((P, bs, H_kv, d)).astype(np.float32)
    vc = rng.standard_normal((P, bs, H_kv, d)).astype(np.float32)
    q = rng.standard_normal((B, H_q, d)).astype(np.float32)
    if bf16:
        import torch

        kc = torch.from_numpy(kc).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
        vc = torch.from_numpy(vc).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    return q, kc, vc, bt, lens


def _to_dev(torch, a, dev):
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).to(dev)
    return torch.from_numpy(a).to(dev)


def _check_two_calls(b2, torch, cuda, oracle, q, kc, vc, bt, lens, max_ctx, tol):
    want_cpu = oracle.decode_attn(q, kc, vc, bt, lens, nthreads=0)
    tq, tk, tv, tbt, tl = (_to_dev(torch, a, cuda) for a in (q, kc, vc, bt, lens))
    want = b2.decode_attn(tq, tk, tv, tbt, tl, max_ctx)
    outs = []
    for call in range(2):
        O = torch.full_like(tq, float("nan"))
        if call == 1:
            torch.cuda.synchronize()
            free_before = torch.cuda.mem_get_info()[0]
        b2.decode_attn_noalloc(tq, tk, tv, tbt, tl, max_ctx, O)
        torch.cuda.synchronize()
        if call == 1:
            assert torch.cuda.mem_get_info()[0] == free_before  # nothing was allocated
        assert b2.device_error() == 0
        np.testing.assert_allclose(O.cpu().numpy(), want_cpu, **tol)
        torch.testing.assert_close(O, want, rtol=1e-4, atol=1e-5)
        outs.append(O)
    torch.testing.assert_close(outs[0], outs[1], rtol=0, atol=0)


@pytest.mark.parametrize("case", [
    dict(B=32, H_q=32, H_kv=8, d=128, lens=list(range(256, 256 + 32 * 61, 61))),   # config-3 shape, ragged
    dict(B=1, H_q=12, H_kv=12, d=64, lens=[1024]),                                 # config 1
    dict(B=5, H_q=8, H_kv=1, d=64, lens=[0, 1, 17, 600, 2000], bf16=True),         # empty splits, bf16
])
def test_noalloc_matches_oracle_and_workspace_entry_point(b2, oracle, cuda, case):
    import torch

    q, kc, vc, bt, lens = _inputs(1234, case["B"], case["H_q"], case["H_kv"], case["d"], case["lens"],
                                  case.get("bf16", False))
    max_ctx = max(1, max(case["lens"]))
    need = b2.decode_attn_workspace_size(case["B"], case["H_q"], case["H_kv"], case["d"], max_ctx)
    assert need <= b2.DECODE_NOALLOC_SCRATCH_BYTES
    _check_two_calls(b2, torch, cuda, oracle, q, kc, vc, bt, lens, max_ctx,
                     BF16_TOL if case.get("bf16") else F32_TOL)


@pytest.mark.parametrize("bf16", [False, True])
def test_noalloc_caps_splits_to_the_scratch(b2, oracle, cuda, bf16):
    """A batch whose balanced schedule needs more workspace than the fixed array holds runs
    each (sequence, KV head) whole in one CTA, which needs no scratch, and still matches."""
    import torch

    B, H_q, H_kv, d, max_ctx = 256, 128, 16, 128, 32768
    assert b2.decode_attn_workspace_size(B, H_q, H_kv, d, max_ctx) > b2.DECODE_NOALLOC_SCRATCH_BYTES
    lens = np.random.default_rng(9).integers(0, 100, B)
    q, kc, vc, bt, lens = _inputs(77, B, H_q, H_kv, d, lens, bf16)
    _check_two_calls(b2, torch, cuda, oracle, q, kc, vc, bt, lens, max_ctx, BF16_TOL if bf16 else F32_TOL)


def test_noalloc_rejects_bad_arguments(b2, cuda):
    """Invalid arguments are refused with a status before anything is launched: a null
    output, an unsupported GQA group, an unsupported cache dtype (host mirror)."""
    import torch

    B, H_q, H_kv, d = 2, 4, 2, 64
    q = torch.zeros(B, H_q, d, device=cuda)
    kc = torch.zeros(4, 16, H_kv, d, device=cuda)
    bt = torch.zeros(B, 4, dtype=torch.int32, device=cuda)
    lens = torch.zeros(B, dtype=torch.int32, device=cuda)
    lib = b2.load_library()
    a = b2.DecodeAttnArgs(B, H_q, H_kv, d, q.data_ptr(), kc.data_ptr(), kc.data_ptr(), b2.B2_KV_F32,
                          bt.data_ptr(), lens.data_ptr(), 64, 16, 4, 4, 0.0, None, None, 0)
    assert lib.b2_decode_attn_noalloc(ctypes.byref(a), None) == b2.B2_ERR_INVALID
    a = b2.DecodeAttnArgs(B, 3, 1, d, q.data_ptr(), kc.data_ptr(), kc.data_ptr(), b2.B2_KV_F32,
                          bt.data_ptr(), lens.data_ptr(), 64, 16, 4, 4, 0.0, q.data_ptr(), None, 0)
    assert lib.b2_decode_attn_noalloc(ctypes.byref(a), None) == b2.B2_ERR_UNSUPPORTED
    with pytest.raises(b2.B2Error, match="KV dtype"):
        b2.decode_attn_noalloc(q, kc.half(), kc.half(), bt, lens, 64, torch.zeros_like(q))

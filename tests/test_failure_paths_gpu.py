"""A bounded device wait that runs out leaves an error status, not a hung GPU.

The row-parallel quantiser of the tensor-parallel decode step waits for every rank's row
maximum. Run as rank 0 of a 2-rank group whose other rank never arrives (its exchange region
is a local buffer nothing writes), each row's wait gives up after its 2 s bound, the kernel
sets B2_DEVERR_TIMEOUT in the device error word and finishes with this rank's own maxima; the
host reads the status, and the same context then runs a decode-attention call correctly."""
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_missing_peer_times_out_and_the_context_stays_usable(b2, oracle, cuda):
    import torch

    rng = np.random.default_rng(21)
    x_np = rng.standard_normal((4, 64)).astype(np.float32)
    x_np[2, 5] = 7.0
    x = torch.from_numpy(x_np).to(cuda)
    b2.device_error(clear=True)
    t0 = time.time()
    q, s = b2.tp_quantize_absent_peer(x)
    torch.cuda.synchronize()
    waited = time.time() - t0
    assert b2.device_error() & b2.B2_DEVERR_TIMEOUT
    assert 1.0 < waited < 60.0
    # the absent rank's slots stayed zero, so the scales are this rank's own row maxima
    q_want, s_want = oracle.quantize(x_np)
    np.testing.assert_array_equal(q.cpu().numpy(), q_want)
    np.testing.assert_array_equal(s.cpu().numpy(), s_want)
    # the context survives: decode attention right after is correct and raises nothing
    from test_decode_attn_gpu import F32_TOL, random_paged, run_b2

    qa, kc, vc, bt, lens = random_paged(rng, 2, 8, 2, 128, [33, 300])
    want = oracle.decode_attn(qa, kc, vc, bt, lens)
    got = run_b2(b2, torch, cuda, qa, kc, vc, bt, lens)
    np.testing.assert_allclose(got, want, **F32_TOL)

"""Tensor-parallel decode (2 GPUs) equals the single-GPU engine.

The sharded engine quantises row-parallel inputs with the global row scale and sums exact
int32 partials over the ranks, so every int8 byte and int32 accumulator matches the unsharded
run, whether the exchange goes through the peer-memory kernels (default) or NCCL all-reduces
(B2_TP_COLLECTIVES=nccl); after the eager steps each rank replays the step as a CUDA graph
from a restart and must produce the same tokens;
attention and the vocab logits are computed per head / per vocab row by the same kernels. The
bar: identical greedy tokens and positions, and logits within 1e-5 relative (the split-K plan
of the attention may merge a different number of splits per head shard)."""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
CFG = dict(n_layers=2, n_heads=8, d_model=512, d_ff=2048, vocab_size=999, max_seq_len=64, d_head=64)
# batch 128 at d_model 2048: the QKV, FC1 and row-parallel FC2 shards (activations of 256 KB and
# more) take the reduce-scatter GEMM split on both the sharded and the single-GPU engine
WIDE = dict(n_layers=1, n_heads=16, d_model=2048, d_ff=8192, vocab_size=999, max_seq_len=32, d_head=128)


def _need_gpus(n):
    import torch

    if torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")


@pytest.mark.parametrize("model,kv_dtype,collectives",
                         [("small", 0, "p2p"), ("small", 1, "p2p"), ("small", 0, "nccl"), ("wide", 0, "p2p")])
def test_tp2_matches_single_gpu(b2, cuda, tmp_path, model, kv_dtype, collectives):
    _need_gpus(2)
    rng = np.random.default_rng(5)
    cfg = CFG if model == "small" else WIDE
    lens = (4, 7, 2) if model == "small" else tuple(int(n) for n in rng.integers(1, 9, 128))
    prompts = [list(map(int, rng.integers(0, cfg["vocab_size"], n))) for n in lens]
    B = len(prompts)
    spec = dict(cfg=cfg, max_batch=B, kv_dtype=kv_dtype, seed=13, block_seed=2, prompts=prompts, new=5, steps=10)
    nid = b2.nccl_unique_id().hex()
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    env.pop("B2_TP_COLLECTIVES", None)
    if collectives == "nccl":
        env["B2_TP_COLLECTIVES"] = "nccl"
    procs = [subprocess.Popen([sys.executable, os.path.join(HERE, "tp_worker.py"), str(r), "2", nid, json.dumps(spec),
                               str(tmp_path / f"r{r}.npz")], env=env) for r in range(2)]
    for p in procs:
        assert p.wait(timeout=300) == 0
    outs = [np.load(tmp_path / f"r{r}.npz") for r in range(2)]
    e = b2.Engine.random(cfg, max_batch=B, kv_dtype=kv_dtype, seed=13)
    e.start(prompts, 5, seed=2)
    e.keep_logits(True)
    ref = []
    for _ in range(spec["steps"]):
        e.step()
        ref.append(e.logits())
    ref = np.stack(ref)
    for o in outs:
        assert np.array_equal(o["tokens"], e.tokens())
        assert np.array_equal(o["pos"], e.positions())
        assert np.array_equal(o["graph_tokens"], e.tokens())
    tp_logits = np.concatenate([outs[0]["logits"], outs[1]["logits"]], axis=2)
    np.testing.assert_allclose(tp_logits, ref, rtol=1e-5, atol=1e-5 * np.abs(ref).max())

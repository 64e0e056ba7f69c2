"""World-size-2 gloo runs of the multi-rank host logic, on the CPU (no GPU needed).

- Config 3 shards by KV head with no collective on the data path: the heads bench.py gives
  each rank, with the KV shard it builds, must reproduce the unsharded attention exactly
  (oracle per head), and the whole-job time is the max over the ranks.
- The tensor-parallel decode step keeps every int8 byte and int32 accumulator of one GPU: a
  row-parallel linear quantises its K slice with the global per-row absmax (all-reduce max)
  and sums exact int32 partials (all-reduce sum); a column-parallel linear computes its own
  output columns; the greedy token is the all-reduce max of the vocab shards' 64-bit keys.
  All are checked bit-exact against the single-rank computation.
- A rank that leaves before a collective, or never starts: the survivor's next collective,
  or its rendezvous, ends with an error within the process group's timeout (5 s here)
  instead of hanging.
"""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(scenario, tmp_path, timeout=240, ranks=WORLD):
    port = _free_port()
    env = dict(os.environ, MASTER_ADDR="127.0.0.1", CUDA_VISIBLE_DEVICES="")
    procs = [subprocess.Popen([sys.executable, os.path.join(HERE, "multirank_worker.py"), scenario, str(r),
                               str(WORLD), str(port), str(tmp_path)], env=env,
                              stdout=subprocess.PIPE, stderr=subprocess.STDOUT) for r in range(ranks)]
    logs = []
    try:
        for p in procs:
            out, _ = p.communicate(timeout=timeout)
            logs.append(out.decode(errors="replace"))
    finally:
        for p in procs:
            if p.poll() is None:
                p.kill()
    for p, log in zip(procs, logs):
        assert p.returncode == 0, log[-3000:]
    return [np.load(tmp_path / f"r{r}.npz") if (tmp_path / f"r{r}.npz").exists() else None for r in range(WORLD)]


def test_kv_head_sharding_reproduces_unsharded_attention(oracle, tmp_path):
    import torch

    import bench
    sys.path.insert(0, HERE)
    from multirank_worker import shard_case

    outs = _run("shard", tmp_path)
    lens, bt, P, q, h_kv, h_q = shard_case()
    kc, vc = bench.make_kv_shard(torch, P, 0, h_kv, torch.float32, torch.device("cpu"))
    want = oracle.decode_attn(q, kc.numpy(), vc.numpy(), bt, lens)
    for r, o in enumerate(outs):
        np.testing.assert_array_equal(o["gathered"], want)
        assert float(o["slowest"]) == 1.5 + (WORLD - 1)  # max over ranks of 1.5 + rank
        h0, hkv, _, _ = bench.head_shard(r, WORLD, h_kv=h_kv, h_q=h_q)
        np.testing.assert_array_equal(o["kc"], kc.numpy()[:, :, h0:h0 + hkv])


def test_head_shard_bounds():
    import bench

    assert [bench.head_shard(r, 4) for r in range(4)] == [(0, 2, 0, 8), (2, 2, 8, 8), (4, 2, 16, 8), (6, 2, 24, 8)]
    with pytest.raises(ValueError):
        bench.head_shard(0, 3)  # 8 KV heads over 3 ranks
    with pytest.raises(ValueError):
        bench.head_shard(2, 2)


def test_tensor_parallel_exchange_is_exact(oracle, tmp_path):
    outs = _run("tp", tmp_path)
    x, w, logits = outs[0]["x"], outs[0]["w"], outs[0]["logits"]
    qx, sx = oracle.quantize(x)
    qw, sw = oracle.quantize(w)
    acc = oracle.int8_gemm_s32(qx, qw)
    full = oracle.epilogue(acc, sx, sw)
    K4 = qx.shape[1]
    for r, o in enumerate(outs):
        # the rank's int8 bytes and row scales equal one GPU's
        np.testing.assert_array_equal(o["qx"], qx[:, r * K4 // WORLD:(r + 1) * K4 // WORLD])
        np.testing.assert_array_equal(o["sx"], sx)
        np.testing.assert_array_equal(o["acc"], acc)
        np.testing.assert_array_equal(o["row_par"], full)
        np.testing.assert_array_equal(o["col_par"], full)
        want = np.array([int(np.argmax(row)) for row in logits])  # lowest index on ties
        np.testing.assert_array_equal(o["argmax"], want)
    assert want[1] == 3


def test_rank_that_leaves_is_an_error_not_a_hang(tmp_path):
    outs = _run("drop", tmp_path, timeout=120)
    o = outs[0]
    assert str(o["err"]), "the barrier with a missing rank returned normally"
    assert float(o["elapsed"]) < 60.0


def test_rank_that_never_starts_ends_the_rendezvous_with_an_error(tmp_path):
    o = _run("absent", tmp_path, timeout=120, ranks=1)[0]
    assert str(o["err"]), "the rendezvous without rank 1 returned normally"
    assert float(o["elapsed"]) < 60.0

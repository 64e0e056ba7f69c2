"""One CPU rank of the gloo tests in tests/test_multirank_cpu.py.

    python tests/multirank_worker.py SCENARIO RANK WORLD PORT OUT_DIR

Scenarios (each rank writes OUT_DIR/r<RANK>.npz for the parent to check):
  shard  - config 3's KV-head sharding (bench.head_shard / bench.make_kv_shard) on a small
           batch: each rank runs the attention oracle on its heads; the ranks' outputs are
           all-gathered, and the max-over-ranks timing reduction is exercised.
  tp     - the tensor-parallel decode step's exchange arithmetic on the host: a row-parallel
           linear quantised with the global per-row absmax (all-reduce max) and summed as
           exact int32 partials (all-reduce sum); a column-parallel linear; the vocab-shard
           argmax keys (all-reduce max).
  drop   - rank 1 leaves before the first collective; rank 0's barrier must end with an
           error within the process group's short timeout instead of hanging.
  absent - only rank 0 starts; its rendezvous must end with an error within the timeout.
"""
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def init(rank, world, port, timeout_s):
    import datetime

    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def shard_case():
    """A small config-3-shaped case: batch 3, 8 query / 4 KV heads, bench's head_dim and
    block size, ragged lengths, seeded block table."""
    import bench

    rng = np.random.default_rng(3)
    lens = np.array([5, 40, 70], np.int32)
    nb = (lens + bench.BS - 1) // bench.BS
    P = int(nb.sum()) + 2
    perm = rng.permutation(P).astype(np.int32)
    bt = np.zeros((len(lens), int(nb.max())), np.int32)
    off = 0
    for b in range(len(lens)):
        bt[b, :nb[b]] = perm[off:off + nb[b]]
        off += int(nb[b])
    q = rng.standard_normal((len(lens), 8, bench.D)).astype(np.float32)
    return lens, bt, P, q, 4, 8


def scenario_shard(dist, rank, world, out):
    import torch

    import bench
    from oracle import oracle

    lens, bt, P, q, h_kv, h_q = shard_case()
    h0, hkv, hq0, hq = bench.head_shard(rank, world, h_kv=h_kv, h_q=h_q)
    kc, vc = bench.make_kv_shard(torch, P, h0, h0 + hkv, torch.float32, torch.device("cpu"))
    o = oracle.decode_attn(q[:, hq0:hq0 + hq], kc.numpy(), vc.numpy(), bt, lens)
    parts = [torch.empty(o.shape, dtype=torch.float32) for _ in range(world)]
    dist.all_gather(parts, torch.from_numpy(o))
    gathered = torch.cat(parts, dim=1).numpy()
    slowest = bench.max_over_ranks(dist, 1.5 + rank, "cpu")
    np.savez(out, gathered=gathered, slowest=slowest, kc=kc.numpy())


def vocab_key(v, idx):
    """The engine's 64-bit argmax key (vocab_tc.cu vt_key): float bits made monotone in
    the high word, 0xFFFFFFFF - index in the low word, so the maximum key is the largest
    logit at the lowest index."""
    u = np.asarray(v, np.float32).view(np.uint32).astype(np.uint64)
    u = np.where(u & 0x80000000, (~u) & 0xFFFFFFFF, u | 0x80000000)
    return (u << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - np.asarray(idx, np.uint64))


def scenario_tp(dist, rank, world, out):
    import torch

    from oracle import oracle

    rng = np.random.default_rng(17)
    M, K, N = 5, 256, 48
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = (0.02 * rng.standard_normal((N, K))).astype(np.float32)
    x[2, 7] = 9.0  # a row whose absmax lives on one rank only
    # weights are quantised per output row over the FULL row, then sliced along K
    qw, sw = oracle.quantize(w)
    k0, k1 = rank * K // world, (rank + 1) * K // world
    xs = x[:, k0:k1]
    # 1) global per-row absmax (max over ranks), then quantise the local slice with it: a pad
    #    column holding the global absmax gives the oracle quantiser exactly that row scale
    amax = torch.from_numpy(np.abs(xs).max(axis=1).astype(np.float32))
    dist.all_reduce(amax, op=dist.ReduceOp.MAX)
    pad = np.zeros((M, 4), np.float32)
    pad[:, 0] = amax.numpy()
    qx_pad, sx = oracle.quantize(np.concatenate([xs, pad], axis=1))
    qx = qx_pad[:, :(k1 - k0) // 4]
    # 2) exact int32 partial products, summed over the ranks
    part = torch.from_numpy(oracle.int8_gemm_s32(qx, qw[:, k0 // 4:k1 // 4]))
    dist.all_reduce(part, op=dist.ReduceOp.SUM)
    row_par = oracle.epilogue(part.numpy(), sx, sw)
    # 3) column-parallel: this rank's output rows of the weight, full activation row
    n0, n1 = rank * N // world, (rank + 1) * N // world
    qxf, sxf = oracle.quantize(x)
    col = torch.from_numpy(oracle.epilogue(oracle.int8_gemm_s32(qxf, qw[n0:n1]), sxf, sw[n0:n1]))
    cols = [torch.empty_like(col) for _ in range(world)]
    dist.all_gather(cols, col)
    # 4) vocab shards: the best key of this shard, reduced with max over the ranks (keys are
    #    unsigned; flipping the top bit maps their order onto the signed int64 reduction)
    V = 40
    logits = np.round(rng.standard_normal((M, V)), 1).astype(np.float32)
    logits[1, 3] = logits[1, 33] = 5.0  # a tie across shards: the lower index must win
    v0, v1 = rank * V // world, (rank + 1) * V // world
    keys = vocab_key(logits[:, v0:v1], np.arange(v0, v1)[None, :].repeat(M, 0)).max(axis=1)
    flip = np.uint64(1 << 63)
    kt = torch.from_numpy((keys ^ flip).view(np.int64).copy())
    dist.all_reduce(kt, op=dist.ReduceOp.MAX)
    best = kt.numpy().view(np.uint64) ^ flip
    argmax = (np.uint64(0xFFFFFFFF) - (best & np.uint64(0xFFFFFFFF))).astype(np.int64)
    np.savez(out, qx=qx, sx=sx, acc=part.numpy(), row_par=row_par, col_par=torch.cat(cols, dim=1).numpy(),
             argmax=argmax, x=x, w=w, logits=logits)


def scenario_drop(dist, rank, world, out):
    if rank == 1:
        os._exit(0)  # leaves without taking part in any collective
    t0 = time.time()
    err = ""
    try:
        dist.barrier()
    except Exception as e:  # the expected outcome
        err = f"{type(e).__name__}: {e}"[:300]
    np.savez(out, elapsed=time.time() - t0, err=np.array(err))


def main():
    scenario, rank, world, port, out_dir = sys.argv[1], int(sys.argv[2]), int(sys.argv[3]), int(sys.argv[4]), \
        sys.argv[5]
    out = os.path.join(out_dir, f"r{rank}.npz")
    if scenario == "absent":  # the other ranks never start: the rendezvous must give up
        t0 = time.time()
        err = ""
        try:
            init(rank, world, port, 5)
        except Exception as e:
            err = f"{type(e).__name__}: {e}"[:300]
        np.savez(out, elapsed=time.time() - t0, err=np.array(err))
        return
    dist = init(rank, world, port, 5 if scenario == "drop" else 120)
    {"shard": scenario_shard, "tp": scenario_tp, "drop": scenario_drop}[scenario](dist, rank, world, out)
    if scenario != "drop":
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

"""Benchmark of the B200 decode hot path (one JSON line on rank 0).

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]
    torchrun --nproc-per-node N bench.py --gpus N ...   (N > 1; heads sharded across ranks)

Headline workload: GQA paged decode attention, batch 32, 32 query /
8 KV heads (group 4), head_dim 128, ragged context lengths U[512, 8192] (seeded), 16-token
blocks behind a seeded random block table, fp32 KV cache, Q/K/V ~ N(0,1). One step = one
decode-attention launch over the whole batch. Metric: algorithmic HBM GB/s = bytes of the
live K/V + Q + O + block table + context lengths per step / step time (workspace traffic
excluded). KV heads are sharded across ranks (no collective on the data path); the
whole-job value is total bytes / max-over-ranks time ("strong": total work is fixed).

Secondary lines (N=1 only): the same batch with a bf16 KV cache, BASELINE config 1 (MHA,
B1 H12 d64 ctx1024), and the INT8 GEMMs of config 2 (2048^3, 64x3072x768) plus the
north-star 8192^3, in TOPS.

--impl reference times the reference's CPU implementation of the path (the oracle's
restatement of its CPU attention harness, all host threads) on a bounded sample of the
same workload, on rank 0 only.
"""
from __future__ import annotations

import argparse
import datetime
import importlib
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

SEED = 42
B, H_Q, H_KV, D, BS = 32, 32, 8, 128, 16
CTX_LO, CTX_HI = 512, 8192
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
PG_TIMEOUT_S = 300  # process-group timeout of multi-GPU runs


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), float(j["bf16_tflops"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, "fallback"


def workload_meta():
    """Context lengths, block table and physical block count of the headline workload
    (identical on every rank; numpy, seeded)."""
    import numpy as np

    rng = np.random.default_rng(SEED)
    lens = rng.integers(CTX_LO, CTX_HI + 1, B).astype(np.int32)
    nb = (lens + BS - 1) // BS
    P = int(nb.sum())
    nbps = int(nb.max())
    perm = rng.permutation(P).astype(np.int32)
    bt = np.zeros((B, nbps), np.int32)
    off = 0
    for b in range(B):
        bt[b, : nb[b]] = perm[off: off + nb[b]]
        off += int(nb[b])
    return lens, bt, P


def head_shard(rank, world, h_kv=H_KV, h_q=H_Q):
    """The heads rank `rank` of `world` holds in the sharded config-3 run: KV heads
    [h0, h0 + hkv) and, with them, the query heads [hq0, hq0 + hq) that read them
    (query head h reads KV head h // (h_q // h_kv), as in the reference's GQA mapping)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    if h_kv % world:
        raise ValueError(f"{h_kv} KV heads do not shard over {world} ranks")
    hkv, hq = h_kv // world, h_q // world
    return rank * hkv, hkv, rank * hq, hq


def max_over_ranks(dist, value, device):
    """The maximum of a per-rank float over all ranks (the slowest rank's time)."""
    import torch

    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def attn_alg_bytes(lens, h_kv, h_q, d, kv_bytes, nbps):
    """Algorithmic HBM bytes of one decode-attention call: live K and V rows, Q, O, the
    block table and context lengths, each once."""
    kv = int(lens.sum()) * 2 * h_kv * d * kv_bytes
    qo = 2 * len(lens) * h_q * d * 4
    return kv + qo + len(lens) * nbps * 4 + len(lens) * 4


class ClockMonitor:
    """Samples nvidia-smi clocks and throttle reasons every 100 ms in the background."""

    Q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []
        self.thread = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            time.sleep(0.25)
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=2)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[0]))
                mx = max(mx, float(f[1]))
            except ValueError:
                continue
            for n, v in zip(names, f[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def time_steps(torch, fn, steps, warmup, dist=None):
    """W untimed steps, then K steps bracketed by barrier + synchronize, timed with CUDA
    events on the current stream; returns the max over ranks of the elapsed ms."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(steps):
        fn()
    e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if dist is not None:
        ms = max_over_ranks(dist, ms, "cuda")
        dist.barrier()
    return ms


def graph_of(torch, fn, warm=3):
    """A CUDA graph holding one call of fn (after `warm` eager calls set up the kernels'
    attributes and tensor maps): replaying it runs one step with no Python launch cost, so a
    short step is timed on the device, not on the host's call rate."""
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    torch.cuda.synchronize()
    return g


def make_kv_shard(torch, P, h0, h1, dtype, device):
    """K/V cache [P, BS, h1-h0, D] for KV heads [h0, h1); each head's values come from its
    own seeded generator, so a shard equals the same heads of the unsharded cache."""
    nh = h1 - h0
    kc = torch.empty(P, BS, nh, D, dtype=dtype, device=device)
    vc = torch.empty_like(kc)
    for i, h in enumerate(range(h0, h1)):
        g = torch.Generator(device=device).manual_seed(SEED * 1000 + h)
        kc[:, :, i].copy_(torch.randn(P, BS, D, generator=g, device=device).to(dtype))
        vc[:, :, i].copy_(torch.randn(P, BS, D, generator=g, device=device).to(dtype))
    return kc, vc


def cpu_sample(torch, kc, vc, bt, lens, seqs):
    """Numpy copy of sequences `seqs` of a device KV cache, with the blocks compacted and
    the block table remapped (for the CPU legs)."""
    import numpy as np

    rows, sub_bt = [], np.zeros((len(seqs), bt.shape[1]), np.int32)
    for i, b in enumerate(seqs):
        nb = (int(lens[b]) + BS - 1) // BS
        sub_bt[i, :nb] = np.arange(len(rows), len(rows) + nb)
        rows.extend(int(x) for x in bt[b, :nb])
    idx = torch.tensor(rows, device=kc.device, dtype=torch.long)

    def host(t):
        h = t[idx]
        if h.dtype == torch.bfloat16:
            return h.view(torch.int16).cpu().numpy().view(np.uint16)
        return h.cpu().numpy()

    return host(kc), host(vc), sub_bt, lens[list(seqs)].copy()


def time_cpu_attention(oracle, q, kc, vc, bt, lens, nthreads, budget_s, min_reps=1):
    """Runs the oracle over the sample until `budget_s` seconds have passed (at least
    min_reps times); returns seconds per repetition."""
    reps, t0 = 0, time.perf_counter()
    while True:
        oracle.decode_attn(q, kc, vc, bt, lens, nthreads=nthreads)
        reps += 1
        el = time.perf_counter() - t0
        if reps >= min_reps and el >= budget_s:
            return el / reps
        if el > 4 * budget_s:
            return el / reps


def gemm_secondary(torch, b2, M, N, K, steps, peak_int8, hbm_peak):
    """TOPS of the INT8 GEMM (fp32 dequantised output, plain epilogue) at M x N x K."""
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(SEED + M + N + K)
    # rotate enough operand copies that the working set of consecutive calls exceeds L2
    per = M * K + N * K + 4 * M * N
    copies = max(1, min(16, (512 << 20) // per + 1))
    bufs = []
    for _ in range(copies):
        A = torch.randint(-127, 128, (M, K), dtype=torch.int8, device=dev, generator=g).view(torch.int32)
        Bt = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev, generator=g).view(torch.int32)
        sA = torch.rand(M, device=dev, generator=g) / 127
        sB = torch.rand(N, device=dev, generator=g) / 127
        C = torch.empty(M, N, device=dev)
        bufs.append((A, Bt, sA, sB, C))
    it = [0]

    def step():
        A, Bt, sA, sB, C = bufs[it[0] % copies]
        it[0] += 1
        b2.int8_gemm(A, Bt, sA, sB, C=C)

    # one CUDA graph holds a full rotation of calls, so host launch cost stays out of the timing
    for _ in range(3):
        step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(copies):
            step()
    reps = max(1, min(steps, 200) // copies)
    ms = time_steps(torch, graph.replay, reps, 3)
    n = reps * copies
    tops = 2.0 * M * N * K / (ms / n * 1e-3) / 1e12
    by = gemm_alg_bytes(M, N, K)
    gbs = by / (ms / n * 1e-3) / 1e9
    return {"tops": round(tops, 2), "us_per_call": round(ms / n * 1e3, 2), "frac_of_int8_peak": round(tops / peak_int8, 4),
            "algorithmic_bytes": by, "gbs": round(gbs, 1), "frac_of_hbm_peak": round(gbs / hbm_peak, 4),
            "operand_copies": copies, "timing": "CUDA graph replays"}


def gemm_alg_bytes(M, N, K):
    """HBM bytes an INT8 GEMM must move once: int8 A [M, K] and B^T [N, K], the two fp32 scale
    vectors, and the fp32 output C [M, N] (a decode-shape GEMM is bound by these, not by its
    2MNK operations)."""
    return M * K + N * K + 4 * (M + N) + 4 * M * N


def run_gpu(args):
    import numpy as np
    import torch

    b2 = importlib.import_module("cuda-llm-inference-engine_b200")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as tdist

        # a rank that dies or never joins ends the others' next collective with an error
        # after PG_TIMEOUT_S instead of holding every GPU of the run
        tdist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                 timeout=datetime.timedelta(seconds=PG_TIMEOUT_S))
        dist = tdist
    try:
        h0, hkv, hq0, hq = head_shard(rank, world)
    except ValueError as e:
        raise SystemExit(str(e))
    b2.load_library()
    dev = torch.device("cuda", local)
    hbm_peak, bf16_peak, peak_kind = measured_peaks()

    lens, bt, P = workload_meta()
    nbps = bt.shape[1]
    kc, vc = make_kv_shard(torch, P, h0, h0 + hkv, torch.float32, dev)
    gq = torch.Generator(device=dev).manual_seed(SEED + 1)
    q_full = torch.randn(B, H_Q, D, generator=gq, device=dev)
    q = q_full[:, hq0:hq0 + hq].contiguous()
    O = torch.empty_like(q)
    btd = torch.from_numpy(bt).to(dev)
    lensd = torch.from_numpy(lens).to(dev)
    max_ctx = int(lens.max())
    ws = b2.make_decode_workspace(B, hq, hkv, D, max_ctx, BS, device=dev)

    def step():
        b2.decode_attn(q, kc, vc, btd, lensd, max_ctx, O=O, workspace=ws)

    # one step = one replay of a graph holding the one decode_attn launch
    step_graph = graph_of(torch, step)
    with ClockMonitor(local) as mon:
        ms = time_steps(torch, step_graph.replay, args.steps, args.warmup, dist)
    clocks = mon.summary()
    assert b2.device_error() == 0, "device error during the timed region"
    bytes_rank = attn_alg_bytes(lens, hkv, hq, D, 4, nbps)
    bytes_total = attn_alg_bytes(lens, H_KV, H_Q, D, 4, nbps)
    ms_step = ms / args.steps
    value = bytes_total / (ms_step * 1e-3) / 1e9
    # dominant (only) kernel: one decode_attn_kernel launch per step on this stream
    achieved = bytes_rank / (ms_step * 1e-3) / 1e9

    # ---- end to end through the public API with host buffers: every step copies its own
    # pinned Q, block table and context lengths in and its O out (the KV cache stays
    # resident). Two buffer sets and two copy streams pipeline the steps as a serving loop
    # does: step i+1's inputs cross PCIe while step i's kernel runs, and step i's O comes
    # back meanwhile; each step's kernel waits for its own inputs, each buffer for its last
    # reader.
    cur = torch.cuda.current_stream()
    h2d_st, d2h_st = torch.cuda.Stream(), torch.cuda.Stream()
    slots = []
    for _ in range(2):
        sl = dict(q_h=q.cpu().pin_memory(), bt_h=torch.from_numpy(bt).pin_memory(),
                  lens_h=torch.from_numpy(lens).pin_memory(), o_h=torch.empty_like(q, device="cpu").pin_memory(),
                  q_d=torch.empty_like(q), bt_d=torch.empty_like(btd), lens_d=torch.empty_like(lensd),
                  O=torch.empty_like(q), ws=b2.make_decode_workspace(B, hq, hkv, D, max_ctx, BS, device=dev),
                  h2d=torch.cuda.Event(), kdone=torch.cuda.Event(), d2h=torch.cuda.Event())
        slots.append(sl)
    it = [0]

    def e2e_step():
        sl = slots[it[0] % 2]
        first = it[0] < 2
        it[0] += 1
        with torch.cuda.stream(h2d_st):
            if not first:
                h2d_st.wait_event(sl["kdone"])  # the kernel two steps back has read these inputs
            sl["q_d"].copy_(sl["q_h"], non_blocking=True)
            sl["bt_d"].copy_(sl["bt_h"], non_blocking=True)
            sl["lens_d"].copy_(sl["lens_h"], non_blocking=True)
            sl["h2d"].record(h2d_st)
        cur.wait_event(sl["h2d"])
        if not first:
            cur.wait_event(sl["d2h"])  # O of two steps back has been read out
        b2.decode_attn(sl["q_d"], kc, vc, sl["bt_d"], sl["lens_d"], max_ctx, O=sl["O"], workspace=sl["ws"])
        sl["kdone"].record(cur)
        with torch.cuda.stream(d2h_st):
            d2h_st.wait_event(sl["kdone"])
            sl["o_h"].copy_(sl["O"], non_blocking=True)
            sl["d2h"].record(d2h_st)

    def e2e_drain():
        for sl in slots:  # the timed region ends when every step's O is on the host
            cur.wait_event(sl["d2h"])

    e2e_steps = max(3, min(args.steps, 500))
    for _ in range(args.warmup):
        e2e_step()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(cur)
    h2d_st.wait_event(ev0)
    for _ in range(e2e_steps):
        e2e_step()
    e2e_drain()
    ev1.record(cur)
    torch.cuda.synchronize()
    ms_e2e = ev0.elapsed_time(ev1)
    if dist is not None:
        ms_e2e = max_over_ranks(dist, ms_e2e, "cuda")
        dist.barrier()
    q_h, bt_h, lens_h, o_h = slots[0]["q_h"], slots[0]["bt_h"], slots[0]["lens_h"], slots[0]["o_h"]
    e2e_value = bytes_total / (ms_e2e / e2e_steps * 1e-3) / 1e9
    h2d = q_h.numel() * 4 + bt_h.numel() * 4 + lens_h.numel() * 4
    d2h = o_h.numel() * 4

    line = {
        "metric": "decode-attn HBM GB/s (GQA paged decode, BASELINE config 3, fp32 KV)",
        "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_step, 5), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (seeded N(0,1) Q/K/V, ragged lengths U[512,8192], random block table)",
        "config": {"workload": "gqa_decode_attn_config3", "batch": B, "h_q": H_Q, "h_kv": H_KV, "head_dim": D,
                   "block_size": BS, "ctx_lens": "U[512,8192] seed 42", "sum_ctx": int(lens.sum()),
                   "kv_dtype": "fp32", "parallelism": f"kv-heads x{world}",
                   "timing": "one CUDA-graph replay (one decode_attn launch) per step", "l2": "inputs larger than L2 "
                   f"({bytes_rank / 1e9:.3f} GB per rank per step vs 126 MB L2)", "algorithmic_bytes": bytes_total},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(achieved / hbm_peak, 4), "peak_kind": peak_kind,
                     "traffic": ncu_traffic("decode_attn_kernel", bytes_rank)},
        "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "mode": "b2.decode_attn with every step's Q, block table and lengths copied in from pinned host "
                        "memory and its O copied out; two buffer sets and copy streams overlap step i+1's "
                        "copies with step i's kernel"},
        "gpu_launches": args.steps,
        "clocks": clocks,
    }
    if world > 1 and os.environ.get("B2_BENCH_SKIP_TP") != "1":
        del kc, vc
        torch.cuda.empty_cache()
        r5 = tp_config5(torch, b2, np, dist, rank, world, hbm_peak)
        line["secondary"] = {"tp_decode_config5": r5}
    if world == 1 and rank == 0:
        line["secondary"] = secondary(torch, b2, np, args, kc, vc, q, btd, lensd, lens, bt, P, hbm_peak, bf16_peak)
        line["cpu_baseline"] = cpu_baseline(torch, q, kc, vc, bt, lens)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


def ncu_traffic(kernel, alg_bytes_per_launch):
    """DRAM bytes per launch of `kernel` from the committed ncu summary
    (profiles/ncu_traffic.json: read+write bytes and the algorithmic bytes of the captured
    launch), scaled to this launch by algorithmic bytes; None when not captured."""
    p = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    try:
        with open(p) as f:
            j = json.load(f)[kernel]
        return int(j["dram_bytes"] / j["alg_bytes"] * alg_bytes_per_launch)
    except Exception:
        return None


def secondary(torch, b2, np, args, kc, vc, q, btd, lensd, lens, bt, P, hbm_peak, bf16_peak):
    out = {}
    max_ctx = int(lens.max())
    n = max(3, min(args.steps, 200))
    # bf16 KV cache, same batch and values rounded to bf16
    kb, vb = kc.to(torch.bfloat16), vc.to(torch.bfloat16)
    O = torch.empty_like(q)
    ws = b2.make_decode_workspace(B, H_Q, H_KV, D, max_ctx, BS)
    ms = time_steps(torch, lambda: b2.decode_attn(q, kb, vb, btd, lensd, max_ctx, O=O, workspace=ws), n, 3)
    by = attn_alg_bytes(lens, H_KV, H_Q, D, 2, bt.shape[1])
    gbs = by / (ms / n * 1e-3) / 1e9
    out["gqa_config3_bf16_kv"] = {"gbs": round(gbs, 1), "frac_of_hbm_peak": round(gbs / hbm_peak, 4),
                                  "us_per_call": round(ms / n * 1e3, 2), "algorithmic_bytes": by}
    del kb, vb
    # the reference-named drop-in run_decode_attn (legacy default stream, the reference's
    # caller-sized workspace [B, H_q, 16, d+2] floats) on the same fp32 batch
    ws_ref = torch.empty(B * H_Q * 16 * (D + 2), dtype=torch.float32, device="cuda")
    O_ref = torch.empty_like(q)
    nbps = bt.shape[1]

    def dropin():
        b2.run_decode_attn(B, H_Q, H_KV, D, q, kc, vc, btd, lensd, max_ctx, BS, nbps, O_ref, ws_ref)

    with torch.cuda.stream(torch.cuda.default_stream()):
        ms = time_steps(torch, dropin, n, 3)
    by = attn_alg_bytes(lens, H_KV, H_Q, D, 4, nbps)
    gbs = by / (ms / n * 1e-3) / 1e9
    out["dropin_run_decode_attn_config3"] = {
        "gbs": round(gbs, 1), "frac_of_hbm_peak": round(gbs / hbm_peak, 4), "us_per_call": round(ms / n * 1e3, 2),
        "api": "run_decode_attn (reference signature, legacy default stream, reference-sized workspace)"}
    del ws_ref, O_ref
    # config 1: MHA B1 H12 d64 ctx1024, 64-block random permutation; 6.3 MB fits in L2, so
    # 40 independent copies (250 MB) are rotated
    rng = np.random.default_rng(SEED)
    copies = 40
    bt1 = torch.from_numpy(rng.permutation(64).astype(np.int32).reshape(1, 64)).cuda()
    l1 = torch.tensor([1024], dtype=torch.int32, device="cuda")
    sets = [(torch.randn(64, 16, 12, 64, device="cuda"), torch.randn(64, 16, 12, 64, device="cuda"),
             torch.randn(1, 12, 64, device="cuda")) for _ in range(copies)]
    O1 = torch.empty(1, 12, 64, device="cuda")
    ws1 = b2.make_decode_workspace(1, 12, 12, 64, 1024, 16)
    it = [0]

    def step1():
        k, v, qq = sets[it[0] % copies]
        it[0] += 1
        b2.decode_attn(qq, k, v, bt1, l1, 1024, O=O1, workspace=ws1)

    # one CUDA graph holds a full rotation of calls, so host launch cost stays out of the timing
    for _ in range(3):
        step1()
    torch.cuda.synchronize()
    graph1 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph1):
        for _ in range(copies):
            step1()
    reps1 = max(3, min(args.steps, 200) // 4)
    ms = time_steps(torch, graph1.replay, reps1, 3)
    n1 = reps1 * copies
    by1 = attn_alg_bytes(np.array([1024]), 12, 12, 64, 4, 64)
    out["mha_config1"] = {"gbs": round(by1 / (ms / n1 * 1e-3) / 1e9, 1), "us_per_call": round(ms / n1 * 1e3, 2),
                          "algorithmic_bytes": by1, "l2": "40 rotated copies (250 MB)",
                          "timing": "CUDA graph replays of 40 calls"}
    del sets
    out["gpt2_small_config4"] = gpt2_config4(torch, b2, np, hbm_peak, cpu_step=True)
    peak_int8 = 2.0 * bf16_peak  # dense int8 rate is twice the bf16 rate on the same tensor cores
    for (M, N, K) in [(2048, 2048, 2048), (64, 3072, 768), (8192, 8192, 8192)]:
        out[f"int8_gemm_{M}x{N}x{K}"] = gemm_secondary(torch, b2, M, N, K, args.steps, peak_int8, hbm_peak)
    out["int8_peak_tops"] = peak_int8
    out["cpu_baselines"] = cpu_secondary(np)
    return out


def host_cpu():
    model = "unknown"
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return {"model": model, "nproc": os.cpu_count()}


def cpu_secondary(np):
    """CPU baselines of the other hot-path pieces (the oracle's scalar restatements; reported,
    not targets): the int32 GEMM loop on the config-2 shapes, and one GPT-2 Small decode step
    at batch 1 (config 4's model, the reference engine's B = 1 loop)."""
    import tempfile

    from oracle import oracle

    out = {"host": host_cpu()}
    rng = np.random.default_rng(SEED)
    for (M, N, K, rows, reps) in ((64, 3072, 768, 64, 10), (2048, 2048, 2048, 256, 1)):
        A = rng.integers(-127, 128, (rows, K), dtype=np.int8).view(np.int32)
        Bt = rng.integers(-127, 128, (N, K), dtype=np.int8).view(np.int32)
        oracle.int8_gemm_s32(A[:1], Bt, nthreads=1)
        t0 = time.perf_counter()
        for _ in range(reps):
            oracle.int8_gemm_s32(A, Bt, nthreads=1)
        sec = (time.perf_counter() - t0) / reps
        gops = 2.0 * rows * N * K / sec / 1e9
        out[f"int8_gemm_{M}x{N}x{K}_scalar"] = {
            "gops": round(gops, 2), "cores": 1, "kind": "port",
            "sample": f"{rows} of the {M} rows of A against all of B^T (int32 accumulators, scalar loop)",
            "est_ms_full": round(2.0 * M * N * K / (gops * 1e9) * 1e3, 1)}
    return out


GPT2_SMALL = dict(n_layers=12, n_heads=12, d_model=768, d_ff=3072, vocab_size=50257, max_seq_len=1024, d_head=64)


def gpt2_step_bytes(cfg, B, ctx_mean):
    """Algorithmic HBM bytes of one batched decode step: int8 weights + scales + biases, the
    fp32 tied embedding (vocab projection), LayerNorm vectors, and the live fp32 K/V."""
    d, ff, L, V = cfg["d_model"], cfg["d_ff"], cfg["n_layers"], cfg["vocab_size"]
    lin = L * (3 * d * d + d * d + ff * d + d * ff)
    vec = L * (8 * (3 * d + d + ff + d) + 4 * 4 * d)
    kv = B * ctx_mean * L * 2 * d * 4
    return lin + vec + V * d * 4 + kv


def gpt2_cpu_step(eng, np, cfg, steps=4):
    """The oracle's restatement of the reference engine's decode step (GPT2Oracle, 1 thread)
    on this model at batch 1, the reference engine's own batch: seconds per token over
    `steps` steps at positions 0.. (short contexts, so the weights dominate)."""
    import shutil
    import tempfile

    from oracle import oracle

    d = tempfile.mkdtemp(prefix="b2gpt2_")
    try:
        eng.export(d)
        orc = oracle.GPT2Oracle(d)
        orc.reset(1)
        orc.step(np.array([11]), np.array([0]), nthreads=1)
        t0 = time.perf_counter()
        for p in range(1, steps + 1):
            orc.step(np.array([100 + p]), np.array([p]), nthreads=1)
        sec = (time.perf_counter() - t0) / steps
    finally:
        shutil.rmtree(d, ignore_errors=True)
    return {"tok_s": round(1.0 / sec, 2), "ms_per_token": round(sec * 1e3, 1), "cores": 1, "kind": "port",
            "sample": f"GPT2Oracle (C restatement of the reference's decode step), batch 1, {steps} steps at "
                      f"positions 1-{steps}"}


def gpt2_config4(torch, b2, np, hbm_peak, steps_new=128, prompt_len=128, B=64, cpu_step=False):
    """GPT-2 Small INT8, batch 64, 128-token prompts fed through the decode
    path, then 128 greedy steps (CUDA-graph replays); tok/s of the generation steps."""
    cfg = GPT2_SMALL
    eng = b2.Engine.random(cfg, max_batch=B, seed=SEED)
    rng = np.random.default_rng(SEED)
    prompts = [list(map(int, rng.integers(0, cfg["vocab_size"], prompt_len))) for _ in range(B)]
    eng.start(prompts, steps_new, seed=block_seed())
    st = torch.cuda.current_stream()
    e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(2))
    # warm-up: one untimed generation (allocates the prefill buffers, captures the step graph,
    # brings the clocks up), then the same prompts from scratch
    eng.prefill(stream=st)
    eng.run_steps(steps_new, stream=st)
    torch.cuda.synchronize()
    eng.start(prompts, steps_new, seed=block_seed())
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    eng.prefill(stream=st)                         # positions 0..126 of every prompt in one pass
    torch.cuda.synchronize()
    pre_ms = (time.perf_counter() - t0) * 1e3      # synchronous call: host clock, end to end
    e1.record(st)
    eng.run_steps(steps_new, stream=st)           # positions 127..254: 128 generated tokens
    e2.record(st)
    torch.cuda.synchronize()
    assert b2.device_error() == 0
    gen_ms = e1.elapsed_time(e2)
    ctx_mean = prompt_len + (steps_new - 1) / 2.0 + 0.5
    by = gpt2_step_bytes(cfg, B, ctx_mean)
    step_s = gen_ms / steps_new * 1e-3
    toks = eng.tokens()
    breakdown = parse_profile(eng.profile_step())
    cpu = gpt2_cpu_step(eng, np, cfg) if cpu_step else None
    eng.close()
    return {"tok_s": round(B * steps_new / (gen_ms * 1e-3), 1), "ms_per_step": round(gen_ms / steps_new, 4),
            "prefill_tok_s": round(B * (prompt_len - 1) / (pre_ms * 1e-3), 1),
            "prefill": "b2_engine_prefill: the 127 x 64 prompt tokens in one batched pass (host clock)",
            "step_bytes": int(by), "gbs": round(by / step_s / 1e9, 1),
            "frac_of_hbm_bound": round(by / step_s / 1e9 / hbm_peak, 4),
            "hbm_bound_tok_s": round(B / (by / (hbm_peak * 1e9)), 1),
            "generated_tokens_valid": bool((toks[:, prompt_len:prompt_len + steps_new] >= 0).all()),
            "timing": "CUDA graph replays of one decode step", "kv_block_seed": block_seed(),
            "step_breakdown": breakdown, "cpu_baseline_b1": cpu}


WIDE = dict(n_layers=32, n_heads=32, d_model=4096, d_ff=16384, vocab_size=50257, max_seq_len=4096 + 64 + 1,
            d_head=128)


def block_seed():
    """KV block placement of the engine legs: 0 = in pool order, as the reference engine
    allocates (src/gpt2_engine.cu:420-429); B2_BENCH_BLOCK_SEED=n scatters the blocks."""
    return int(os.environ.get("B2_BENCH_BLOCK_SEED", "0"))


def parse_profile(text):
    """Engine.profile_step() report -> {"step_us": T, "us": {kernel class: total µs}} (eager
    step with an event before every launch: a breakdown, not a timing of record)."""
    lines = text.strip().splitlines()
    out = {"step_us": float(lines[0].split()[1]), "us": {}}
    for ln in lines[1:]:
        f = ln.split()
        out["us"][f[0]] = float(f[2])
    return out


def tp_config5(torch, b2, np, dist, rank, world, hbm_peak, steps=64, ctx=4096, B=128):
    """the widened GPT-2 (32 L, d 4096, 32 x 128 heads, d_ff 16384) decoding
    a batch of 128 at context 4096 for 64 greedy steps, bf16 KV, tensor-parallel over the
    ranks. The 4096-token context is a seeded synthetic KV fill (no prefill); timed with CUDA
    events over CUDA-graph replays, max over ranks."""
    cfg = WIDE
    nid = torch.zeros(128, dtype=torch.uint8, device="cuda")
    if rank == 0:
        nid.copy_(torch.frombuffer(bytearray(b2.nccl_unique_id()), dtype=torch.uint8))
    dist.broadcast(nid, 0)
    eng = b2.Engine.random_tp(cfg, B, bytes(nid.cpu().numpy().tobytes()), rank, world, kv_dtype=b2.B2_KV_BF16,
                              seed=SEED)
    rng = np.random.default_rng(SEED)
    eng.start([[int(t)] for t in rng.integers(0, cfg["vocab_size"], B)], steps + 1, seed=block_seed())
    eng.fill_kv_random(ctx, seed=SEED)
    st = torch.cuda.current_stream()
    eng.run_steps(2, stream=st)  # warm-up (captures the graph); positions ctx, ctx+1
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    eng.run_steps(steps, stream=st)
    e1.record(st)
    torch.cuda.synchronize()
    ms = max_over_ranks(dist, e0.elapsed_time(e1), "cuda")
    assert b2.device_error() == 0
    breakdown = parse_profile(eng.profile_step())  # every rank takes part (collectives inside)
    d, L = cfg["d_model"], cfg["n_layers"]
    ctx_mean = ctx + 2 + (steps - 1) / 2.0 + 1
    lin = L * (3 * d * d + d * d + 2 * cfg["d_ff"] * d)
    kv = B * ctx_mean * L * 2 * d * 2
    by_total = lin + 2 * cfg["vocab_size"] * d * 2 + kv  # int8 weights + bf16 vocab halves + bf16 K/V
    step_s = ms / steps * 1e-3
    eng.close()
    return {"tok_s": round(B * steps / (ms * 1e-3), 1), "ms_per_step": round(ms / steps, 3),
            "step_bytes_all_ranks": int(by_total), "gbs_all_ranks": round(by_total / step_s / 1e9, 1),
            "frac_of_hbm_bound": round(by_total / step_s / 1e9 / (hbm_peak * world), 4),
            "hbm_bound_tok_s": round(B / (by_total / (hbm_peak * 1e9 * world)), 1),
            "parallelism": f"tensor-parallel x{world} (row-parallel out-proj and FC2: "
                           + ("NCCL all-reduces" if os.environ.get("B2_TP_COLLECTIVES") == "nccl"
                              else "peer-memory scale exchange and int32 reduce kernels over NVLink") + ")",
            "context": "seeded synthetic KV fill of 4096 tokens, then 2 warm-up + 64 timed steps",
            "kv_block_seed": block_seed(),
            "step_breakdown_rank0": breakdown}


def cpu_baseline(torch, q, kc, vc, bt, lens):
    """The oracle (C restatement of the reference's CPU attention), 1 thread, on the first
    4 sequences of the workload, repeated for ~10 s."""
    from oracle import oracle

    seqs = [0, 1, 2, 3]
    k, v, sbt, sl = cpu_sample(torch, kc, vc, bt, lens, seqs)
    qs = q[seqs].cpu().numpy()
    sec = time_cpu_attention(oracle, qs, k, v, sbt, sl, 1, 10.0)
    by = attn_alg_bytes(sl, H_KV, H_Q, D, 4, bt.shape[1])
    return {"value": round(by / sec / 1e9, 3), "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": f"sequences 0-3 of the workload (ctx {list(map(int, sl))}), all 32 heads, fp32 KV, "
                      f"{sec * 1e3:.0f} ms per pass"}


def reference_line(args, value, ms_step, kind, cores, sample):
    return {
        "impl": "reference", "metric": "decode-attn HBM GB/s (GQA paged decode, BASELINE config 3, fp32 KV)",
        "value": round(value, 3), "unit": "GB/s", "n_gpus": int(os.environ.get("WORLD_SIZE", "1")),
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1), ragged lengths U[512,8192])",
        "config": {"workload": "gqa_decode_attn_config3", "batch": B, "h_q": H_Q, "h_kv": H_KV, "head_dim": D,
                   "block_size": BS, "kv_dtype": "fp32", "parallelism": "host threads"},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": cores, "kind": kind, "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def run_reference_harness(args):
    """The reference's own CPU attention, gqa_cpu_reference (tests/test_paged_attention.cu:
    138-179, compiled unchanged from its sources into oracle/_ref/libref.so), in its own
    form: N query rows of one sequence against its N keys, all 32 query / 8 KV heads, d 128,
    fp32. Each row is the work of one decode call at context N (every K/V byte of the
    sequence read once, the same arithmetic per key), so a call counts N decode calls'
    algorithmic bytes. Each step runs one call per host thread in parallel (the harness is
    single-threaded; ctypes releases the GIL), N sized so the run stays within ~2 minutes."""
    import numpy as np
    from concurrent.futures import ThreadPoolExecutor

    from oracle import oracle

    threads = max(1, min(os.cpu_count() or 1, 64))
    rng = np.random.default_rng(SEED)

    def sample(n):
        return (rng.standard_normal((1, H_Q, n, D)).astype(np.float32),
                rng.standard_normal((1, H_KV, n, D)).astype(np.float32),
                rng.standard_normal((1, H_KV, n, D)).astype(np.float32))

    n0 = 128
    probe = sample(n0)
    oracle.ref_gqa_cpu(*probe)
    t0 = time.perf_counter()
    oracle.ref_gqa_cpu(*probe)
    t_probe = time.perf_counter() - t0
    # a call costs ~N^2: aim at ~100 s for the whole run (B2_REF_BUDGET_S overrides)
    target = float(os.environ.get("B2_REF_BUDGET_S", "100")) / max(1, args.steps + args.warmup)
    n = int(n0 * (target / max(t_probe, 1e-6)) ** 0.5) // 16 * 16
    n = max(32, min(n, 1024))
    sets = [sample(n) for _ in range(threads)]
    pool = ThreadPoolExecutor(max_workers=threads)

    def step():
        list(pool.map(lambda qkv: oracle.ref_gqa_cpu(*qkv), sets))

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    sec = time.perf_counter() - t0
    pool.shutdown()
    row_bytes = attn_alg_bytes(np.array([n]), H_KV, H_Q, D, 4, (n + BS - 1) // BS)
    by = threads * n * row_bytes  # per step
    v = by * args.steps / sec / 1e9
    smp = (f"reference gqa_cpu_reference (oracle/_ref, its own compiled code): per step {threads} calls in "
           f"parallel, each {n} query rows x {n} keys, H 32/8, d 128, fp32; a row = one decode call at context {n}")
    print(json.dumps(reference_line(args, v, sec / args.steps * 1e3, "reference", threads, smp)), flush=True)


def run_reference(args):
    """The reference's CPU implementation of the path on all host threads, timed on a
    bounded sample of the headline workload per step, rank 0 only: its own compiled CPU
    attention harness when oracle/_ref was built (run_reference_harness), else the oracle's
    restatement of that harness (tests/test_paged_attention.cu:138-179) over the workload's
    paged sequences."""
    import numpy as np

    if int(os.environ.get("RANK", "0")) != 0:
        return
    from oracle import oracle

    if oracle.ref_available() and os.environ.get("B2_REF_ARM") != "port":
        return run_reference_harness(args)
    lens, bt, P = workload_meta()
    threads = oracle.max_threads()
    rng = np.random.default_rng(SEED)
    # size the per-step sample so the whole run stays within ~2 minutes
    probe = [0]
    nb0 = (int(lens[0]) + BS - 1) // BS
    kc = rng.standard_normal((nb0, BS, H_KV, D)).astype(np.float32)
    vc = rng.standard_normal((nb0, BS, H_KV, D)).astype(np.float32)
    q = rng.standard_normal((1, H_Q, D)).astype(np.float32)
    sbt = np.arange(nb0, dtype=np.int32).reshape(1, nb0)
    t1 = time_cpu_attention(oracle, q, kc, vc, sbt, lens[probe], threads, 0.2)
    per_seq = t1 * float(lens.mean()) / float(lens[0])
    nseq = int(max(1, min(B, 120.0 / max(1, args.steps + args.warmup) / per_seq)))
    seqs = list(range(nseq))
    sl = lens[seqs]
    nbs = [(int(l) + BS - 1) // BS for l in sl]
    Ptot = sum(nbs)
    kc = rng.standard_normal((Ptot, BS, H_KV, D)).astype(np.float32)
    vc = rng.standard_normal((Ptot, BS, H_KV, D)).astype(np.float32)
    q = rng.standard_normal((nseq, H_Q, D)).astype(np.float32)
    sbt = np.zeros((nseq, max(nbs)), np.int32)
    off = 0
    for i, nb in enumerate(nbs):
        sbt[i, :nb] = rng.permutation(np.arange(off, off + nb))
        off += nb
    for _ in range(args.warmup):
        oracle.decode_attn(q, kc, vc, sbt, sl, nthreads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.decode_attn(q, kc, vc, sbt, sl, nthreads=threads)
    sec = time.perf_counter() - t0
    by = attn_alg_bytes(sl, H_KV, H_Q, D, 4, sbt.shape[1])
    v = by * args.steps / sec / 1e9
    sample = f"sequences 0-{nseq - 1} of the workload per step (sum ctx {int(sl.sum())}), all heads, fp32 KV"
    print(json.dumps(reference_line(args, v, sec / args.steps * 1e3, "port", threads, sample)), flush=True)


def run_only(args):
    """One workload, W + K launches, no secondary legs (a small, fixed command for ncu)."""
    import torch

    b2 = importlib.import_module("cuda-llm-inference-engine_b200")
    b2.load_library()
    dev = torch.device("cuda", 0)
    if args.only == "gpt2":
        import numpy as np

        r = gpt2_config4(torch, b2, np, measured_peaks()[0], steps_new=max(1, args.steps), prompt_len=128)
        print(f"gpt2: {json.dumps(r)} (not a bench value)", flush=True)
        return
    if args.only == "attn_wide":
        # config 5's per-layer attention shape on one GPU: MHA 32 x 128, bf16 KV, context 4096
        # (batch 32 of the 128, so the case stays near 2 GB for profiling)
        import numpy as np

        # B2_WIDE="B,H,ctx[,max_ctx]" overrides the shape (max_ctx: the bound passed to the launch)
        wide = [int(v) for v in os.environ.get("B2_WIDE", "32,32,4096").split(",")]
        Bw, Hw, ctxw = wide[:3]
        mcw = wide[3] if len(wide) > 3 else ctxw
        nb = (mcw + BS - 1) // BS
        P = Bw * nb
        g = torch.Generator(device=dev).manual_seed(SEED)
        kc = torch.randn(P, BS, Hw, D, generator=g, device=dev).to(torch.bfloat16)
        vc = torch.randn(P, BS, Hw, D, generator=g, device=dev).to(torch.bfloat16)
        q = torch.randn(Bw, Hw, D, device=dev)
        O = torch.empty_like(q)
        btd = torch.randperm(P, generator=g, device=dev).to(torch.int32).view(Bw, nb)
        lensd = torch.full((Bw,), ctxw, dtype=torch.int32, device=dev)
        ws = b2.make_decode_workspace(Bw, Hw, Hw, D, mcw, BS, device=dev)
        fn = lambda: b2.decode_attn(q, kc, vc, btd, lensd, mcw, O=O, workspace=ws)  # noqa: E731
        by = attn_alg_bytes(np.full(Bw, ctxw), Hw, Hw, D, 2, nb)
    elif args.only == "attn_c1":
        # MHA B1 H12 d64 ctx 1024, 64-block random permutation, 40 rotated
        # copies (250 MB) in one graph, as the default run's secondary line
        import numpy as np

        rng = np.random.default_rng(SEED)
        copies = 40
        bt1 = torch.from_numpy(rng.permutation(64).astype(np.int32).reshape(1, 64)).to(dev)
        l1 = torch.tensor([1024], dtype=torch.int32, device=dev)
        sets = [(torch.randn(64, 16, 12, 64, device=dev), torch.randn(64, 16, 12, 64, device=dev),
                 torch.randn(1, 12, 64, device=dev)) for _ in range(copies)]
        O1 = torch.empty(1, 12, 64, device=dev)
        ws1 = b2.make_decode_workspace(1, 12, 12, 64, 1024, 16)
        it = [0]

        def fn1():
            k, v, qq = sets[it[0] % copies]
            it[0] += 1
            b2.decode_attn(qq, k, v, bt1, l1, 1024, O=O1, workspace=ws1)

        graph = graph_of(torch, lambda: [fn1() for _ in range(copies)])
        steps = max(1, args.steps // copies)
        ms = time_steps(torch, graph.replay, steps, args.warmup) / copies
        print(f"attn_c1: {ms / steps * 1e3:.2f} us/launch (40 copies rotated; not a bench value)", flush=True)
        return
    elif args.only == "attn_gpt2":
        # config 4's per-layer attention: B64, 12 heads x 64, fp32 KV, every sequence at the
        # same context (B2_GPT2_CTX, default 192: the middle of the 128 decode steps); twelve
        # caches (one per layer) are cycled so that, as in the decode step, the KV is not
        # L2-resident between launches
        import numpy as np

        ctx = int(os.environ.get("B2_GPT2_CTX", "192"))
        Bg, Hg, Dg, NL = 64, 12, 64, 12
        nb = (ctx + BS - 1) // BS
        P = Bg * nb
        g = torch.Generator(device=dev).manual_seed(SEED)
        caches = [(torch.randn(P, BS, Hg, Dg, generator=g, device=dev),
                   torch.randn(P, BS, Hg, Dg, generator=g, device=dev)) for _ in range(NL)]
        q = torch.randn(Bg, Hg, Dg, device=dev)
        O = torch.empty_like(q)
        btd = torch.randperm(P, generator=g, device=dev).to(torch.int32).view(Bg, nb)
        lensd = torch.full((Bg,), ctx, dtype=torch.int32, device=dev)
        ws = b2.make_decode_workspace(Bg, Hg, Hg, Dg, 1024, BS, device=dev)
        it = [0]

        def fn():
            kc, vc = caches[it[0] % NL]
            it[0] += 1
            b2.decode_attn(q, kc, vc, btd, lensd, 1024, O=O, workspace=ws)

        by = attn_alg_bytes(np.full(Bg, ctx), Hg, Hg, Dg, 4, nb)
        graph = graph_of(torch, lambda: [fn() for _ in range(NL)])
        ms = time_steps(torch, graph.replay, max(1, args.steps // NL), args.warmup) / NL
        steps = max(1, args.steps // NL)
        print(f"attn_gpt2 ctx {ctx}: {ms / steps * 1e3:.2f} us/launch, {by / (ms / steps * 1e-3) / 1e9:.1f} GB/s "
              "(12 caches cycled; not a bench value)", flush=True)
        return
    elif args.only.startswith("attn"):
        dt = torch.bfloat16 if args.only == "attn_bf16" else torch.float32
        # B2_ATTN_SHARD=n: the KV-head shard one rank of n holds (the per-rank launch of --gpus n)
        nshard = int(os.environ.get("B2_ATTN_SHARD", "1"))
        hkv, hq = H_KV // nshard, H_Q // nshard
        lens, bt, P = workload_meta()
        kc, vc = make_kv_shard(torch, P, 0, hkv, dt, dev)
        q = torch.randn(B, hq, D, device=dev)
        O = torch.empty_like(q)
        btd, lensd = torch.from_numpy(bt).to(dev), torch.from_numpy(lens).to(dev)
        ws = b2.make_decode_workspace(B, hq, hkv, D, int(lens.max()), BS, device=dev)
        fn = lambda: b2.decode_attn(q, kc, vc, btd, lensd, int(lens.max()), O=O, workspace=ws)  # noqa: E731
        by = attn_alg_bytes(lens, hkv, hq, D, 2 if dt == torch.bfloat16 else 4, bt.shape[1])
    elif args.only == "gemm_c5":
        # config-5 decode GEMM shapes per tensor-parallel shard (batch 128, d 4096, d_ff 16384):
        # 12 weight copies rotated in one graph so the weights stream from HBM, not L2
        copies = 12
        for (M, N, K, tag) in [(128, 3072, 4096, "qkv tp4"), (128, 4096, 4096, "fc1/fc2 tp4"),
                               (128, 1536, 4096, "qkv tp8"), (128, 2048, 4096, "fc1/fc2 tp8"),
                               (128, 4096, 1024, "out tp4"), (128, 6144, 4096, "qkv tp2"),
                               (128, 8192, 4096, "fc1/fc2 tp2")]:
            A = torch.randint(-127, 128, (M, K), dtype=torch.int8, device=dev).view(torch.int32)
            Bts = [torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev).view(torch.int32)
                   for _ in range(copies)]
            sA, sB = torch.rand(M, device=dev), torch.rand(N, device=dev)
            C = torch.empty(M, N, device=dev)
            ws = b2.make_gemm_workspace(M, N, K, device=dev)
            for wname, w in (("no workspace", None), ("workspace", ws)):
                g = graph_of(torch, lambda: [b2.int8_gemm(A, Bt, sA, sB, C=C, workspace=w) for Bt in Bts])
                steps = max(2, args.steps // copies)
                ms = time_steps(torch, g.replay, steps, args.warmup) / (steps * copies)
                assert b2.device_error() == 0
                by = N * K + M * K + 4 * (M * N + M + N)
                print(f"gemm_c5 {M}x{N}x{K} ({tag}, {wname}): {ms * 1e3:.2f} us/launch, "
                      f"{by / (ms * 1e-3) / 1e9:.0f} GB/s (not a bench value)", flush=True)
            del Bts
        return
    else:
        M, N, K = {"gemm2048": (2048,) * 3, "gemm8192": (8192,) * 3, "gemm_rect": (64, 3072, 768)}[args.only]
        A = torch.randint(-127, 128, (M, K), dtype=torch.int8, device=dev).view(torch.int32)
        Bt = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev).view(torch.int32)
        sA, sB = torch.rand(M, device=dev), torch.rand(N, device=dev)
        C = torch.empty(M, N, device=dev)
        fn = lambda: b2.int8_gemm(A, Bt, sA, sB, C=C)  # noqa: E731
        by = 2 * M * N * K
    ms = time_steps(torch, graph_of(torch, fn).replay, args.steps, args.warmup)
    assert b2.device_error() == 0
    print(f"{args.only}: {ms / args.steps * 1e3:.2f} us/launch, {by / (ms / args.steps * 1e-3) / 1e9:.1f} "
          f"{'GB/s' if args.only.startswith('attn') else 'GOP/s'} (not a bench value)", flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b2", choices=["b2", "reference"])
    ap.add_argument("--only", default=None,
                    choices=["attn", "attn_bf16", "attn_wide", "attn_gpt2", "attn_c1", "gemm2048", "gemm8192", "gemm_rect", "gemm_c5", "gpt2"],
                    help="run one workload for a few steps with no JSON line (for profiling)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.only:
        run_only(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()

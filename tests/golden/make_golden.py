"""Generates the golden fixtures in tests/golden/ from the reference itself.

    python tests/golden/make_golden.py   (needs the reference mounted at $REF, default /root/reference,
                                          and oracle/_ref/libref.so from oracle/build_ref.sh)

quantize_golden.npz  inputs and outputs of the reference's numpy quantiser
                     `quantize_per_row` (python/export_gpt2.py:10-40), imported from the
                     reference tree: random rows, an all-zero row, exact half-way ties,
                     a single huge outlier, denormal-scale rows.
attention_golden.npz inputs and outputs of the reference harness's CPU attention
                     `gqa_cpu_reference` (tests/test_paged_attention.cu:138-179), compiled
                     from the reference sources into oracle/_ref/libref.so. Non-causal; the
                     decode output of a sequence of length N is row N-1, whose query is the
                     last query row.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
REF = os.environ.get("REF", "/root/reference")


def quantize_cases():
    rng = np.random.default_rng(20260401)
    cases = {}
    cases["normal_8x64"] = rng.standard_normal((8, 64)).astype(np.float32)
    cases["normal_64x768"] = rng.standard_normal((64, 768)).astype(np.float32)
    z = rng.standard_normal((4, 32)).astype(np.float32)
    z[1] = 0.0
    cases["zero_row"] = z
    # amax = 127 -> scale = 1, inv = 1: x*inv hits .5 exactly; round-half-even decides
    t = np.array([[127.0, 0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 126.5, -126.5, 3.5, -3.5, 0.0]], np.float32)
    cases["ties"] = np.concatenate([t, -t], axis=0)
    o = rng.standard_normal((3, 16)).astype(np.float32) * 1e-3
    o[:, 5] = 1e4
    cases["outlier"] = o
    cases["tiny"] = (rng.standard_normal((2, 8)) * 1e-38).astype(np.float32)
    cases["uniform_ref_style"] = rng.uniform(-1, 1, (16, 256)).astype(np.float32)
    return cases


def make_quantize():
    sys.path.insert(0, os.path.join(REF, "python"))
    from export_gpt2 import quantize_per_row  # the reference's own quantiser

    out = {}
    for name, x in quantize_cases().items():
        packed, scales = quantize_per_row(x)
        out[f"{name}__x"] = x
        out[f"{name}__packed"] = np.asarray(packed, np.int32)
        out[f"{name}__scales"] = np.asarray(scales, np.float32)
    np.savez_compressed(os.path.join(HERE, "quantize_golden.npz"), **out)
    print("quantize_golden.npz:", len(out) // 3, "cases")


def make_attention():
    sys.path.insert(0, ROOT)
    from oracle import oracle

    rng = np.random.default_rng(20260402)
    out = {}
    # (B, H_q, H_kv, N, d): MHA and GQA 2/4/8, d 64 and 128, lengths off the block grid
    for (B, H_q, H_kv, N, d) in [(1, 4, 4, 37, 64), (2, 8, 2, 50, 64), (1, 8, 1, 17, 128),
                                 (1, 4, 2, 64, 128), (2, 2, 2, 1, 64)]:
        Q = rng.standard_normal((B, H_q, N, d)).astype(np.float32)
        K = rng.standard_normal((B, H_kv, N, d)).astype(np.float32)
        V = rng.standard_normal((B, H_kv, N, d)).astype(np.float32)
        O = oracle.ref_gqa_cpu(Q, K, V, causal=False)
        tag = f"B{B}_Hq{H_q}_Hkv{H_kv}_N{N}_d{d}"
        out[f"{tag}__q"] = Q[:, :, N - 1, :].copy()
        out[f"{tag}__K"] = K
        out[f"{tag}__V"] = V
        out[f"{tag}__O"] = O[:, :, N - 1, :].copy()
    np.savez_compressed(os.path.join(HERE, "attention_golden.npz"), **out)
    print("attention_golden.npz:", len(out) // 4, "cases")


if __name__ == "__main__":
    make_quantize()
    make_attention()

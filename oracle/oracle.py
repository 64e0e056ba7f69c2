"""ctypes front end of the oracle (TEST INFRASTRUCTURE ONLY).

Only tests/, __graft_entry__.smoke() and bench.py's CPU legs use this module, as the
checker. It wraps:
  - liboracle.so: the C restatement in oracle.c (numpy arrays in, numpy arrays out);
  - _ref/libref.so: the reference's own sources compiled by build_ref.sh — its CPU
    attention harness, and its K13/K14/K12 CUDA kernels (device pointers in).
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libref.so")

_fp = ctypes.POINTER(ctypes.c_float)
_ip = ctypes.POINTER(ctypes.c_int32)
_vp = ctypes.c_void_p
_i = ctypes.c_int

_lib = None
_ref = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO):
            raise RuntimeError(f"{ORACLE_SO} missing: run oracle/build_ref.sh")
        L = ctypes.CDLL(ORACLE_SO)
        L.oracle_decode_attn.argtypes = [_i, _i, _i, _i, _vp, _vp, _vp, _i, _vp, _vp, _i, _i, _vp, _i]
        L.oracle_quantize.argtypes = [_i, _i, _vp, _vp, _vp]
        L.oracle_int8_gemm_s32.argtypes = [_i, _i, _i, _vp, _vp, _vp, _i]
        L.oracle_int8_gemm.argtypes = [_i, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i]
        L.oracle_epilogue.argtypes = [_i, _i, _vp, _vp, _vp, _vp, _vp, _vp, _i]
        L.oracle_max_threads.restype = _i
        _lib = L
    return _lib


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref():
    global _ref
    if _ref is None:
        if not ref_available():
            raise RuntimeError(f"{REF_SO} missing: run oracle/build_ref.sh where the reference is mounted")
        R = ctypes.CDLL(REF_SO, mode=ctypes.RTLD_LOCAL)
        R.ref_gqa_cpu_reference.argtypes = [_i, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _i]
        R.ref_run_decode_attn.argtypes = [_i, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _vp, _vp]
        R.ref_run_gqa_paged_attn.argtypes = [_i, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _vp, _i]
        R.ref_run_quantize_fp32_to_int8.argtypes = [_i, _i, _vp, _vp, _vp]
        R.ref_run_int8_gemm.argtypes = [_i, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i]
        R.ref_sync.restype = _i
        _ref = R
    return _ref


def _c(a, dtype):
    a = np.ascontiguousarray(a, dtype=dtype)
    return a, a.ctypes.data


def max_threads() -> int:
    return int(lib().oracle_max_threads())


def decode_attn(Q, k_cache, v_cache, block_table, context_lens, nthreads=1):
    """Q [B,H_q,d] f32; caches [P,bs,H_kv,d] f32 or bf16 given as uint16 (kv_dtype by dtype)."""
    Q, qp = _c(Q, np.float32)
    B, H_q, d = Q.shape[0], Q.shape[1], Q.shape[-1]
    P, bs, H_kv, _ = k_cache.shape
    if k_cache.dtype == np.uint16:
        kvd = 1
        k_cache, kp = _c(k_cache, np.uint16)
        v_cache, vp = _c(v_cache, np.uint16)
    else:
        kvd = 0
        k_cache, kp = _c(k_cache, np.float32)
        v_cache, vp = _c(v_cache, np.float32)
    bt, btp = _c(block_table, np.int32)
    cl, clp = _c(context_lens, np.int32)
    O = np.zeros((B, H_q, d), np.float32)
    lib().oracle_decode_attn(B, H_q, H_kv, d, qp, kp, vp, kvd, btp, clp, bs, bt.shape[1], O.ctypes.data, nthreads)
    return O


def quantize(x):
    x, xp = _c(x, np.float32)
    rows, cols = x.shape
    out = np.zeros((rows, cols // 4), np.int32)
    sc = np.zeros(rows, np.float32)
    lib().oracle_quantize(rows, cols, xp, out.ctypes.data, sc.ctypes.data)
    return out, sc


def int8_gemm_s32(A_packed, BT_packed, nthreads=1):
    A, ap = _c(A_packed, np.int32)
    BT, bp = _c(BT_packed, np.int32)
    M, N, K = A.shape[0], BT.shape[0], 4 * A.shape[1]
    C = np.zeros((M, N), np.int32)
    lib().oracle_int8_gemm_s32(M, N, K, ap, bp, C.ctypes.data, nthreads)
    return C


def epilogue(acc, sA, sB, bias=None, residual=None, epi=0):
    acc, accp = _c(acc, np.int32)
    M, N = acc.shape
    sA, sap = _c(sA, np.float32)
    sB, sbp = _c(sB, np.float32)
    bias_a, bip = _c(bias if bias is not None else np.zeros(N), np.float32)
    res_a, rp = _c(residual if residual is not None else np.zeros((1,)), np.float32)
    C = np.zeros((M, N), np.float32)
    lib().oracle_epilogue(M, N, accp, sap, sbp, bip, rp, C.ctypes.data, epi)
    return C


def int8_gemm(A_packed, BT_packed, sA, sB, bias=None, residual=None, epi=0, nthreads=1):
    return epilogue(int8_gemm_s32(A_packed, BT_packed, nthreads), sA, sB, bias, residual, epi)


def ref_gqa_cpu(Q, K, V, causal=False):
    """The reference harness's own CPU attention: Q [B,H_q,N,d], K/V [B,H_kv,N,d]."""
    Q, qp = _c(Q, np.float32)
    K, kp = _c(K, np.float32)
    V, vp = _c(V, np.float32)
    B, H_q, N, d = Q.shape
    H_kv = K.shape[1]
    O = np.zeros_like(Q)
    ref().ref_gqa_cpu_reference(B, H_q, H_kv, N, d, qp, kp, vp, O.ctypes.data, 1 if causal else 0)
    return O

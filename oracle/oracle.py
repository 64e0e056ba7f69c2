"""ctypes front end of the oracle (TEST INFRASTRUCTURE ONLY).

Only tests/, __graft_entry__.smoke() and bench.py's CPU legs use this module, as the
checker. It wraps:
  - liboracle.so: the C restatement in oracle.c (numpy arrays in, numpy arrays out);
  - _ref/libref.so: the reference's own sources compiled by build_ref.sh — its CPU
    attention harness, and its K12/K13/K14/K15 CUDA kernels (device pointers in);
  - _ref/libref_engine.so: the reference's GPT2Engine, greedy generation (model directory in).
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libref.so")
REF_ENGINE_SO = os.path.join(HERE, "_ref", "libref_engine.so")

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
        L.oracle_layernorm.argtypes = [_i, _i, _vp, _vp, _vp, ctypes.c_float, _vp]
        L.oracle_vocab_proj.argtypes = [_i, _i, _i, _vp, _vp, _vp, _i]
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
        R.ref_run_layernorm.argtypes = [_i, _i, _vp, _vp, _vp, _vp, ctypes.c_float]
        R.ref_sync.restype = _i
        _ref = R
    return _ref


_ref_engine = None


def ref_engine_available() -> bool:
    return os.path.exists(REF_ENGINE_SO)


def ref_engine_generate(model_dir, prompt, max_new, want_logits=True, vocab=None, token_by_token=False):
    """The reference's own GPT2Engine (src/gpt2_engine.cu, compiled unchanged into
    oracle/_ref/libref_engine.so): greedy generate(prompt, max_new) on a fresh session, the
    prompt through its FlashAttention prefill (or, token_by_token, through its decode path).
    Returns (tokens [n], logits [n, vocab] or None); logits[i] chose tokens[i]. Needs a GPU."""
    global _ref_engine
    if _ref_engine is None:
        if not ref_engine_available():
            raise RuntimeError(f"{REF_ENGINE_SO} missing: run oracle/build_ref.sh where the reference is mounted")
        R = ctypes.CDLL(REF_ENGINE_SO, mode=ctypes.RTLD_LOCAL)
        R.ref_engine_generate.argtypes = [ctypes.c_char_p, _vp, _i, _i, _vp, _vp, _i]
        R.ref_engine_generate.restype = _i
        _ref_engine = R
    p = np.ascontiguousarray(prompt, np.int32)
    toks = np.zeros(max_new + 1, np.int32)
    lg = np.zeros((max_new + 1, vocab), np.float32) if want_logits else None
    n = _ref_engine.ref_engine_generate(model_dir.encode(), p.ctypes.data, len(p), max_new, toks.ctypes.data,
                                        lg.ctypes.data if lg is not None else None, 1 if token_by_token else 0)
    if n < 0:
        raise RuntimeError("reference engine failed")
    return toks[:n], (lg[:n] if lg is not None else None)


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


def layernorm(x, gamma, beta, eps=1e-5):
    x, xp = _c(x, np.float32)
    g, gp = _c(gamma, np.float32)
    b, bp = _c(beta, np.float32)
    y = np.zeros_like(x)
    lib().oracle_layernorm(x.shape[0], x.shape[1], xp, gp, bp, eps, y.ctypes.data)
    return y


def vocab_proj(h, wte, nthreads=0):
    h, hp = _c(h, np.float32)
    w, wp = _c(wte, np.float32)
    out = np.zeros((h.shape[0], w.shape[0]), np.float32)
    lib().oracle_vocab_proj(h.shape[0], w.shape[0], h.shape[1], hp, wp, out.ctypes.data, nthreads)
    return out


class GPT2Oracle:
    """CPU restatement of the reference GPT2Engine decode step (src/gpt2_engine.cu:447-528,
    612-620) over a model directory in the reference's format, batched over sequences with
    their own positions. KV caches are kept paged with identity block tables."""

    LINEARS = [("qkv", 3), ("out", 1), ("ffn_up", None), ("ffn_down", 1)]

    def __init__(self, model_dir):
        import json
        import os

        txt = open(os.path.join(model_dir, "config.json")).read()
        c = json.loads(txt)
        self.cfg = c
        L, d, ff, V, S = c["n_layers"], c["d_model"], c["d_ff"], c["vocab_size"], c["max_seq_len"]
        f = lambda name, n: np.fromfile(os.path.join(model_dir, name), np.float32, n)  # noqa: E731
        i = lambda name, n: np.fromfile(os.path.join(model_dir, name), np.int32, n)  # noqa: E731
        self.wte = f("wte.bin", V * d).reshape(V, d)
        self.wpe = f("wpe.bin", S * d).reshape(S, d)
        self.lnf = (f("ln_f_gamma.bin", d), f("ln_f_beta.bin", d))
        self.layers = []
        shapes = {"qkv": (3 * d, d), "out": (d, d), "ffn_up": (ff, d), "ffn_down": (d, ff)}
        for l in range(L):
            ld = "layer_%02d/" % l
            lay = {"ln1": (f(ld + "ln1_gamma.bin", d), f(ld + "ln1_beta.bin", d)),
                   "ln2": (f(ld + "ln2_gamma.bin", d), f(ld + "ln2_beta.bin", d))}
            for name, (N, K) in shapes.items():
                lay[name] = (i(ld + name + "_weight.bin", N * K // 4).reshape(N, K // 4),
                             f(ld + name + "_scale.bin", N), f(ld + name + "_bias.bin", N))
            self.layers.append(lay)

    def reset(self, batch):
        c = self.cfg
        self.B = batch
        self.nb = (c["max_seq_len"] + 15) // 16
        shape = (c["n_layers"], batch * self.nb, 16, c["n_heads"], c["d_head"])
        self.k = np.zeros(shape, np.float32)
        self.v = np.zeros(shape, np.float32)
        self.bt = np.arange(batch * self.nb, dtype=np.int32).reshape(batch, self.nb)

    def step(self, tokens, pos, nthreads=0):
        """Appends tokens[b] at position pos[b] for every sequence; returns logits [B, V]."""
        c = self.cfg
        d, H, dh = c["d_model"], c["n_heads"], c["d_head"]
        tokens = np.asarray(tokens)
        pos = np.asarray(pos)
        x = (self.wte[tokens] + self.wpe[pos]).astype(np.float32)
        for l, lay in enumerate(self.layers):
            y = layernorm(x, *lay["ln1"])
            q8, s = quantize(y)
            w, ws, wb = lay["qkv"]
            qkv = int8_gemm(q8, w, s, ws, wb, None, 1, nthreads)
            for b in range(self.B):
                p = int(pos[b])
                blk, slot = self.bt[b, p // 16], p % 16
                self.k[l, blk, slot] = qkv[b, d:2 * d].reshape(H, dh)
                self.v[l, blk, slot] = qkv[b, 2 * d:].reshape(H, dh)
            att = decode_attn(qkv[:, :d].reshape(self.B, H, dh), self.k[l], self.v[l], self.bt,
                              (pos + 1).astype(np.int32), nthreads=nthreads).reshape(self.B, d)
            q8, s = quantize(att)
            w, ws, wb = lay["out"]
            x = int8_gemm(q8, w, s, ws, wb, x, 3, nthreads)
            y = layernorm(x, *lay["ln2"])
            q8, s = quantize(y)
            w, ws, wb = lay["ffn_up"]
            h = int8_gemm(q8, w, s, ws, wb, None, 2, nthreads)
            q8, s = quantize(h)
            w, ws, wb = lay["ffn_down"]
            x = int8_gemm(q8, w, s, ws, wb, x, 3, nthreads)
        xf = layernorm(x, *self.lnf)
        return vocab_proj(xf, self.wte, nthreads)

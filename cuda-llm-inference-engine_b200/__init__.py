"""B200 (sm_100a) GPT-2 decode hot path: host-side mirror of the reference's launch API.

The kernels live in ``libb2decode.so`` (built in-tree from ``csrc/`` by ``build_lib.py``)
and are reached only through its C ABI (``include/b2decode.h``) and the reference-named
C++ entry points (``include/b2_reference_api.h``). Torch tensors are used here purely as
device memory and for the current CUDA stream; every computation runs in the library.

Reference-named functions (same argument order and meaning as the reference):
    run_decode_attn              kernels/decode/13_decode_attn.cuh:192-199
    run_quantize_fp32_to_int8    kernels/quantization/14_int8_gemm.cuh:20-23
    run_int8_gemm[_bias|_bias_gelu|_bias_residual]  kernels/quantization/14_int8_gemm.cuh:28-64
They call the library's reference-compatible C++ symbols on the legacy default stream,
exactly as the reference's wrappers launch. Where the reference fails silently (an
unsupported GQA group is a no-op, 13_decode_attn.cu:306) these raise ``B2Error``.

Extended entry points (C ABI): ``decode_attn`` (bf16 KV, head_dim 128, explicit stream,
bounds-checked block table), ``int8_gemm`` and ``int8_gemm_s32`` (raw int32 accumulators).

There is no CPU path: importing works anywhere, but every call needs the built library
and a CUDA device, and fails loudly otherwise.
"""
from __future__ import annotations

import ctypes
import os

_PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG_DIR, "libb2decode.so")

B2_OK, B2_ERR_INVALID, B2_ERR_UNSUPPORTED, B2_ERR_WORKSPACE, B2_ERR_CUDA, B2_ERR_TIMEOUT = 0, 1, 2, 3, 4, 5
B2_DEVERR_TIMEOUT, B2_DEVERR_CTX_RANGE, B2_DEVERR_BLOCK_RANGE = 1, 2, 4
B2_KV_F32, B2_KV_BF16 = 0, 1
EPI_PLAIN, EPI_BIAS, EPI_BIAS_GELU, EPI_BIAS_RESIDUAL = 0, 1, 2, 3
DA_MAX_SPLITS = 16  # reference kernels/decode/13_decode_attn.cuh:12; sizes run_decode_attn's workspace

# Mangled names of the reference-compatible C++ entry points (include/b2_reference_api.h).
_CXX = {
    "run_decode_attn": "_Z15run_decode_attniiiiPKfS0_S0_PKiS2_iiiPfS3_",
    "run_quantize_fp32_to_int8": "_Z25run_quantize_fp32_to_int8iiPKfPiPf",
    "run_int8_gemm": "_Z13run_int8_gemmiiiPKiS0_PKfS2_Pf",
    "run_int8_gemm_bias": "_Z18run_int8_gemm_biasiiiPKiS0_PKfS2_S2_Pf",
    "run_int8_gemm_bias_gelu": "_Z23run_int8_gemm_bias_geluiiiPKiS0_PKfS2_S2_Pf",
    "run_int8_gemm_bias_residual": "_Z27run_int8_gemm_bias_residualiiiPKiS0_PKfS2_S2_S2_Pf",
}

# Every symbol include/*.h declares (checked by the CPU tests).
C_ABI_SYMBOLS = [
    "b2_decode_attn_workspace_size", "b2_decode_attn", "b2_decode_attn_noalloc", "b2_quantize_fp32_to_int8", "b2_int8_gemm",
    "b2_int8_gemm_workspace_size", "b2_int8_gemm_ws", "b2_int8_gemm_s32", "b2_int8_gemm_s32_ws", "b2_layernorm", "b2_get_device_error", "b2_last_status", "b2_status_string", "b2_version",
]


class B2Error(RuntimeError):
    """A library call returned a non-OK status, or the device error word was set."""


class DecodeAttnArgs(ctypes.Structure):
    """Mirror of ``b2_decode_attn_args`` (include/b2decode.h)."""

    _fields_ = [
        ("B", ctypes.c_int), ("H_q", ctypes.c_int), ("H_kv", ctypes.c_int), ("head_dim", ctypes.c_int),
        ("Q", ctypes.c_void_p), ("k_cache", ctypes.c_void_p), ("v_cache", ctypes.c_void_p),
        ("kv_dtype", ctypes.c_int), ("block_table", ctypes.c_void_p), ("context_lens", ctypes.c_void_p),
        ("max_context_len", ctypes.c_int), ("block_size", ctypes.c_int), ("num_blocks_per_seq", ctypes.c_int),
        ("num_phys_blocks", ctypes.c_int), ("scale", ctypes.c_float), ("O", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t),
    ]


_lib = None


def load_library(path: str | None = None) -> ctypes.CDLL:
    """Loads libb2decode.so (raises if it has not been built)."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = path or LIB_PATH
    if not os.path.exists(p):
        raise B2Error(f"{p} is missing: build it with `python {_PKG_DIR}/build_lib.py` "
                      "(there is no CPU fallback)")
    lib = ctypes.CDLL(p, mode=ctypes.RTLD_LOCAL)
    vp, i, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t
    lib.b2_decode_attn_workspace_size.argtypes = [i, i, i, i, i, i]
    lib.b2_decode_attn_workspace_size.restype = sz
    lib.b2_decode_attn.argtypes = [ctypes.POINTER(DecodeAttnArgs), vp]
    lib.b2_decode_attn.restype = i
    lib.b2_decode_attn_noalloc.argtypes = [ctypes.POINTER(DecodeAttnArgs), vp]
    lib.b2_decode_attn_noalloc.restype = i
    lib.b2_quantize_fp32_to_int8.argtypes = [i, i, vp, vp, vp, vp]
    lib.b2_quantize_fp32_to_int8.restype = i
    lib.b2_int8_gemm.argtypes = [i, i, i, vp, vp, vp, vp, vp, vp, vp, i, vp]
    lib.b2_int8_gemm.restype = i
    lib.b2_int8_gemm_workspace_size.argtypes = [i, i, i]
    lib.b2_int8_gemm_workspace_size.restype = sz
    lib.b2_int8_gemm_ws.argtypes = [i, i, i, vp, vp, vp, vp, vp, vp, vp, i, vp, sz, vp]
    lib.b2_int8_gemm_ws.restype = i
    lib.b2_int8_gemm_s32.argtypes = [i, i, i, vp, vp, vp, vp]
    lib.b2_int8_gemm_s32.restype = i
    lib.b2_int8_gemm_s32_ws.argtypes = [i, i, i, vp, vp, vp, vp, sz, vp]
    lib.b2_int8_gemm_s32_ws.restype = i
    lib.b2_layernorm.argtypes = [i, i, vp, vp, vp, ctypes.c_float, vp, vp, vp, vp]
    lib.b2_layernorm.restype = i
    lib.b2_get_device_error.argtypes = [i]
    lib.b2_get_device_error.restype = ctypes.c_uint
    lib.b2_last_status.argtypes = []
    lib.b2_last_status.restype = i
    lib.b2_status_string.argtypes = [i]
    lib.b2_status_string.restype = ctypes.c_char_p
    lib.b2_version.argtypes = []
    lib.b2_version.restype = i
    cx = {}
    for name, mangled in _CXX.items():
        f = getattr(lib, mangled)
        f.restype = None
        cx[name] = f
    f = cx["run_decode_attn"]
    f.argtypes = [i, i, i, i, vp, vp, vp, vp, vp, i, i, i, vp, vp]
    cx["run_quantize_fp32_to_int8"].argtypes = [i, i, vp, vp, vp]
    cx["run_int8_gemm"].argtypes = [i, i, i, vp, vp, vp, vp, vp]
    cx["run_int8_gemm_bias"].argtypes = [i, i, i, vp, vp, vp, vp, vp, vp]
    cx["run_int8_gemm_bias_gelu"].argtypes = [i, i, i, vp, vp, vp, vp, vp, vp]
    cx["run_int8_gemm_bias_residual"].argtypes = [i, i, i, vp, vp, vp, vp, vp, vp, vp]
    lib._cxx = cx
    if path is None:
        _lib = lib
    return lib


def _ptr(t):
    if t is None:
        return None
    if not t.is_cuda:
        raise B2Error("expected a CUDA tensor (all pointers are device pointers)")
    if not t.is_contiguous():
        raise B2Error("expected a contiguous tensor")
    return t.data_ptr()


def _stream(stream):
    if stream is not None:
        return ctypes.c_void_p(getattr(stream, "cuda_stream", stream))
    import torch

    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _check(status: int, what: str):
    if status != B2_OK:
        msg = load_library().b2_status_string(status).decode()
        raise B2Error(f"{what}: {msg} (status {status})")


def _check_last(what: str):
    _check(load_library().b2_last_status(), what)


def device_error(clear: bool = True) -> int:
    """Synchronises the device and returns (and by default clears) the device error bits."""
    return int(load_library().b2_get_device_error(1 if clear else 0))


# ---------------------------------------------------------------- reference-named API
def run_decode_attn(B, H_q, H_kv, d, Q, k_cache, v_cache, block_table, context_lens, max_context_len,
                    block_size, num_blocks_per_seq, O, workspace):
    """K13 decode attention with the reference's signature (13_decode_attn.cuh:192-199).

    fp32 KV cache; workspace is the reference's ``[B, H_q, DA_MAX_SPLITS, d+2]`` floats."""
    lib = load_library()
    lib._cxx["run_decode_attn"](B, H_q, H_kv, d, _ptr(Q), _ptr(k_cache), _ptr(v_cache), _ptr(block_table),
                                _ptr(context_lens), max_context_len, block_size, num_blocks_per_seq, _ptr(O),
                                _ptr(workspace))
    _check_last("run_decode_attn")


def run_quantize_fp32_to_int8(rows, cols, input, output_packed, scales):
    """Per-row int8 quantiser with the reference's signature (14_int8_gemm.cuh:20-23)."""
    load_library()._cxx["run_quantize_fp32_to_int8"](rows, cols, _ptr(input), _ptr(output_packed), _ptr(scales))
    _check_last("run_quantize_fp32_to_int8")


def run_int8_gemm(M, N, K, A_packed, BT_packed, scale_A, scale_B, C):
    load_library()._cxx["run_int8_gemm"](M, N, K, _ptr(A_packed), _ptr(BT_packed), _ptr(scale_A), _ptr(scale_B),
                                         _ptr(C))
    _check_last("run_int8_gemm")


def run_int8_gemm_bias(M, N, K, A_packed, BT_packed, scale_A, scale_B, bias, C):
    load_library()._cxx["run_int8_gemm_bias"](M, N, K, _ptr(A_packed), _ptr(BT_packed), _ptr(scale_A),
                                              _ptr(scale_B), _ptr(bias), _ptr(C))
    _check_last("run_int8_gemm_bias")


def run_int8_gemm_bias_gelu(M, N, K, A_packed, BT_packed, scale_A, scale_B, bias, C):
    load_library()._cxx["run_int8_gemm_bias_gelu"](M, N, K, _ptr(A_packed), _ptr(BT_packed), _ptr(scale_A),
                                                   _ptr(scale_B), _ptr(bias), _ptr(C))
    _check_last("run_int8_gemm_bias_gelu")


def run_int8_gemm_bias_residual(M, N, K, A_packed, BT_packed, scale_A, scale_B, bias, residual, C):
    load_library()._cxx["run_int8_gemm_bias_residual"](M, N, K, _ptr(A_packed), _ptr(BT_packed), _ptr(scale_A),
                                                       _ptr(scale_B), _ptr(bias), _ptr(residual), _ptr(C))
    _check_last("run_int8_gemm_bias_residual")


# ---------------------------------------------------------------- C-ABI API
def decode_attn_workspace_size(B, H_q, H_kv, head_dim, max_context_len, block_size=16) -> int:
    return int(load_library().b2_decode_attn_workspace_size(B, H_q, H_kv, head_dim, max_context_len, block_size))


def make_decode_workspace(B, H_q, H_kv, head_dim, max_context_len, block_size=16, device=None):
    """Allocates (torch) and zeroes a workspace for ``decode_attn``."""
    import torch

    n = max(256, decode_attn_workspace_size(B, H_q, H_kv, head_dim, max_context_len, block_size))
    return torch.zeros(n, dtype=torch.uint8, device=device or "cuda")


def _decode_shapes(Q, k_cache, v_cache, block_size=None):
    """Validates the decode-attention operands before anything is launched and returns
    (B, H_q, d, P, block_size, H_kv, kv_dtype). The KV cache must be fp32 or bf16, k and v
    must agree in shape and dtype, and head_dim must equal Q's last dimension: a wrong
    element size would make the kernels address past the caches' allocations."""
    import torch

    B, H_q, d = Q.shape[0], Q.shape[1], Q.shape[-1]
    if Q.dtype != torch.float32:
        raise B2Error(f"Q must be float32, got {Q.dtype}")
    if k_cache.dim() != 4:
        raise B2Error("k_cache must be [P, block_size, H_kv, head_dim]")
    P, bs, H_kv, d2 = k_cache.shape
    if d2 != d or v_cache.shape != k_cache.shape or v_cache.dtype != k_cache.dtype:
        raise B2Error("k_cache / v_cache / Q shapes disagree")
    if block_size is not None and block_size != bs:
        raise B2Error("block_size disagrees with k_cache.shape[1]")
    if k_cache.dtype == torch.float32:
        kvd = B2_KV_F32
    elif k_cache.dtype == torch.bfloat16:
        kvd = B2_KV_BF16
    else:
        raise B2Error(f"unsupported KV dtype {k_cache.dtype}")
    return B, H_q, d, P, bs, H_kv, kvd


def decode_attn(Q, k_cache, v_cache, block_table, context_lens, max_context_len, O=None, workspace=None,
                block_size=None, num_phys_blocks=None, scale=0.0, stream=None):
    """Paged decode attention through ``b2_decode_attn``.

    Q [B, H_q, d] (or [B, H_q, 1, d]) fp32; k/v_cache [P, block_size, H_kv, d] fp32 or bf16;
    block_table [B, nbps] int32; context_lens [B] int32. Returns O (same shape as Q)."""
    import torch

    B, H_q, d, P, bs, H_kv, kvd = _decode_shapes(Q, k_cache, v_cache, block_size)
    if O is None:
        O = torch.empty_like(Q)
    if workspace is None:
        workspace = make_decode_workspace(B, H_q, H_kv, d, max_context_len, bs, device=Q.device)
    a = DecodeAttnArgs(B, H_q, H_kv, d, _ptr(Q), _ptr(k_cache), _ptr(v_cache), kvd, _ptr(block_table),
                       _ptr(context_lens), int(max_context_len), bs, block_table.shape[1],
                       int(P if num_phys_blocks is None else num_phys_blocks), float(scale), _ptr(O),
                       _ptr(workspace), workspace.numel() * workspace.element_size())
    _check(load_library().b2_decode_attn(ctypes.byref(a), _stream(stream)), "b2_decode_attn")
    return O


DECODE_NOALLOC_SCRATCH_BYTES = 16 << 20  # B2_DECODE_NOALLOC_SCRATCH_BYTES


def decode_attn_noalloc(Q, k_cache, v_cache, block_table, context_lens, max_context_len, O, scale=0.0,
                        num_phys_blocks=None, stream=None):
    """Decode attention through ``b2_decode_attn_noalloc``: the library allocates nothing and
    uses its fixed per-GPU scratch array instead of a workspace. For callers that cannot
    allocate device memory; O must be provided. Overlapping calls on one GPU race on the
    shared scratch, so issue them on one stream (or otherwise serialise them)."""
    B, H_q, d, P, bs, H_kv, kvd = _decode_shapes(Q, k_cache, v_cache)
    if O is None or O.shape != Q.shape or O.dtype != Q.dtype:
        raise B2Error("O must be provided with Q's shape and dtype")
    a = DecodeAttnArgs(B, H_q, H_kv, d, _ptr(Q), _ptr(k_cache), _ptr(v_cache), kvd, _ptr(block_table),
                       _ptr(context_lens), int(max_context_len), bs, block_table.shape[1],
                       int(P if num_phys_blocks is None else num_phys_blocks), float(scale), _ptr(O), None, 0)
    _check(load_library().b2_decode_attn_noalloc(ctypes.byref(a), _stream(stream)), "b2_decode_attn_noalloc")
    return O


def layernorm(x, gamma, beta, eps=1e-5, out=None, quantize=False, stream=None):
    """LayerNorm of x [rows, cols] fp32 (b2_layernorm), in the reference kernel's summation
    order. quantize=True also returns the per-row int8 quantisation: (out, q_packed, scales)."""
    import torch

    rows, cols = x.shape
    if out is None:
        out = torch.empty_like(x)
    q = s = None
    if quantize:
        q = torch.empty(rows, cols // 4, dtype=torch.int32, device=x.device)
        s = torch.empty(rows, dtype=torch.float32, device=x.device)
    _check(load_library().b2_layernorm(rows, cols, _ptr(x), _ptr(gamma), _ptr(beta), float(eps), _ptr(out), _ptr(q),
                                       _ptr(s), _stream(stream)), "b2_layernorm")
    return (out, q, s) if quantize else out


def quantize_fp32_to_int8(x, out=None, scales=None, stream=None):
    """Returns (packed int32 [rows, cols/4], scales fp32 [rows])."""
    import torch

    rows, cols = x.shape
    if out is None:
        out = torch.empty(rows, cols // 4, dtype=torch.int32, device=x.device)
    if scales is None:
        scales = torch.empty(rows, dtype=torch.float32, device=x.device)
    _check(load_library().b2_quantize_fp32_to_int8(rows, cols, _ptr(x), _ptr(out), _ptr(scales), _stream(stream)),
           "b2_quantize_fp32_to_int8")
    return out, scales


def int8_gemm(A_packed, BT_packed, scale_A, scale_B, bias=None, residual=None, epilogue=EPI_PLAIN, C=None,
              stream=None, workspace=None):
    """INT8 GEMM; with ``workspace`` (make_gemm_workspace) skinny shapes are split along K."""
    import torch

    M, K4 = A_packed.shape
    N = BT_packed.shape[0]
    if C is None:
        C = torch.empty(M, N, dtype=torch.float32, device=A_packed.device)
    lib = load_library()
    if workspace is None:
        _check(lib.b2_int8_gemm(M, N, 4 * K4, _ptr(A_packed), _ptr(BT_packed), _ptr(scale_A), _ptr(scale_B),
                                _ptr(bias), _ptr(residual), _ptr(C), epilogue, _stream(stream)), "b2_int8_gemm")
    else:
        _check(lib.b2_int8_gemm_ws(M, N, 4 * K4, _ptr(A_packed), _ptr(BT_packed), _ptr(scale_A), _ptr(scale_B),
                                   _ptr(bias), _ptr(residual), _ptr(C), epilogue, _ptr(workspace),
                                   workspace.numel() * workspace.element_size(), _stream(stream)), "b2_int8_gemm_ws")
    return C


def int8_gemm_workspace_size(M, N, K) -> int:
    return int(load_library().b2_int8_gemm_workspace_size(M, N, K))


def make_gemm_workspace(M, N, K, device=None):
    """Allocates (torch) and zeroes a split-K workspace for ``int8_gemm(..., workspace=...)``."""
    import torch

    return torch.zeros(max(256, int8_gemm_workspace_size(M, N, K)), dtype=torch.uint8, device=device or "cuda")


def int8_gemm_s32(A_packed, BT_packed, C=None, stream=None, workspace=None):
    """Raw int32 accumulators; ``workspace`` (make_gemm_workspace) as for ``int8_gemm``."""
    import torch

    M, K4 = A_packed.shape
    N = BT_packed.shape[0]
    if C is None:
        C = torch.empty(M, N, dtype=torch.int32, device=A_packed.device)
    lib = load_library()
    if workspace is None:
        _check(lib.b2_int8_gemm_s32(M, N, 4 * K4, _ptr(A_packed), _ptr(BT_packed), _ptr(C), _stream(stream)),
               "b2_int8_gemm_s32")
    else:
        _check(lib.b2_int8_gemm_s32_ws(M, N, 4 * K4, _ptr(A_packed), _ptr(BT_packed), _ptr(C), _ptr(workspace),
                                       workspace.numel() * workspace.element_size(), _stream(stream)),
               "b2_int8_gemm_s32_ws")
    return C


# ---------------------------------------------------------------- GPT-2 decode engine (include/b2engine.h)
class GPT2Config(ctypes.Structure):
    """Mirror of ``b2_gpt2_config`` (the reference's GPT2Config, include/gpt2_types.cuh:6-14)."""

    _fields_ = [(n, ctypes.c_int) for n in
                ("n_layers", "n_heads", "d_model", "d_ff", "vocab_size", "max_seq_len", "d_head")]


ENGINE_SYMBOLS = ["b2_engine_create_random", "b2_nccl_unique_id", "b2_engine_create_random_tp",
                  "b2_engine_fill_kv_random", "b2_engine_load", "b2_engine_export", "b2_engine_destroy",
                  "b2_engine_config", "b2_engine_start", "b2_engine_step", "b2_engine_run_steps", "b2_engine_decode_step",
                  "b2_engine_read_tokens", "b2_engine_keep_logits", "b2_engine_read_logits", "b2_engine_positions",
                  "b2_engine_profile_step", "b2_engine_prefill", "b2_tp_exchange_bytes",
                  "b2_tp_quantize_absent_peer"]


def _engine_lib():
    lib = load_library()
    if getattr(lib, "_engine_ready", False):
        return lib
    vp, i, u64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint64
    pe = ctypes.POINTER(vp)
    lib.b2_engine_create_random.argtypes = [ctypes.POINTER(GPT2Config), i, i, u64, pe]
    lib.b2_engine_load.argtypes = [ctypes.c_char_p, i, i, pe]
    lib.b2_nccl_unique_id.argtypes = [vp, ctypes.c_size_t]
    lib.b2_engine_create_random_tp.argtypes = [ctypes.POINTER(GPT2Config), i, i, u64, vp, i, i, pe]
    lib.b2_engine_fill_kv_random.argtypes = [vp, i, u64]
    lib.b2_engine_export.argtypes = [vp, ctypes.c_char_p]
    lib.b2_engine_destroy.argtypes = [vp]
    lib.b2_engine_destroy.restype = None
    lib.b2_engine_config.argtypes = [vp, ctypes.POINTER(GPT2Config)]
    lib.b2_engine_start.argtypes = [vp, i, vp, vp, i, i, u64]
    lib.b2_engine_step.argtypes = [vp, vp]
    lib.b2_engine_run_steps.argtypes = [vp, i, vp]
    lib.b2_engine_decode_step.argtypes = [vp, vp, vp, vp]
    lib.b2_engine_profile_step.argtypes = [vp, ctypes.c_char_p, ctypes.c_size_t]
    lib.b2_engine_prefill.argtypes = [vp, vp]
    lib.b2_engine_read_tokens.argtypes = [vp, vp, i]
    lib.b2_engine_keep_logits.argtypes = [vp, i, ctypes.POINTER(vp)]
    lib.b2_engine_read_logits.argtypes = [vp, vp]
    lib.b2_engine_positions.argtypes = [vp, vp]
    lib.b2_tp_exchange_bytes.argtypes = [i]
    lib.b2_tp_quantize_absent_peer.argtypes = [i, i, vp, vp, vp, vp, vp, vp]
    for n in ENGINE_SYMBOLS:
        if n != "b2_engine_destroy":
            getattr(lib, n).restype = i
    lib.b2_tp_exchange_bytes.restype = ctypes.c_size_t
    lib._engine_ready = True
    return lib


class Engine:
    """Batched GPT-2 INT8 decode engine: one greedy token per sequence per step, on the GPU.

    Engine.random(cfg, max_batch) builds seeded N(0, 0.02) weights; Engine.load(dir) reads the
    reference's model directory format; start() sets prompts; step()/run_steps() decode."""

    def __init__(self, handle):
        self._h = handle
        self._lib = _engine_lib()
        c = GPT2Config()
        _check(self._lib.b2_engine_config(self._h, ctypes.byref(c)), "b2_engine_config")
        self.cfg = {n: getattr(c, n) for n, _ in GPT2Config._fields_}
        self.batch = 0

    @classmethod
    def random(cls, cfg: dict, max_batch: int, kv_dtype: int = B2_KV_F32, seed: int = 0):
        lib = _engine_lib()
        c = GPT2Config(**cfg)
        h = ctypes.c_void_p()
        _check(lib.b2_engine_create_random(ctypes.byref(c), max_batch, kv_dtype, seed, ctypes.byref(h)),
               "b2_engine_create_random")
        return cls(h)

    @classmethod
    def random_tp(cls, cfg: dict, max_batch: int, nccl_id: bytes, rank: int, world: int, kv_dtype: int = B2_KV_F32,
                  seed: int = 0):
        """Tensor-parallel rank of the same seeded model (b2_engine_create_random_tp)."""
        lib = _engine_lib()
        c = GPT2Config(**cfg)
        h = ctypes.c_void_p()
        buf = ctypes.create_string_buffer(nccl_id, len(nccl_id))
        _check(lib.b2_engine_create_random_tp(ctypes.byref(c), max_batch, kv_dtype, seed, buf, rank, world,
                                              ctypes.byref(h)), "b2_engine_create_random_tp")
        e = cls(h)
        e.tp_rank, e.tp_size = rank, world
        return e

    def fill_kv_random(self, ctx_len: int, seed: int = 0):
        _check(self._lib.b2_engine_fill_kv_random(self._h, ctx_len, seed), "b2_engine_fill_kv_random")

    @classmethod
    def load(cls, model_dir: str, max_batch: int, kv_dtype: int = B2_KV_F32):
        lib = _engine_lib()
        h = ctypes.c_void_p()
        _check(lib.b2_engine_load(model_dir.encode(), max_batch, kv_dtype, ctypes.byref(h)), "b2_engine_load")
        return cls(h)

    def export(self, model_dir: str):
        _check(self._lib.b2_engine_export(self._h, model_dir.encode()), "b2_engine_export")

    def start(self, prompts, max_new_tokens: int, seed: int = 0):
        """prompts: list of token-id lists (one per sequence)."""
        import numpy as np

        B = len(prompts)
        stride = max(len(p) for p in prompts)
        arr = np.zeros((B, stride), np.int32)
        for b, p in enumerate(prompts):
            arr[b, : len(p)] = p
        lens = np.array([len(p) for p in prompts], np.int32)
        _check(self._lib.b2_engine_start(self._h, B, arr.ctypes.data, lens.ctypes.data, stride, max_new_tokens, seed),
               "b2_engine_start")
        self.batch = B
        self._stride = stride + max_new_tokens + 1

    def step(self, stream=None):
        _check(self._lib.b2_engine_step(self._h, _stream(stream)), "b2_engine_step")

    def prefill(self, stream=None):
        """Right after start(): all prompt tokens but the last of each sequence in one batched
        pass (b2_engine_prefill); the next step predicts the first new token."""
        _check(self._lib.b2_engine_prefill(self._h, _stream(stream)), "b2_engine_prefill")

    def run_steps(self, steps: int, stream=None):
        _check(self._lib.b2_engine_run_steps(self._h, steps, _stream(stream)), "b2_engine_run_steps")

    def decode_step(self, tokens_in, next_out=None, stream=None):
        """One step on caller-chosen input tokens (b2_engine_decode_step): tokens_in [batch]
        int32 (a torch tensor on the device or on the host, or a numpy array); returns the
        greedy next tokens (numpy int32 [batch]) unless next_out (a tensor) is given, which
        is then filled asynchronously."""
        import numpy as np

        if isinstance(tokens_in, np.ndarray):
            tin = np.ascontiguousarray(tokens_in, np.int32)
            tin_p = tin.ctypes.data
        else:
            tin_p = _ptr(tokens_in)
        if next_out is None:
            out = np.zeros(self.batch, np.int32)
            _check(self._lib.b2_engine_decode_step(self._h, tin_p, out.ctypes.data, _stream(stream)),
                   "b2_engine_decode_step")
            return out
        _check(self._lib.b2_engine_decode_step(self._h, tin_p, _ptr(next_out), _stream(stream)),
               "b2_engine_decode_step")
        return next_out

    def profile_step(self) -> str:
        """One eager step with a CUDA event before every launch; returns the per-kernel-class
        breakdown (b2_engine_profile_step). Under tensor parallelism every rank must call it."""
        buf = ctypes.create_string_buffer(8192)
        _check(self._lib.b2_engine_profile_step(self._h, buf, ctypes.sizeof(buf)), "b2_engine_profile_step")
        return buf.value.decode()

    def keep_logits(self, enable: bool = True):
        _check(self._lib.b2_engine_keep_logits(self._h, 1 if enable else 0, None), "b2_engine_keep_logits")

    def logits(self):
        """Last step's logits [batch, vocab rows held by this rank] (all of them unless sharded)."""
        import numpy as np

        world = getattr(self, "tp_size", 1)
        per = (self.cfg["vocab_size"] + world - 1) // world
        v0 = min(self.cfg["vocab_size"], getattr(self, "tp_rank", 0) * per)
        out = np.zeros((self.batch, max(1, min(per, self.cfg["vocab_size"] - v0))), np.float32)
        _check(self._lib.b2_engine_read_logits(self._h, out.ctypes.data), "b2_engine_read_logits")
        return out

    def tokens(self):
        """[batch, stride] greedy token chosen after the step at position p-1 (-1: none yet)."""
        import numpy as np

        out = np.zeros((self.batch, self._stride), np.int32)
        _check(self._lib.b2_engine_read_tokens(self._h, out.ctypes.data, self._stride), "b2_engine_read_tokens")
        return out

    def positions(self):
        import numpy as np

        out = np.zeros(self.batch, np.int32)
        _check(self._lib.b2_engine_positions(self._h, out.ctypes.data), "b2_engine_positions")
        return out

    def close(self):
        if self._h:
            self._lib.b2_engine_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def nccl_unique_id() -> bytes:
    """An NCCL unique id for Engine.random_tp (rank 0 creates it, the caller shares it)."""
    buf = ctypes.create_string_buffer(128)
    _check(_engine_lib().b2_nccl_unique_id(buf, 128), "b2_nccl_unique_id")
    return buf.raw


def tp_quantize_absent_peer(x, stream=None):
    """Failure path of the tensor-parallel scale exchange (``b2_tp_quantize_absent_peer``):
    quantises x [rows, cols] as rank 0 of a 2-rank group whose other rank never arrives.
    Every row's bounded wait gives up and sets B2_DEVERR_TIMEOUT; returns (q_packed, scales)."""
    import torch

    lib = _engine_lib()
    rows, cols = x.shape
    nbytes = int(lib.b2_tp_exchange_bytes(rows))
    xchg = torch.zeros(2, (nbytes + 255) // 256 * 256, dtype=torch.uint8, device=x.device)
    q = torch.empty(rows, cols // 4, dtype=torch.int32, device=x.device)
    s = torch.empty(rows, dtype=torch.float32, device=x.device)
    _check(lib.b2_tp_quantize_absent_peer(rows, cols, _ptr(x), _ptr(q), _ptr(s), xchg[0].data_ptr(),
                                          xchg[1].data_ptr(), _stream(stream)), "b2_tp_quantize_absent_peer")
    return q, s

"""CPU checks of the boundary: the library loads without a GPU and exports every symbol
declared in include/*.h; host-side argument validation needs no device."""
import ctypes
import os
import re
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_c_symbols(header="b2decode.h"):
    txt = open(os.path.join(ROOT, "include", header)).read()
    return sorted(set(re.findall(r"\b(b2_[a-z0-9_]+)\s*\(", txt)))


def declared_cxx_symbols():
    txt = open(os.path.join(ROOT, "include", "b2_reference_api.h")).read()
    return sorted(set(re.findall(r"^void\s+(run_[a-z0-9_]+)\s*\(", txt, re.M)))


def test_header_symbol_lists_match_package(b2):
    assert declared_c_symbols() == sorted(b2.C_ABI_SYMBOLS)
    assert declared_c_symbols("b2engine.h") == sorted(b2.ENGINE_SYMBOLS)
    assert declared_cxx_symbols() == sorted(b2._CXX)


def test_library_exports_every_declared_symbol(b2):
    lib = b2.load_library()
    for s in declared_c_symbols() + declared_c_symbols("b2engine.h"):
        assert hasattr(lib, s), s
    out = subprocess.run(["nm", "-D", "--defined-only", b2.LIB_PATH], capture_output=True, text=True).stdout
    for name, mangled in b2._CXX.items():
        assert f" T {mangled}" in out, name
        demangled = subprocess.run(["c++filt", mangled], capture_output=True, text=True).stdout
        assert demangled.startswith(name + "("), demangled


def test_version_and_status_strings(b2):
    lib = b2.load_library()
    assert lib.b2_version() >= 100
    assert lib.b2_status_string(b2.B2_ERR_UNSUPPORTED) == b"unsupported shape"
    assert lib.b2_status_string(99) == b"unknown status"


def test_host_validation_without_device(b2):
    """Argument errors are reported before any CUDA call is made."""
    lib = b2.load_library()
    a = b2.DecodeAttnArgs()
    a.B, a.H_q, a.H_kv, a.head_dim, a.block_size = 1, 3, 1, 64, 16
    a.Q = a.k_cache = a.v_cache = a.block_table = a.context_lens = a.O = 16
    assert lib.b2_decode_attn(ctypes.byref(a), None) == b2.B2_ERR_UNSUPPORTED  # group 3
    a.H_q, a.head_dim = 2, 96
    assert lib.b2_decode_attn(ctypes.byref(a), None) == b2.B2_ERR_UNSUPPORTED  # head_dim 96
    a.head_dim = 64
    a.k_cache = 8
    assert lib.b2_decode_attn(ctypes.byref(a), None) == b2.B2_ERR_INVALID     # misaligned cache
    assert lib.b2_decode_attn(None, None) == b2.B2_ERR_INVALID
    assert lib.b2_quantize_fp32_to_int8(2, 6, 16, 16, 16, None) == b2.B2_ERR_INVALID  # cols % 4
    assert lib.b2_int8_gemm(2, 2, 6, 16, 16, 16, 16, None, None, 16, 0, None) == b2.B2_ERR_INVALID
    assert lib.b2_int8_gemm(2, 2, 8, 16, 16, 16, 16, None, None, 16, 1, None) == b2.B2_ERR_INVALID  # no bias
    assert lib.b2_int8_gemm(0, 2, 8, 16, 16, 16, 16, None, None, 16, 0, None) == b2.B2_OK  # empty


def test_workspace_size_query(b2):
    lib = b2.load_library()
    # 1 split (short context): counters only; long context: partial rows + counters
    short = lib.b2_decode_attn_workspace_size(1, 12, 12, 64, 32, 16)
    long_ = lib.b2_decode_attn_workspace_size(32, 32, 8, 128, 8192, 16)
    assert short > 0 and long_ > short
    assert lib.b2_decode_attn_workspace_size(0, 1, 1, 64, 1, 16) == 0


def test_missing_library_fails_loudly(b2, tmp_path):
    with pytest.raises(b2.B2Error, match="no CPU fallback"):
        b2.load_library(str(tmp_path / "nope.so"))


def test_library_before_torch_keeps_torch_importable():
    """Loading the library first must not pull a second NCCL into the process (NCCL is
    resolved at run time only for tensor parallelism), so torch still imports afterwards."""
    code = ("import sys, importlib; sys.path.insert(0, %r); "
            "b2 = importlib.import_module('cuda-llm-inference-engine_b200'); b2.load_library(); "
            "import torch; print('ok')" % ROOT)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stderr[-2000:]


def test_bench_reference_arm_runs_the_reference_harness():
    """bench.py --impl reference prints its JSON line from the reference's own compiled CPU
    attention when oracle/_ref is built (a short budget keeps this quick)."""
    import json

    from oracle import oracle

    if not oracle.ref_available():
        pytest.skip("oracle/_ref not built")
    env = dict(os.environ, B2_REF_BUDGET_S="2", CUDA_VISIBLE_DEVICES="")
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "1"], capture_output=True, text=True, timeout=300, env=env)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "reference" and line["e2e"]["h2d_bytes_per_step"] == 0


def test_decode_operand_validation_before_launch(b2):
    """The host mirror refuses caches the kernels cannot address (fp16/int8 elements, k and v
    that disagree in shape or dtype, a head_dim other than Q's) before it loads or launches
    anything, for both the workspace and the allocation-free entry points."""
    import torch

    q = torch.zeros(2, 4, 64)
    kc = torch.zeros(3, 16, 2, 64)
    bt = torch.zeros(2, 3, dtype=torch.int32)
    lens = torch.zeros(2, dtype=torch.int32)
    O = torch.zeros_like(q)
    for fn in (lambda k, v: b2.decode_attn(q, k, v, bt, lens, 48),
               lambda k, v: b2.decode_attn_noalloc(q, k, v, bt, lens, 48, O)):
        with pytest.raises(b2.B2Error, match="KV dtype"):
            fn(kc.half(), kc.half())
        with pytest.raises(b2.B2Error, match="KV dtype"):
            fn(kc.to(torch.int8), kc.to(torch.int8))
        with pytest.raises(b2.B2Error, match="disagree"):
            fn(kc, kc.bfloat16())
        with pytest.raises(b2.B2Error, match="disagree"):
            fn(kc, torch.zeros(4, 16, 2, 64))
        with pytest.raises(b2.B2Error, match="disagree"):
            fn(torch.zeros(3, 16, 2, 128), torch.zeros(3, 16, 2, 128))
    with pytest.raises(b2.B2Error, match="O must"):
        b2.decode_attn_noalloc(q, kc, kc, bt, lens, 48, None)

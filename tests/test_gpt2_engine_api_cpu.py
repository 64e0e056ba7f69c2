"""The GPT2Engine drop-in without a GPU: a caller written against the reference's API
(tests/gpt2_engine_driver.cpp) compiles against include/gpt2_engine.cuh and links with
libb2decode.so, which exports the class's members; a missing model directory is an
exception, not a process exit."""
import os
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(ROOT, "cuda-llm-inference-engine_b200")


def build_driver(out_dir):
    exe = os.path.join(out_dir, "gpt2_engine_driver")
    cmd = ["g++", "-std=c++17", "-O1", "-I", os.path.join(ROOT, "include"),
           os.path.join(ROOT, "tests", "gpt2_engine_driver.cpp"), "-o", exe, "-L", LIBDIR, "-lb2decode",
           f"-Wl,-rpath,{LIBDIR}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_driver_builds_and_reports_missing_model(b2, tmp_path):
    b2.load_library()
    exe = build_driver(str(tmp_path))
    r = subprocess.run([exe, str(tmp_path / "no_model"), "4", "greedy", "1", "2"], capture_output=True, text=True,
                       timeout=300, env=dict(os.environ, CUDA_VISIBLE_DEVICES=""))
    assert r.returncode == 1 and r.stdout.startswith("error: b2_engine_load"), r.stdout + r.stderr


def test_library_exports_gpt2engine_members(b2):
    out = subprocess.run(["nm", "-DC", "--defined-only", b2.LIB_PATH], capture_output=True, text=True).stdout
    for sym in ("GPT2Engine::GPT2Engine(std::__cxx11::basic_string<char, std::char_traits<char>, "
                "std::allocator<char> > const&, InferenceBackend)",
                "GPT2Engine::~GPT2Engine()",
                "GPT2Engine::generate(std::vector<int, std::allocator<int> > const&, int, float, int, bool, "
                "std::function<void (int)>, InferenceMetrics&, bool)",
                "GPT2Engine::reset_session()"):
        assert sym in out, sym

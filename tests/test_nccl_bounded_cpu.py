"""Bounded NCCL communicator creation and enqueue (csrc/nccl_bounded.h), on the host with fake
NCCL functions: a peer that joins late is waited for; one that never joins ends in
B2_ERR_TIMEOUT within the bound with the communicator aborted; NCCL errors become
B2_ERR_CUDA (aborted too); an enqueue that reports ncclInProgress is waited out or times out;
teardown finalizes and destroys a quiescent communicator and aborts one whose peer is gone.
The communicator is always requested in non-blocking mode."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HERE = os.path.join(ROOT, "tests")


@pytest.fixture(scope="module")
def fakes_output(tmp_path_factory):
    if shutil.which("g++") is None or not os.path.exists("/usr/include/nccl.h"):
        pytest.skip("needs g++ and nccl.h")
    exe = str(tmp_path_factory.mktemp("nccl") / "fakes")
    cuda_inc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "include")
    subprocess.run(["g++", "-std=c++17", "-O1", "-I", os.path.join(ROOT, "cuda-llm-inference-engine_b200", "csrc"),
                    "-I", os.path.join(ROOT, "include"), "-I", cuda_inc, os.path.join(HERE, "nccl_bounded_fakes.cpp"),
                    "-o", exe], check=True, capture_output=True, text=True)
    out = subprocess.run([exe], check=True, capture_output=True, text=True, timeout=60).stdout
    return {line.split()[0]: line.split()[1:] for line in out.splitlines()}


def test_communicator_creation_is_bounded(b2, fakes_output):
    st, aborted, secs, have, blocking = fakes_output["joins_after_polls"]
    assert (int(st), int(aborted), int(have), int(blocking)) == (b2.B2_OK, 0, 1, 0)
    st, aborted, secs, have, _ = fakes_output["never_joins"]
    assert (int(st), int(aborted), int(have)) == (b2.B2_ERR_TIMEOUT, 1, 0)
    assert 0.25 < float(secs) < 5.0  # the 0.3 s bound, not a hang
    st, aborted, _, have, _ = fakes_output["init_error"]
    assert (int(st), int(aborted), int(have)) == (b2.B2_ERR_CUDA, 1, 0)
    st, aborted, _, have, _ = fakes_output["async_error"]
    assert (int(st), int(aborted), int(have)) == (b2.B2_ERR_CUDA, 1, 0)


def test_enqueue_in_progress_is_bounded(b2, fakes_output):
    assert int(fakes_output["enqueue_in_progress"][0]) == b2.B2_OK
    assert int(fakes_output["enqueue_stuck"][0]) == b2.B2_ERR_TIMEOUT
    assert int(fakes_output["enqueue_error"][0]) == b2.B2_ERR_CUDA


def test_teardown_is_bounded(b2, fakes_output):
    st, destroyed, aborted = map(int, fakes_output["destroy_quiescent"])
    assert (st, destroyed, aborted) == (b2.B2_OK, 1, 0)
    st, destroyed, aborted = map(int, fakes_output["destroy_peer_gone"])
    assert (st, destroyed, aborted) == (b2.B2_ERR_TIMEOUT, 0, 1)


def test_timeout_status_string(b2):
    assert b2.load_library().b2_status_string(b2.B2_ERR_TIMEOUT) == b"peer timeout"

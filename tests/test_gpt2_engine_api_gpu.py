"""GPT2Engine (include/gpt2_engine.cuh), the reference's generation API, driven through its C++
symbols by tests/gpt2_engine_driver.cpp (the reference's src/main.cpp call pattern, compiled
against the header and linked with libb2decode.so), against the C ABI engine run on the same
model directory: identical greedy tokens for a fresh session and for a continuation
(reset_kv = false), and top-k sampling that only ever picks among the k largest logits."""
import os
import subprocess

import numpy as np
import pytest

from test_gpt2_engine_api_cpu import build_driver

pytestmark = pytest.mark.gpu

CFG = dict(n_layers=2, n_heads=12, d_model=768, d_ff=3072, vocab_size=50257, max_seq_len=256, d_head=64)


def _run(driver, model_dir, max_new, mode, prompt, max_new2=None, prompt2=None):
    args = [driver, model_dir, str(max_new), mode] + [str(t) for t in prompt]
    if prompt2:
        args += ["--", str(max_new2)] + [str(t) for t in prompt2]
    r = subprocess.run(args, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    lines = r.stdout.splitlines()
    toks = [list(map(int, l.split()[1:])) for l in lines if l.startswith("tokens:")]
    return toks, lines


def _expected(b2, model_dir, prompt, n1, prompt2=None, n2=0):
    """The same generation through b2_engine_decode_step (greedy), following GPT2Engine's
    loop: feed the prompt, then each chosen token until n tokens were handed out."""
    eng = b2.Engine.load(model_dir, max_batch=1)
    eng.start([prompt], CFG["max_seq_len"] - len(prompt))
    eng.prefill()
    nxt = int(eng.decode_step(np.array([prompt[-1]], np.int32))[0])
    out1 = []
    for _ in range(n1):
        if nxt == 50256:
            break
        out1.append(nxt)
        nxt = int(eng.decode_step(np.array([nxt], np.int32))[0])
    out2 = []
    if prompt2:
        for t in prompt2:
            nxt = int(eng.decode_step(np.array([t], np.int32))[0])
        for _ in range(n2):
            if nxt == 50256:
                break
            out2.append(nxt)
            nxt = int(eng.decode_step(np.array([nxt], np.int32))[0])
    eng.close()
    return out1, out2


@pytest.fixture(scope="module")
def model_dir(b2, cuda, tmp_path_factory):
    d = str(tmp_path_factory.mktemp("gpt2api"))
    e = b2.Engine.random(CFG, max_batch=1, seed=99)
    e.export(d)
    e.close()
    return d


def test_generate_greedy_matches_c_abi(b2, model_dir, tmp_path):
    driver = build_driver(str(tmp_path))
    rng = np.random.default_rng(4)
    prompt = list(map(int, rng.integers(0, CFG["vocab_size"], 20)))
    prompt2 = list(map(int, rng.integers(0, CFG["vocab_size"], 5)))
    toks, lines = _run(driver, model_dir, 16, "greedy", prompt, 12, prompt2)
    want1, want2 = _expected(b2, model_dir, prompt, 16, prompt2, 12)
    assert toks[0] == want1 and toks[1] == want2, "\n".join(lines)
    session = [int(l.split()[1]) for l in lines if l.startswith("session")]
    assert session[0] == len(prompt) + len(want1)
    assert session[1] == session[0] + len(prompt2) + len(want2)
    m = [l for l in lines if l.startswith("metrics:")][0].split()
    assert int(m[2]) == len(want2) and float(m[8]) > 0  # tokens_generated, tps


def test_generate_topk_samples_within_top_k(b2, model_dir, tmp_path):
    driver = build_driver(str(tmp_path))
    prompt = [464, 3616, 286, 1204, 318]
    toks, lines = _run(driver, model_dir, 12, "topk", prompt)
    assert len(toks[0]) >= 1, "\n".join(lines)
    # every sampled token must be among the 40 largest logits at its position
    eng = b2.Engine.load(model_dir, max_batch=1)
    eng.start([prompt], 64)
    eng.prefill()
    eng.keep_logits(True)
    seq = [prompt[-1]] + toks[0]
    for i, t in enumerate(toks[0]):
        eng.decode_step(np.array([seq[i]], np.int32))
        top = np.argsort(-eng.logits()[0])[:40]
        assert t in top, f"step {i}: sampled {t} outside the top 40"
    eng.close()

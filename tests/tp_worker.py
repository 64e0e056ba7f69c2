"""One rank of a tensor-parallel engine run (launched by tests/test_engine_tp_gpu.py).

    python tests/tp_worker.py RANK WORLD NCCL_ID_HEX SPEC_JSON OUT_NPZ

Runs the seeded engine's steps on GPU RANK and saves the greedy tokens, the logits shard of
every step and the final positions; then restarts the same prompts and replays the step as a
CUDA graph, saving those tokens too."""
import importlib
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main():
    rank, world = int(sys.argv[1]), int(sys.argv[2])
    nid = bytes.fromhex(sys.argv[3])
    spec = json.loads(sys.argv[4])
    import torch

    torch.cuda.set_device(rank)
    b2 = importlib.import_module("cuda-llm-inference-engine_b200")
    e = b2.Engine.random_tp(spec["cfg"], spec["max_batch"], nid, rank, world, kv_dtype=spec["kv_dtype"],
                            seed=spec["seed"])
    e.start(spec["prompts"], spec["new"], seed=spec["block_seed"])
    e.keep_logits(True)
    logits = []
    for _ in range(spec["steps"]):
        e.step()
        logits.append(e.logits())
    assert b2.device_error() == 0
    tokens, pos = e.tokens(), e.positions()
    e.start(spec["prompts"], spec["new"], seed=spec["block_seed"] + 1)
    e.run_steps(spec["steps"])
    assert b2.device_error() == 0
    np.savez(sys.argv[5], tokens=tokens, logits=np.stack(logits), pos=pos, graph_tokens=e.tokens())
    e.close()


if __name__ == "__main__":
    main()

"""Golden vectors of the full 9B-shaped synthetic package (config 2 shapes, seed 2024) from
the reference library compiled from its sources (oracle/_ref): a 32-token prompt, the hidden
state after prefill, 8 greedy decode tokens and the hidden state after them. The GPU test
rebuilds the same package from the same seed and compares the CUDA path with this file.

    python tests/golden/make_golden_9b.py      (about a minute on 8 cores; 6.6 GB package)
"""
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import __graft_entry__  # noqa: E402

__graft_entry__.load_package()
from xqwen35_b200.packer import synthetic  # noqa: E402
import oracle as O  # noqa: E402

SEED = 2024
PROMPT = 32
STEPS = 8


def prompt_ids():
    return np.random.default_rng(SEED + 77).integers(0, 248320, PROMPT).astype(np.int32)


def main():
    d = os.path.join(os.environ.get("TMPDIR", "/tmp"), "xq_bench", f"qwen35_9b_s{SEED}")
    synthetic.make_package(d, synthetic.preset("cfg2"), seed=SEED)
    s = O.RefSession(d, threads=8)
    t = time.time()
    ids = prompt_ids()
    s.prefill(ids)
    h0 = s.hidden()
    toks = np.array([s.decode_one() for _ in range(STEPS)], np.int32)
    h1 = s.hidden()
    s.close()
    np.savez_compressed(os.path.join(HERE, "model_9b_s2024.npz"), ids=ids, tokens=toks, hidden_prefill=h0,
                        hidden_after=h1)
    print(f"tokens {toks.tolist()} in {time.time() - t:.0f}s")


if __name__ == "__main__":
    main()

"""Golden vectors of the full 9B-shaped synthetic package (config 2 shapes, seed 2024) from
the reference library compiled from its sources (oracle/_ref).

Two files:

* model_9b_s2024.npz: a 32-token prompt, the hidden state after prefill, 8 greedy decode
  tokens and the hidden state after them (the quick full-size check).
* model_9b_p512_s2024.npz: the benchmark shape, a 512-token prompt then 32 greedy steps. At
  the checkpoints (after prefill, after decode steps 1, 8 and 32) it stores the reference's
  post-final-norm hidden state and its top-10 lm_head logits (values and indices), computed
  with the reference's own gemvW4A16Neon (xq_gemv_w4a16_neon.cpp:259-291) on that hidden
  state, the way CustomModel::debugJson does (custom_model.cpp:1382-1436) but at full fp32
  precision (debugJson prints 6 significant digits). The random-init package greedily emits
  nearly one token id, so token equality alone says little; the logits and hidden states
  carry the check. The top-1 / top-2 margins are printed for the record.
* model_cfg1_p512_s2024.npz: config 1 (two layers, DeltaNet + full attention, vocab 1024)
  with a 512-token prompt (KV cache filled to 512) and 8 decode steps, same checkpoints
  (after prefill and after steps 1 and 8).

    python tests/golden/make_golden_9b.py [quick|p512|cfg1]   (default: all; p512 takes about
    ten minutes on 8 cores, the 6.6 GB package is rebuilt from its seed where bench.py keeps it)
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
P512 = 512
P512_STEPS = 32
P512_CHECKPOINTS = (1, 8, 32)
CFG1_STEPS = 8
CFG1_CHECKPOINTS = (1, 8)
TOPK = 10


def prompt_ids():
    return np.random.default_rng(SEED + 77).integers(0, 248320, PROMPT).astype(np.int32)


def prompt_ids_p512(vocab=248320):
    return np.random.default_rng(SEED + 512).integers(0, vocab, P512).astype(np.int32)


def bench_dir(name):
    base = os.environ.get("XQ_BENCH_DIR", os.path.join(os.environ.get("TMPDIR", "/tmp"), "xq_bench"))
    return os.path.join(base, name)


def topk(lm_head, hidden, k=TOPK):
    """Top-k of the reference's lm_head GEMV: values descending, ties to the lower index (the
    order debugJson's insertion keeps)."""
    logits = O.ref_gemv(lm_head, hidden)
    order = np.lexsort((np.arange(logits.size), -logits.astype(np.float64)))[:k]
    return logits[order].astype(np.float32), order.astype(np.int32)


def run_checkpointed(d, ids, steps, checkpoints, threads=8):
    lm = O.Matrix.from_xq4(synthetic.read_xq4(os.path.join(d, "lm_head_weight.xq4")))
    s = O.RefSession(d, threads=threads)
    t = time.time()
    s.prefill(ids)
    print(f"prefill {ids.size} tokens in {time.time() - t:.0f}s", flush=True)
    hid, vals, idx, at = [], [], [], []

    def mark(step):
        h = s.hidden()
        v, i = topk(lm, h)
        hid.append(h)
        vals.append(v)
        idx.append(i)
        at.append(step)
        print(f"step {step}: top1 {i[0]} ({v[0]:.6g}), margin top1-top2 {v[0] - v[1]:.4g}", flush=True)

    mark(0)
    toks = []
    for k in range(1, steps + 1):
        toks.append(s.decode_one())
        if k in checkpoints:
            mark(k)
    s.close()
    return dict(ids=ids, tokens=np.array(toks, np.int32), steps=np.array(at, np.int32), hidden=np.stack(hid),
                topk_values=np.stack(vals), topk_indices=np.stack(idx))


def quick():
    d = bench_dir(f"qwen35_9b_s{SEED}")
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


def p512():
    d = bench_dir(f"qwen35_9b_s{SEED}")
    synthetic.make_package(d, synthetic.preset("cfg2"), seed=SEED)
    g = run_checkpointed(d, prompt_ids_p512(), P512_STEPS, P512_CHECKPOINTS)
    np.savez_compressed(os.path.join(HERE, "model_9b_p512_s2024.npz"), **g)
    print(f"tokens {g['tokens'].tolist()}")


def cfg1():
    cfg = synthetic.preset("cfg1")
    d = bench_dir(f"qwen35_cfg1_s{SEED}")
    synthetic.make_package(d, cfg, seed=SEED)
    # Every config-1 GEMV uses one or all eight pool threads (lm_head: 1024 rows / 128 per thread).
    g = run_checkpointed(d, prompt_ids_p512(cfg.vocab_size), CFG1_STEPS, CFG1_CHECKPOINTS)
    np.savez_compressed(os.path.join(HERE, "model_cfg1_p512_s2024.npz"), **g)
    print(f"tokens {g['tokens'].tolist()}")


if __name__ == "__main__":
    which = sys.argv[1:] or ["quick", "p512", "cfg1"]
    for w in which:
        {"quick": quick, "p512": p512, "cfg1": cfg1}[w]()

"""Tensor-parallel decode (xq_tp_*) on two GPUs against the compiled reference: config 1 (one
DeltaNet and one full-attention layer at 9B shapes, vocab 1024) with the 512-token prompt of
the reference golden, then 8 greedy steps. Both ranks hold half of every matrix (heads, MLP
rows, K slices of the output projections, vocabulary rows) and sum partial outputs with NCCL:
their hidden states must be identical, within 1e-4 of the reference's after prefill and after
steps 1 and 8, and the tokens exactly the reference's. Needs two visible GPUs (skipped
otherwise); each rank is its own process."""
import os

import numpy as np
import pytest

from conftest import GOLDEN, PKG, rel_err
from xqwen35_b200.packer import synthetic

pytestmark = pytest.mark.gpu

CFG1_512 = os.path.join(GOLDEN, "model_cfg1_p512_s2024.npz")


def _gpus():
    import torch

    return torch.cuda.device_count()


def _rank(rank, world, uid, d, ids, steps, q):
    try:
        t = PKG.Tp(d, world, rank, uid, max_context=600, device=rank)
        t.prefill(ids)
        hid = [t.hidden()]
        toks = []
        done = 0
        for k in steps[1:]:
            _, tk = t.decode(k - done)
            toks += list(tk)
            done = k
            hid.append(t.hidden())
        t.close()
        q.put((rank, "ok", toks, np.stack(hid)))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, repr(e), None, None))


@pytest.mark.skipif(not os.path.exists(CFG1_512), reason="cfg1 512-token golden file not generated")
def test_tp2_cfg1_matches_reference_golden():
    if _gpus() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    G = np.load(CFG1_512)
    d = os.path.join(os.environ.get("XQ_BENCH_DIR", os.path.join(os.environ.get("TMPDIR", "/tmp"), "xq_bench")),
                     "qwen35_cfg1_s2024")
    synthetic.make_package(d, synthetic.preset("cfg1"), seed=2024)
    steps = [int(s) for s in G["steps"]]
    assert steps[0] == 0 and steps[-1] == len(G["tokens"])
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")  # plain peer transfers: no multicast objects
    uid = PKG.Tp.unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, uid, d, G["ids"], steps, q), daemon=True) for r in range(2)]
    for p in procs:
        p.start()
    got = sorted(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    for rank, status, _, _ in got:
        assert status == "ok", (rank, status)
    (_, _, t0, h0), (_, _, t1, h1) = got
    assert np.array_equal(h0, h1) and t0 == t1  # the residual stream is replicated exactly
    for j in range(len(steps)):
        assert rel_err(h0[j], G["hidden"][j]) <= 1e-4, steps[j]
    assert t0 == list(G["tokens"])


@pytest.mark.skipif(not os.path.exists(CFG1_512), reason="cfg1 512-token golden file not generated")
def test_tp1_cfg1_matches_reference_golden():
    """The tensor-parallel engine on one GPU (a one-rank NCCL communicator, whole matrices):
    the same golden bars, on the path the multi-GPU runs take."""
    G = np.load(CFG1_512)
    d = os.path.join(os.environ.get("XQ_BENCH_DIR", os.path.join(os.environ.get("TMPDIR", "/tmp"), "xq_bench")),
                     "qwen35_cfg1_s2024")
    synthetic.make_package(d, synthetic.preset("cfg1"), seed=2024)
    steps = [int(s) for s in G["steps"]]
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    t = PKG.Tp(d, 1, 0, PKG.Tp.unique_id(), max_context=600, device=0)
    try:
        t.prefill(G["ids"])
        assert rel_err(t.hidden(), G["hidden"][0]) <= 1e-4
        toks, done = [], 0
        for j, k in enumerate(steps[1:], start=1):
            _, tk = t.decode(k - done)
            toks += list(tk)
            done = k
            assert rel_err(t.hidden(), G["hidden"][j]) <= 1e-4, k
        assert toks == list(G["tokens"])
    finally:
        t.close()


def test_tp2_shared_kv_head_matches_single_gpu_session():
    """More ranks than kv heads (the N = 8 layout of the 9B model, here on two GPUs): one kv
    head, replicated on both ranks, each rank with half of the query heads. Tokens and hidden
    states equal the single-GPU session's (itself pinned to the reference)."""
    if _gpus() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    cfg = synthetic.ModelConfig(hidden_size=2048, intermediate_size=2048, vocab_size=4096, num_attention_heads=8,
                                num_key_value_heads=1, head_dim=256, linear_num_key_heads=8, linear_num_value_heads=16,
                                layer_types=["linear_attention", "full_attention"])
    d = os.path.join(os.environ.get("XQ_BENCH_DIR", os.path.join(os.environ.get("TMPDIR", "/tmp"), "xq_bench")),
                     "tp_shared_kv_s5")
    synthetic.make_package(d, cfg, seed=5)
    assert PKG.tp_plan(d, 2, 0)["kv_heads"] == PKG.tp_plan(d, 2, 1)["kv_heads"] == [0, 1]
    ids = np.random.default_rng(8).integers(0, 4096, 40).astype(np.int32)
    steps = [0, 1, 6]
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    uid = PKG.Tp.unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, uid, d, ids, steps, q), daemon=True) for r in range(2)]
    for p in procs:
        p.start()
    got = sorted(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    for rank, status, _, _ in got:
        assert status == "ok", (rank, status)
    (_, _, t0, h0), (_, _, t1, h1) = got
    assert np.array_equal(h0, h1) and t0 == t1
    s = PKG.Session(d, device=0)
    try:
        s.prefill(ids)
        assert rel_err(h0[0], s.hidden()) <= 1e-4
        toks = []
        for j, k in enumerate(steps[1:], start=1):
            while len(toks) < k:
                toks.append(s.decode_one())
            assert rel_err(h0[j], s.hidden()) <= 1e-4, k
        assert t0 == toks
    finally:
        s.close()

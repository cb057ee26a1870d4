"""Tensor-parallel bookkeeping without a GPU: the shard plan the library computes from a
package manifest (xq_tp_plan) covers every head, intermediate row and vocabulary row exactly
once across the ranks (kv heads are shared when there are more ranks than kv heads), and the
cross-rank argmax rule (xq_tp_argmax_combine) keeps the reference's tie rule (the first maximum
wins, gemvW4A16ArgmaxNeon, xq_gemv_w4a16_neon.cpp:315-318). A gloo world-size-2 run exchanges
the plans and the per-shard (max, index) pairs between two processes as the NCCL path does."""
import json
import os
import socket

import numpy as np
import pytest

from conftest import PKG

DIMS_9B = {"format": "xqwen35_custom_w4a16", "hidden_size": 4096, "intermediate_size": 12288, "vocab_size": 248320,
           "num_hidden_layers": 32, "num_attention_heads": 16, "num_key_value_heads": 4, "head_dim": 256,
           "linear_key_head_dim": 128, "linear_value_head_dim": 128, "linear_num_key_heads": 16,
           "linear_num_value_heads": 32, "linear_conv_kernel_dim": 4, "rms_norm_eps": 0.000001,
           "rope_theta": 10000000, "partial_rotary_factor": 0.25}


def manifest_dir(tmp_path, **over):
    d = dict(DIMS_9B)
    d.update(over)
    p = tmp_path / "pkg"
    p.mkdir(exist_ok=True)
    (p / "xqwen35_manifest.json").write_text(json.dumps(d))
    return str(p)


def covered(plans, key, total):
    seen = np.zeros(total, np.int64)
    for p in plans:
        a, b = p[key]
        assert 0 <= a < b <= total
        seen[a:b] += 1
    return seen


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_plan_covers_every_shard_once(tmp_path, world):
    d = manifest_dir(tmp_path)
    plans = [PKG.tp_plan(d, world, r) for r in range(world)]
    for key, total in (("q_heads", 16), ("k_heads", 16), ("v_heads", 32), ("inter", 12288), ("vocab", 248320)):
        assert np.all(covered(plans, key, total) == 1), key
    kv = covered(plans, "kv_heads", 4)
    assert np.all(kv == max(1, world // 4))  # world 8: each kv head on the two ranks of its query heads
    for p in plans:  # a rank's query heads attend only to its kv heads
        group = 16 // 4
        assert p["q_heads"][0] // group >= p["kv_heads"][0] and (p["q_heads"][1] - 1) // group < p["kv_heads"][1]
        # DeltaNet: value head v uses key head v // 2
        assert p["v_heads"][0] // 2 == p["k_heads"][0] and p["v_heads"][1] // 2 == p["k_heads"][1]


def test_plan_rejects_uneven_splits(tmp_path):
    d = manifest_dir(tmp_path)
    for world, rank in ((3, 0), (16, 0), (2, 2), (0, 0)):
        with pytest.raises(ValueError):
            PKG.tp_plan(d, world, rank)
    with pytest.raises(ValueError):  # down's K slice 4608 / 2 = 2304 is not a multiple of 512
        PKG.tp_plan(manifest_dir(tmp_path, intermediate_size=4096 + 512), 2, 0)


def test_argmax_combine_rule():
    assert PKG.tp_argmax_combine([1.0, 3.0, 3.0], [5, 9, 2]) == 2      # equal maxima: the lowest index
    assert PKG.tp_argmax_combine([np.nan, 0.5], [0, 7]) == 7           # NaN never wins
    assert PKG.tp_argmax_combine([-np.inf, -np.inf], [4, 3]) == 3
    assert PKG.tp_argmax_combine([2.0], [11]) == 11


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _gloo_rank(rank, world, port, d, logits, q):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        plan = PKG.tp_plan(d, world, rank)
        t0, t1 = plan["vocab"]
        shard = logits[t0:t1]
        # this rank's (max, lowest index), offset to the global vocabulary, as the kernel does
        k = int(np.argmax(shard))
        pair = torch.tensor([float(shard[k]), float(t0 + k)], dtype=torch.float64)
        pairs = [torch.zeros(2, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(pairs, pair)
        plans = [None] * world
        dist.all_gather_object(plans, plan)
        vals = np.array([p[0].item() for p in pairs], np.float32)
        idx = np.array([int(p[1].item()) for p in pairs], np.int32)
        q.put((rank, PKG.tp_argmax_combine(vals, idx), plans))
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks_exchange_plan_and_argmax(tmp_path):
    import torch.multiprocessing as mp

    d = manifest_dir(tmp_path)
    rng = np.random.default_rng(3)
    logits = rng.standard_normal(248320).astype(np.float32)
    top = float(logits.max()) + 1.0
    logits[124159] = top  # the last row of rank 0's shard ...
    logits[124160] = top  # ... ties with the first row of rank 1's: rank 0's (lower) index wins
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_rank, args=(r, 2, port, d, logits, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, token, plans in got:
        assert token == 124159 == int(np.argmax(logits))
        assert [p["vocab"] for p in plans] == [[0, 124160], [124160, 248320]]

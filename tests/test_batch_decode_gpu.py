"""Batched decode (xq_batch_*): B independent sequences share one weight pass per step (tcgen05
GEMMs with the sequences' tokens as rows) but keep their own DeltaNet state, KV cache and
position. Every sequence must follow its own single-session run (xq_session: prefill then
xq_decode_one, the reference's order custom_model.cpp:1340-1356): the same greedy tokens, and
the post-final-norm hidden state within 2e-4 of the session's (the batched GEMMs use split-bf16
operands, about 2^-16 relative per product, where the session's decode path is exact-integer
plus fp32). Prompts of different lengths put the sequences at different positions."""
import numpy as np
import pytest

from conftest import PKG, package, rel_err

pytestmark = pytest.mark.gpu


def session_run(d, ids, steps, kv_fp16=False):
    s = PKG.Session(d, device=0, kv_fp16=kv_fp16)
    try:
        s.prefill(ids)
        toks = [s.decode_one() for _ in range(steps)]
        return toks, s.hidden()
    finally:
        s.close()


@pytest.mark.parametrize("kv_fp16", [False, True])
def test_batch_matches_single_sessions(small_pkg, kv_fp16):
    rng = np.random.default_rng(3)
    lens = [5, 17, 40, 9]
    prompts = [rng.integers(0, 4096, n).astype(np.int32) for n in lens]
    steps = 6
    b = PKG.Batch(small_pkg, batch=len(lens), max_context=64, kv_fp16=kv_fp16)
    try:
        for i, p in enumerate(prompts):
            b.prefill(i, p)
        toks = np.stack([b.decode() for _ in range(steps)])  # [steps][B]
        for i, p in enumerate(prompts):
            want_t, want_h = session_run(small_pkg, p, steps, kv_fp16)
            assert list(toks[:, i]) == want_t, i
            assert rel_err(b.hidden(i), want_h) <= (1e-3 if kv_fp16 else 2e-4), i
    finally:
        b.close()


def test_batch_timed_steps_and_not_ready(small_pkg):
    b = PKG.Batch(small_pkg, batch=3, max_context=64)
    try:
        b.prefill(0, np.arange(7, dtype=np.int32))
        with pytest.raises(RuntimeError) as e:
            b.decode()
        assert str(PKG.XQ_ERR_NOT_READY) in str(e.value)
        b.prefill(1, np.arange(3, dtype=np.int32) + 11)
        b.prefill(2, np.arange(12, dtype=np.int32) + 100)
        ms, toks = b.decode_timed(5)
        assert ms > 0 and toks.shape == (5, 3)
        # sequence 1 against its session: 1 untimed capture step, then the 5 timed ones
        want_t, _ = session_run(small_pkg, np.arange(3, dtype=np.int32) + 11, 6)
        assert list(toks[:, 1]) == want_t[1:]
    finally:
        b.close()


def test_batch_cfg1_at_512_context():
    d = package("cfg1", seed=1)
    rng = np.random.default_rng(4)
    prompts = [rng.integers(0, 1024, n).astype(np.int32) for n in (512, 300)]
    b = PKG.Batch(d, batch=2, max_context=600)
    try:
        for i, p in enumerate(prompts):
            b.prefill(i, p)
        toks = np.stack([b.decode() for _ in range(3)])
        for i, p in enumerate(prompts):
            want_t, want_h = session_run(d, p, 3)
            assert list(toks[:, i]) == want_t
            assert rel_err(b.hidden(i), want_h) <= 2e-4
    finally:
        b.close()

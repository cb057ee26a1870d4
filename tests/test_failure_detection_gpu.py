"""Failure detection without a GPU fault: every wait in the persistent step kernel is bounded,
and a wait that runs out is reported, not hung.

The session is created with a short wait limit (XQ_STEP_WAIT_MS) and the test hook
XQ_TEST_STALL_LAUNCH=N, which makes the N-th step-kernel launch wait at a grid barrier for one
arrival more than there are blocks. Nothing provides it, so that wait runs out; the kernel
records the timeout in its error word, every later wait returns at once, the launch ends, and
the host reports XQ_ERR_RUNTIME (session.cpp:359-363 is the reference's runtime-failure
status). xq_reset then clears the error word and the barrier counters, and the session
decodes exactly as a clean one."""
import numpy as np
import pytest

from conftest import PKG

pytestmark = pytest.mark.gpu


def clean_run(d, ids, n):
    s = PKG.Session(d, device=0)
    try:
        s.prefill(ids)
        toks = [s.decode_one() for _ in range(n)]
        return toks, s.hidden()
    finally:
        s.close()


@pytest.mark.parametrize("api", ["decode_one", "generate", "decode_timed"])
def test_stalled_barrier_reports_runtime_error_and_session_recovers(small_pkg, monkeypatch, api):
    ids = np.random.default_rng(5).integers(0, 4096, 4).astype(np.int32)
    want_toks, want_h = clean_run(small_pkg, ids, 3)
    monkeypatch.setenv("XQ_STEP_WAIT_MS", "50")
    # launches 0..3 are the prefill below; generate's own prefill takes 4..7, its first token
    # comes from launch 8 (decode_one) and the rest from the batched launches 9, 10
    stall = {"decode_one": 4, "generate": 9, "decode_timed": 4}[api]
    monkeypatch.setenv("XQ_TEST_STALL_LAUNCH", str(stall))
    s = PKG.Session(small_pkg, device=0)
    monkeypatch.delenv("XQ_STEP_WAIT_MS")
    monkeypatch.delenv("XQ_TEST_STALL_LAUNCH")
    try:
        info = s.json("backend")
        if '"persistent_step_kernel":true' not in info.replace(" ", ""):
            pytest.skip("the step kernel does not serve this package")
        s.prefill(ids)  # launches 0 .. 3 are normal
        with pytest.raises(RuntimeError) as e:
            if api == "decode_one":
                s.decode_one()
            elif api == "generate":
                s.generate(ids, 3)
            else:
                s.decode_timed(2)
        msg = str(e.value)
        assert str(PKG.XQ_ERR_RUNTIME) in msg
        if api == "decode_one":
            assert "ran out of time" in msg
        # the session is usable again after xq_reset
        assert s.reset() == PKG.XQ_OK
        s.prefill(ids)
        toks = [s.decode_one() for _ in range(3)]
        assert toks == want_toks
        assert np.array_equal(s.hidden(), want_h)
    finally:
        s.close()

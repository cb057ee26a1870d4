"""Session snapshot / restore (xq_snapshot_*; no reference counterpart, the reference only
resets, session.cpp:505-525): restoring a saved decode state must reproduce exactly the tokens
and hidden state the session produced from that state, in the same and in another session of
the same model, for fp32 and fp16 KV caches and across KV-cache growth; buffers of another
shape or a damaged header are refused with XQ_ERR_INVALID_ARGUMENT."""
import ctypes as C

import numpy as np
import pytest

from conftest import PKG, package

pytestmark = pytest.mark.gpu


def run(s, n):
    toks = [s.decode_one() for _ in range(n)]
    return toks, s.hidden()


@pytest.mark.parametrize("kv_fp16", [False, True])
def test_restore_reproduces_decode_exactly(small_pkg, kv_fp16):
    ids = (np.arange(23, dtype=np.int32) * 37) % 997
    a = PKG.Session(small_pkg, device=0, kv_fp16=kv_fp16)
    b = PKG.Session(small_pkg, device=0, kv_fp16=kv_fp16)
    try:
        a.prefill(ids)
        snap = a.snapshot()
        t1, h1 = run(a, 6)
        # same session, back to the saved state
        assert a.restore(snap) == PKG.XQ_OK
        t2, h2 = run(a, 6)
        assert t2 == t1
        assert np.array_equal(h2, h1)
        # another session of the same model (never prefilled) continues identically
        assert b.restore(snap) == PKG.XQ_OK
        t3, h3 = run(b, 6)
        assert t3 == t1
        assert np.array_equal(h3, h1)
    finally:
        a.close()
        b.close()


def test_snapshot_after_decode_and_kv_growth(small_pkg):
    """A state taken mid-generation past the initial KV capacity (the cache grows on restore
    into a fresh session too)."""
    ids = (np.arange(40, dtype=np.int32) * 11) % 1000
    a = PKG.Session(small_pkg, device=0, max_context_tokens=48)
    b = PKG.Session(small_pkg, device=0, max_context_tokens=48)
    try:
        a.prefill(ids)
        run(a, 30)  # position 70 > initial capacity 64
        snap = a.snapshot()
        t1, h1 = run(a, 5)
        assert b.restore(snap) == PKG.XQ_OK
        t2, h2 = run(b, 5)
        assert t2 == t1 and np.array_equal(h2, h1)
    finally:
        a.close()
        b.close()


def test_snapshot_status_codes(small_pkg):
    s = PKG.Session(small_pkg, device=0)
    other = PKG.Session(package("cfg1", seed=11), device=0)
    fp16 = PKG.Session(small_pkg, device=0, kv_fp16=True)
    try:
        L = s.L
        n = C.c_size_t()
        assert L.xq_snapshot_size(s.h, C.byref(n)) == PKG.XQ_ERR_NOT_READY  # before prefill
        s.prefill(np.arange(5, dtype=np.int32))
        assert L.xq_snapshot_size(s.h, C.byref(n)) == PKG.XQ_OK and n.value > 64
        w = C.c_size_t()
        small = C.create_string_buffer(16)
        assert L.xq_snapshot_save(s.h, small, 16, C.byref(w)) == PKG.XQ_ERR_BUFFER_TOO_SMALL
        assert w.value == n.value
        snap = s.snapshot()
        assert len(snap) == n.value
        assert other.restore(snap) == PKG.XQ_ERR_INVALID_ARGUMENT  # other shape
        assert fp16.restore(snap) == PKG.XQ_ERR_INVALID_ARGUMENT  # other KV type
        bad = bytearray(snap)
        bad[0] ^= 0xFF
        assert s.restore(bytes(bad)) == PKG.XQ_ERR_INVALID_ARGUMENT  # damaged magic
        assert s.restore(snap[:-4]) == PKG.XQ_ERR_INVALID_ARGUMENT  # truncated
        assert s.restore(snap) == PKG.XQ_OK
    finally:
        s.close()
        other.close()
        fp16.close()

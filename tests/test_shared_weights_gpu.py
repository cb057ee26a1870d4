"""Sessions of one package on one device share its read-only weights (matrices, tile copy,
norms, embeddings) and nothing else: a second session reuses the first one's weights, both
decode exactly as a session alone would (bit-identical hidden states, same tokens) when their
steps interleave, and a session keeps working after the session that loaded the weights is
destroyed."""
import json
import shutil

import numpy as np
import pytest

from conftest import PKG, package

pytestmark = pytest.mark.gpu


def info(s):
    return json.loads(s.json("backend"))


def alone(d, ids, n):
    s = PKG.Session(d, device=0)
    try:
        s.prefill(ids)
        toks = [s.decode_one() for _ in range(n)]
        return toks, s.hidden()
    finally:
        s.close()


def test_sessions_share_weights_and_nothing_else(tmp_path):
    d = str(tmp_path / "pkg")
    shutil.copytree(package("small", seed=7), d)  # a path no other live session uses
    ids1 = (np.arange(11, dtype=np.int32) * 17) % 4000
    ids2 = (np.arange(7, dtype=np.int32) * 29 + 3) % 4000
    ref1, h1 = alone(d, ids1, 6)
    ref2, h2 = alone(d, ids2, 8)

    a = PKG.Session(d, device=0)
    b = PKG.Session(d, device=0)
    try:
        ia, ib = info(a), info(b)
        assert not ia["weights_reused"] and ib["weights_reused"]
        assert ib["weights_users"] == 2
        a.prefill(ids1)
        b.prefill(ids2)
        ta, tb = [], []
        for _ in range(4):  # interleaved steps on the shared weights
            ta.append(a.decode_one())
            tb.append(b.decode_one())
        ta += [a.decode_one(), a.decode_one()]
        assert ta == ref1 and np.array_equal(a.hidden(), h1)
        a.close()  # the session that loaded the weights goes away
        assert info(b)["weights_users"] == 1
        tb += [b.decode_one() for _ in range(4)]
        assert tb == ref2 and np.array_equal(b.hidden(), h2)
    finally:
        a.close()
        b.close()
    c = PKG.Session(d, device=0)  # nobody holds them any more: loaded afresh
    try:
        assert not info(c)["weights_reused"]
    finally:
        c.close()

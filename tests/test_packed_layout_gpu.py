"""Loading the packed B200 layout (b200/*.b200 written by xq_pack_b200_layout) gives the same
device weights as re-tiling the xq4 files: prefill hidden state and greedy tokens are
bit-identical, on the symmetric (fp16 scale) and the affine (scale, offset) layouts; a packed
matrix that disagrees with the manifest is refused with XQ_ERR_MODEL."""
import ctypes as C
import json
import os
import shutil
import struct

import numpy as np
import pytest

from conftest import PKG, package

pytestmark = pytest.mark.gpu


def decode(d, ids, n):
    s = PKG.Session(d, device=0)
    try:
        info = json.loads(s.json("backend"))
        s.prefill(ids)
        h0 = s.hidden()
        toks = [s.decode_one() for _ in range(n)]
        return info["packed_layout"], h0, toks, s.hidden()
    finally:
        s.close()


@pytest.mark.parametrize("quant", ["sym", "asym"])
def test_packed_layout_loads_identically(tmp_path, quant):
    src = package("small", seed=7, quant=quant)
    d = str(tmp_path / "pkg")
    shutil.copytree(src, d)
    PKG.pack_b200(d)
    ids = (np.arange(17, dtype=np.int32) * 13) % 900
    p0, h0, t0, e0 = decode(src, ids, 6)
    p1, h1, t1, e1 = decode(d, ids, 6)
    assert not p0 and p1
    assert np.array_equal(h0, h1) and t0 == t1 and np.array_equal(e0, e1)


def test_mismatched_packed_matrix_is_refused(tmp_path):
    src = package("small", seed=7)
    d = str(tmp_path / "pkg")
    shutil.copytree(src, d)
    PKG.pack_b200(d)
    path = os.path.join(d, "b200", "layers_0_down.b200")
    raw = bytearray(open(path, "rb").read())
    rows = struct.unpack_from("<I", raw, 16)[0]
    struct.pack_into("<I", raw, 16, rows - 1)  # header now disagrees with its size and the manifest
    open(path, "wb").write(bytes(raw))
    out = C.c_void_p()
    assert PKG.lib().xq_create(d.encode(), None, C.byref(out)) == PKG.XQ_ERR_MODEL and not out.value

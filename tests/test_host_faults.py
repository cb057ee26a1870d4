"""Package faults are reported, not run: an XQ4 file with a bad magic, a short payload, a header
whose sizes disagree with rows/cols/group, or a matrix whose shape disagrees with the manifest
gives XQ_ERR_MODEL with a message naming the file (readXq4, custom_model.cpp:218-262; the
shape checks of CustomModel::load, custom_model.cpp:455-553). The CPU tests reach the reader
through the host-only packer (xq_pack_b200_layout); the GPU tests through xq_create."""
import ctypes as C
import os
import shutil
import struct

import pytest

from conftest import PKG, package

MATRIX = "layers_0_mlp_down_proj_weight.xq4"


def corrupt(d, how):
    p = os.path.join(d, MATRIX)
    raw = bytearray(open(p, "rb").read())
    if how == "magic":
        raw[0:8] = b"NOTXQ4\0\0"
    elif how == "short":
        raw = raw[: len(raw) - 1000]
    elif how == "sizes":  # packed_bytes no longer rows * cols / 2
        off = 8 + 5 * 4
        (packed,) = struct.unpack_from("<Q", raw, off)
        struct.pack_into("<Q", raw, off, packed + 2)
    elif how == "shape":  # a valid file of the wrong shape: rows halved, payload to match
        rows, cols, group = struct.unpack_from("<3I", raw, 12)
        r2 = rows // 2
        gpr = cols // group
        head = bytearray(raw[:52])  # magic, 5 x u32, 3 x u64 (custom_model.cpp:218-262)
        struct.pack_into("<I", head, 12, r2)
        struct.pack_into("<3Q", head, 28, r2 * cols // 2, r2 * gpr, r2 * gpr)
        p0 = 52
        packed = raw[p0:p0 + r2 * cols // 2]
        s0 = p0 + rows * cols // 2
        scales = raw[s0:s0 + 4 * r2 * gpr]
        z0 = s0 + 4 * rows * gpr
        zeros = raw[z0:z0 + 4 * r2 * gpr]
        raw = head + packed + scales + zeros
    open(p, "wb").write(bytes(raw))


EXPECT = {"magic": b"bad xq4 magic", "short": b"short xq4 payload", "sizes": b"inconsistent xq4 sizes",
          "shape": b"unexpected shape"}


def broken_copy(tmp_path, how):
    d = str(tmp_path / f"broken_{how}")
    shutil.copytree(package("small", seed=7), d)
    corrupt(d, how)
    return d


@pytest.mark.parametrize("how", sorted(EXPECT))
def test_packer_rejects_corrupt_xq4(tmp_path, how):
    d = broken_copy(tmp_path, how)
    err = C.create_string_buffer(512)
    assert PKG.lib().xq_pack_b200_layout(d.encode(), err, len(err)) == PKG.XQ_ERR_MODEL
    assert EXPECT[how] in err.value, err.value
    assert (b"down" if how == "shape" else MATRIX.encode()) in err.value
    assert not os.path.exists(os.path.join(d, "b200", "layout.json"))


@pytest.mark.gpu
@pytest.mark.parametrize("how", sorted(EXPECT))
def test_create_rejects_corrupt_xq4(tmp_path, how):
    d = broken_copy(tmp_path, how)
    with pytest.raises(RuntimeError) as e:
        PKG.Session(d, device=0)
    assert f"failed: {PKG.XQ_ERR_MODEL}" in str(e.value)
    assert EXPECT[how].decode() in str(e.value)


@pytest.mark.gpu
def test_create_rejects_missing_embeddings(tmp_path):
    d = str(tmp_path / "no_emb")
    shutil.copytree(package("small", seed=7), d)
    os.remove(os.path.join(d, "embeddings_bf16.bin"))
    with pytest.raises(RuntimeError) as e:
        PKG.Session(d, device=0)
    assert "embeddings_bf16.bin" in str(e.value)

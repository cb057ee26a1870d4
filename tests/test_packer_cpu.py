"""The packed B200 weight layout (xq_pack_b200_layout; host only): every fused matrix of a
package is written in the kernels' row layout, and decoding those rows gives back exactly the
xq4 sources (nibbles byte for byte, symmetric scales as the fp16 they equal, affine scales and
offsets as float pairs), with gate/up rows interleaved and the in_proj parts concatenated in
the loader's order."""
import json
import os
import shutil
import struct

import numpy as np
import pytest

from conftest import PKG, package, synthetic

HEADER = struct.Struct("<8s8IQ16s")  # magic, version, kind, rows, cols, group, xq4 version, stride, meta, bytes


def read_b200(path):
    with open(path, "rb") as f:
        raw = f.read()
    magic, ver, kind, rows, cols, group, xver, stride, meta, nbytes, _res = HEADER.unpack(raw[:64])
    assert magic == b"XQB200\0\0" and ver == 1
    body = np.frombuffer(raw[64:], np.uint8)
    assert body.size == nbytes == rows * stride
    return dict(kind=kind, rows=rows, cols=cols, group=group, stride=stride, meta=meta,
                rows_bytes=body.reshape(rows, stride))


def expected_rows(parts, interleave):
    """The loader's row order: parts concatenated, or gate/up pairs interleaved."""
    if interleave:
        a, b = parts
        out = []
        for r in range(a["rows"]):
            out += [(a, r), (b, r)]
        return out
    return [(p, r) for p in parts for r in range(p["rows"])]


def check_matrix(path, sources, interleave):
    m = read_b200(path)
    parts = [synthetic.read_xq4(s) for s in sources]
    K, gpr = m["cols"], m["cols"] // 64
    sym = all(p["version"] == 1 and np.all(p["zeros"] == 8.0) for p in parts)
    assert m["kind"] == (0 if sym else 1) and m["meta"] == K // 2
    assert m["stride"] == K // 2 + (2 if sym else 8) * gpr
    rows = expected_rows(parts, interleave)
    assert m["rows"] == len(rows)
    for i, (p, r) in enumerate(rows):
        got = m["rows_bytes"][i]
        assert np.array_equal(got[:K // 2], p["packed"][r])
        sc = p["scales"][r * gpr:(r + 1) * gpr]
        if sym:
            assert np.array_equal(got[K // 2:].view("<f2").astype(np.float32), sc)
        else:
            pair = got[K // 2:].view("<f4").reshape(gpr, 2)
            z = p["zeros"][r * gpr:(r + 1) * gpr]
            off = z if p["version"] == 2 else (-z * sc).astype(np.float32)
            assert np.array_equal(pair[:, 0], sc) and np.array_equal(pair[:, 1], off)


@pytest.mark.parametrize("quant", ["sym", "asym"])
def test_packed_rows_decode_to_the_xq4_sources(tmp_path, quant):
    src = package("small", seed=7, quant=quant)
    d = str(tmp_path / "pkg")
    shutil.copytree(src, d)
    PKG.pack_b200(d)
    layout = json.load(open(os.path.join(d, "b200", "layout.json")))
    assert layout["format"] == "xq_b200_rows" and layout["version"] == 1
    check_matrix(os.path.join(d, "b200", "lm_head.b200"), [os.path.join(d, "lm_head_weight.xq4")], False)
    man = json.load(open(os.path.join(d, "xqwen35_manifest.json")))
    n_layers = sum(1 for f in os.listdir(d) if f.endswith("input_layernorm_weight.f32"))
    assert layout["matrices"] == 1 + 4 * n_layers
    for i in range(n_layers):
        p = os.path.join(d, f"layers_{i}_")
        b = os.path.join(d, "b200", f"layers_{i}_")
        check_matrix(b + "gate_up.b200", [p + "mlp_gate_proj_weight.xq4", p + "mlp_up_proj_weight.xq4"], True)
        check_matrix(b + "down.b200", [p + "mlp_down_proj_weight.xq4"], False)
        if os.path.exists(p + "self_attn_q_proj_weight.xq4"):
            check_matrix(b + "in_proj.b200", [p + f"self_attn_{n}_proj_weight.xq4" for n in "qkv"], False)
            check_matrix(b + "out_proj.b200", [p + "self_attn_o_proj_weight.xq4"], False)
        else:
            check_matrix(b + "in_proj.b200", [p + f"linear_attn_in_proj_{n}_weight.xq4" for n in ("qkv", "z", "a", "b")],
                         False)
            check_matrix(b + "out_proj.b200", [p + "linear_attn_out_proj_weight.xq4"], False)
    assert man  # the reference's manifest is left untouched


def test_packer_reports_package_problems(tmp_path):
    import ctypes as C

    L = PKG.lib()
    err = C.create_string_buffer(256)
    assert L.xq_pack_b200_layout(None, err, len(err)) == PKG.XQ_ERR_INVALID_ARGUMENT
    assert L.xq_pack_b200_layout(str(tmp_path).encode(), err, len(err)) == PKG.XQ_ERR_MODEL
    assert b"manifest" in err.value
    src = package("small", seed=7)
    d = str(tmp_path / "broken")
    shutil.copytree(src, d)
    os.remove(os.path.join(d, "layers_0_mlp_down_proj_weight.xq4"))
    assert L.xq_pack_b200_layout(d.encode(), err, len(err)) == PKG.XQ_ERR_MODEL
    assert not os.path.exists(os.path.join(d, "b200", "layout.json"))

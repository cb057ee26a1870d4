"""W4A16 GEMV on the GPU through the kernel C ABI vs the oracle / reference golden outputs.

Tolerance: max |y - y_ref| / max |y_ref| <= 1e-5 (fp32 accumulation; the north-star bar is
1e-3). argmax indices must match exactly, ties to the lowest index."""
import os

import numpy as np
import pytest

from conftest import GOLDEN, PKG, rel_err

pytestmark = pytest.mark.gpu
K = np.load(os.path.join(GOLDEN, "kernel_cases.npz"))
TOL = 1e-5


def _torch():
    import torch

    return torch


def run_gemv(m, x):
    torch = _torch()
    xd = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    yd = torch.zeros(m.rows, dtype=torch.float32, device="cuda")
    m.gemv(xd.data_ptr(), yd.data_ptr())
    torch.cuda.synchronize()
    return yd.cpu().numpy()


def seeded(rows, cols, quant, seed=0, group=64):
    rng = np.random.default_rng(seed)
    packed = rng.integers(0, 256, size=rows * ((cols + 1) // 2), dtype=np.uint8)
    n = rows * ((cols + group - 1) // group)
    s = (np.abs(rng.standard_normal(n)) * 0.02).astype(np.float32)
    if quant == "sym":
        s = s.astype(np.float16).astype(np.float32)
        z, version = np.full(n, 8.0, np.float32), 1
    elif quant == "asym":
        z, version = rng.integers(0, 16, n).astype(np.float32), 1
    else:
        z, version = (rng.standard_normal(n) * 0.1).astype(np.float32), 2
    x = rng.standard_normal(cols).astype(np.float32)
    return packed, s, z, version, x


def test_golden_sym_gemv():
    m = PKG.Matrix(K["sym_packed"], K["sym_scales"], K["sym_zeros"], 1024, 2048, 64)
    assert m.info()["fast"] and m.info()["kind"] == 0
    assert rel_err(run_gemv(m, K["sym_x"]), K["sym_y"]) <= TOL


@pytest.mark.parametrize("rows,cols,quant", [(12288, 4096, "sym"), (4096, 12288, "sym"), (1000, 4096, "asym"),
                                             (514, 4096, "v2"), (248, 2048, "sym"), (3, 1024, "asym")])
def test_gemv_vs_oracle(oracle, rows, cols, quant):
    packed, s, z, version, x = seeded(rows, cols, quant, seed=rows)
    m = PKG.Matrix(packed, s, z, rows, cols, 64, version)
    assert m.info()["fast"]
    ref = oracle.port_gemv(oracle.Matrix(rows, cols, 64, version, packed, s, z), x)
    assert rel_err(run_gemv(m, x), ref) <= TOL


def test_generic_layout_kat_group8():
    m = PKG.Matrix(K["kat_packed"], K["kat_scales"], K["kat_zeros"], 7, 24, 8)
    assert not m.info()["fast"]
    assert np.abs(run_gemv(m, K["kat_x"]) - K["kat_y"]).max() <= 1e-5


def test_generic_layout_affine_v2_kat():
    m = PKG.Matrix(K["v2_packed"], K["v2_scales"], K["v2_zeros"], 2, 4, 4, 2)
    assert np.abs(run_gemv(m, K["v2_x"]) - K["v2_y"]).max() <= 1e-6


def test_host_buffer_entry_point():
    packed, s, z, version, x = seeded(12288, 4096, "sym", seed=1)
    m = PKG.Matrix(packed, s, z, 12288, 4096, 64, version)
    assert np.array_equal(m.gemv_host(x), run_gemv(m, x))


def run_argmax(m, x):
    torch = _torch()
    xd = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    idx = torch.zeros(1, dtype=torch.int32, device="cuda")
    val = torch.zeros(1, dtype=torch.float32, device="cuda")
    m.argmax(xd.data_ptr(), idx.data_ptr(), val.data_ptr())
    torch.cuda.synchronize()
    return int(idx.item()), float(val.item())


def test_argmax_golden():
    m = PKG.Matrix(K["sym_packed"], K["sym_scales"], K["sym_zeros"], 1024, 2048, 64)
    i, v = run_argmax(m, K["sym_x"])
    assert i == int(K["sym_argmax"][0])
    assert abs(v - float(K["sym_argmax_value"][0])) <= TOL * abs(v)


@pytest.mark.parametrize("rows", [248320, 4097])
def test_argmax_matches_oracle_and_ties(oracle, rows):
    packed, s, z, version, x = seeded(rows, 4096, "sym", seed=9)
    p = packed.reshape(rows, -1)
    s2 = s.reshape(rows, -1)
    best = int(np.argmax(oracle.port_gemv(oracle.Matrix(rows, 4096, 64, 1, packed, s, z), x)))
    hi = rows - 3
    p[hi] = p[best]
    s2[hi] = s2[best]  # identical row later in the matrix: the tie goes to the lower index
    p[best // 2] = p[best]
    s2[best // 2] = s2[best]
    m = PKG.Matrix(p.reshape(-1), s2.reshape(-1), z, rows, 4096, 64)
    i, _ = run_argmax(m, x)
    oi, _ = oracle.port_argmax(oracle.Matrix(rows, 4096, 64, 1, p.reshape(-1), s2.reshape(-1), z), x)
    assert i == oi == best // 2


def test_nan_input_propagates():
    packed, s, z, version, x = seeded(256, 4096, "sym", seed=2)
    x[17] = np.nan
    m = PKG.Matrix(packed, s, z, 256, 4096, 64)
    assert np.isnan(run_gemv(m, x)).all()


def run_gemv_mma(m, x):
    torch = _torch()
    xd = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    yd = torch.full((m.rows,), float("nan"), dtype=torch.float32, device="cuda")
    m.gemv_mma(xd.data_ptr(), yd.data_ptr())
    torch.cuda.synchronize()
    return yd.cpu().numpy()


@pytest.mark.parametrize("rows,cols", [(24576, 4096), (4096, 12288), (1000, 4096), (7, 512), (333, 1024)])
def test_tensor_core_gemv_vs_oracle(oracle, rows, cols):
    """The mma.sync tile-layout GEMV: every row written (ragged last tile), within the fp32 bar."""
    packed, s, z, version, x = seeded(rows, cols, "sym", seed=rows + 5)
    x[::7] *= 1e-3  # small and large values in one group
    m = PKG.Matrix(packed, s, z, rows, cols, 64, version)
    ref = oracle.port_gemv(oracle.Matrix(rows, cols, 64, version, packed, s, z), x)
    y = run_gemv_mma(m, x)
    assert np.all(np.isfinite(y))
    assert rel_err(y, ref) <= TOL
    assert rel_err(y, run_gemv(m, x)) <= TOL


def test_tensor_core_gemv_refuses_other_layouts():
    packed, s, z, version, x = seeded(64, 4096, "asym", seed=3)
    m = PKG.Matrix(packed, s, z, 64, 4096, 64, version)
    torch = _torch()
    xd = torch.zeros(4096, device="cuda")
    yd = torch.zeros(64, device="cuda")
    with pytest.raises(RuntimeError):
        m.gemv_mma(xd.data_ptr(), yd.data_ptr())


def test_tensor_core_gemv_nan_input_propagates():
    packed, s, z, version, x = seeded(256, 4096, "sym", seed=2)
    x[17] = np.nan
    m = PKG.Matrix(packed, s, z, 256, 4096, 64)
    torch = _torch()
    xd = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    yd = torch.zeros(256, dtype=torch.float32, device="cuda")
    m.gemv_mma(xd.data_ptr(), yd.data_ptr())
    torch.cuda.synchronize()
    assert np.isnan(yd.cpu().numpy()).all()


def test_config0_fp16_gemv_vs_oracle(oracle):
    """Config 0 as specified: W [12288 x 4096] int4 g64 symmetric, x fp16 ~ N(0, 1), y fp16 with
    fp32 accumulation. The oracle runs the reference algorithm in fp32 on the same fp16 x; the
    only extra error is y's final rounding to fp16 (relative 2^-11 per element), so the bar is
    the fp32 bar plus that rounding: |y - y_ref| <= 1e-5 * max|y_ref| + 2^-11 * |y_ref|."""
    torch = _torch()
    rows, cols = 12288, 4096
    packed, s, z, version, _ = seeded(rows, cols, "sym", seed=12288)
    x16 = np.random.default_rng(0).standard_normal(cols).astype(np.float16)
    m = PKG.Matrix(packed, s, z, rows, cols, 64, version)
    ref = oracle.port_gemv(oracle.Matrix(rows, cols, 64, version, packed, s, z), x16.astype(np.float32))
    xd = torch.from_numpy(x16).cuda()
    for _ in range(2):  # twice: the second launch overlaps nothing but must agree as well
        yd = torch.full((rows,), float("nan"), dtype=torch.float16, device="cuda")
        m.gemv_mma_f16(xd.data_ptr(), yd.data_ptr())
        torch.cuda.synchronize()
        y = yd.cpu().numpy().astype(np.float32)
        assert np.all(np.isfinite(y))
        bound = 1e-5 * np.abs(ref).max() + 2.0 ** -11 * np.abs(ref)
        assert np.all(np.abs(y - ref) <= bound)

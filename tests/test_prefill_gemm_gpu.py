"""The batched-prefill W4A16 GEMM on tcgen05 / TMEM (xqk_prefill_gemm_w4a16) against a float64
reference of the same operands.

* One bf16 pass (config 3 as specified: activations bf16, int4 weights dequantised to bf16 in
  shared memory): the reference multiplies the same bf16 X by W rounded to bf16 once
  (bf16((code - 8) * scale)), so only the fp32 accumulation differs: max error <= 2e-5 of
  max |Y|. At M <= 64 tokens the small-M kernel multiplies the exact codes and scales each
  group's partial sum, so its reference is the same bf16 X times the exact W.
* Split mode (X = X_hi + X_lo and W = W_hi + W_lo as bf16 pairs, three products): against the
  exact product of the fp32 X and the exact int4 weights, max error <= 1e-4 of max |Y| (the
  dropped terms are about 2^-16 relative).
Ragged shapes cover partial 128-row weight tiles and partial token tiles; the add mode and the
bf16 output are checked too. The small-M cases cover every token tile (16 / 32 / 64) and the
split-K cluster sizes the launcher picks for these shapes (1, 3, 4 and 8 CTAs per row tile), and
check that two runs give bit-identical results (the cluster reduction has a fixed order)."""
import numpy as np
import pytest

from conftest import PKG

pytestmark = pytest.mark.gpu


def _torch():
    import torch

    return torch


def sym_matrix(rows, cols, seed):
    rng = np.random.default_rng(seed)
    codes = rng.integers(0, 16, size=(rows, cols), dtype=np.uint8)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8).reshape(-1)
    s = (np.abs(rng.standard_normal(rows * (cols // 64))) * 0.02).astype(np.float16).astype(np.float32)
    w = (codes.astype(np.float32) - 8.0) * np.repeat(s.reshape(rows, cols // 64), 64, axis=1)
    m = PKG.Matrix(packed, s, np.full(s.size, 8.0, np.float32), rows, cols, 64)
    return m, w


def run(m, x_hi, x_lo, n, ldy, out_kind=0, y0=None):
    torch = _torch()
    if out_kind == 2:
        y = torch.zeros((n, ldy), dtype=torch.bfloat16, device="cuda")
    else:
        y = torch.full((n, ldy), float("nan"), dtype=torch.float32, device="cuda") if y0 is None else y0.clone()
    m.prefill_gemm(x_hi.data_ptr(), x_lo.data_ptr() if x_lo is not None else None, n, y.data_ptr(), ldy, out_kind)
    torch.cuda.synchronize()
    return y.float().cpu().numpy()


def max_rel(y, ref):
    return float(np.abs(y - ref).max() / np.abs(ref).max())


@pytest.mark.parametrize("rows,cols,n", [(256, 1024, 40), (333, 1024, 300), (12288, 4096, 512), (4096, 12288, 512),
                                         (128, 1024, 1), (1000, 4096, 257)])
def test_one_pass_bf16_vs_reference(rows, cols, n):
    torch = _torch()
    m, w = sym_matrix(rows, cols, seed=rows + cols)
    x = torch.randn((n, cols), device="cuda").to(torch.bfloat16)
    y = run(m, x, None, n, rows)
    wb = w.astype(np.float64) if n <= 64 else torch.from_numpy(w).to(torch.bfloat16).double().numpy()
    ref = x.double().cpu().numpy() @ wb.T
    assert np.all(np.isfinite(y))
    assert max_rel(y, ref) <= 2e-5


@pytest.mark.parametrize("rows,cols,n", [(256, 2048, 40), (333, 1024, 300), (4096, 12288, 130), (12352, 4096, 64)])
def test_split_mode_vs_exact(rows, cols, n):
    torch = _torch()
    m, w = sym_matrix(rows, cols, seed=rows * 3 + cols)
    x32 = torch.randn((n, cols), device="cuda") * 3.0
    x_hi = x32.to(torch.bfloat16)
    x_lo = (x32 - x_hi.float()).to(torch.bfloat16)
    y = run(m, x_hi, x_lo, n, rows)
    ref = x32.double().cpu().numpy() @ w.astype(np.float64).T
    assert np.all(np.isfinite(y))
    assert max_rel(y, ref) <= 1e-4


def test_add_mode_and_bf16_output_and_row_stride():
    torch = _torch()
    rows, cols, n, ldy = 384, 1024, 70, 400  # ldy > rows: padding columns untouched
    m, w = sym_matrix(rows, cols, seed=9)
    x = torch.randn((n, cols), device="cuda").to(torch.bfloat16)
    wb = torch.from_numpy(w).to(torch.bfloat16).double().numpy()
    ref = x.double().cpu().numpy() @ wb.T
    y0 = torch.randn((n, ldy), device="cuda")
    y = run(m, x, None, n, ldy, out_kind=1, y0=y0)
    base = y0.cpu().numpy()
    assert max_rel(y[:, :rows] - base[:, :rows], ref) <= 5e-5
    assert np.array_equal(y[:, rows:], base[:, rows:])
    yb = run(m, x, None, n, rows, out_kind=2)
    assert max_rel(yb, ref) <= 8e-3  # bf16 output rounding


@pytest.mark.parametrize("rows,cols,n", [(4096, 4096, 8), (4096, 12288, 64), (12288, 4096, 16), (512, 4096, 33),
                                         (333, 1024, 5), (1000, 2048, 1), (12352, 4096, 64), (4096, 4096, 17)])
def test_small_m_split_and_one_pass_vs_exact(rows, cols, n):
    torch = _torch()
    m, w = sym_matrix(rows, cols, seed=rows * 7 + cols + n)
    x32 = torch.randn((n, cols), device="cuda") * 2.0
    x_hi = x32.to(torch.bfloat16)
    x_lo = (x32 - x_hi.float()).to(torch.bfloat16)
    y = run(m, x_hi, x_lo, n, rows)
    ref = x32.double().cpu().numpy() @ w.astype(np.float64).T
    assert np.all(np.isfinite(y))
    assert max_rel(y, ref) <= 2e-5
    assert np.array_equal(y, run(m, x_hi, x_lo, n, rows))  # fixed reduction order
    y1 = run(m, x_hi, None, n, rows)
    ref1 = x_hi.double().cpu().numpy() @ w.astype(np.float64).T
    assert max_rel(y1, ref1) <= 2e-5


def test_small_m_add_mode_bf16_output_and_row_stride():
    torch = _torch()
    rows, cols, n, ldy = 4000, 4096, 9, 4100  # split-K cluster, partial last row tile, padded rows
    m, w = sym_matrix(rows, cols, seed=11)
    x = torch.randn((n, cols), device="cuda").to(torch.bfloat16)
    ref = x.double().cpu().numpy() @ w.astype(np.float64).T
    y0 = torch.randn((n, ldy), device="cuda")
    y = run(m, x, None, n, ldy, out_kind=1, y0=y0)
    base = y0.cpu().numpy()
    assert max_rel(y[:, :rows] - base[:, :rows], ref) <= 5e-5
    assert np.array_equal(y[:, rows:], base[:, rows:])
    yb = run(m, x, None, n, rows, out_kind=2)
    assert max_rel(yb, ref) <= 8e-3

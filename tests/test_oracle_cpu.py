"""Pins the oracle restatement (oracle/xq_oracle.c) to the reference: bit-exact against the
golden outputs the compiled reference produced (tests/golden/make_golden.py) and, where the
reference library is present, against live reference runs on further seeds and formats."""
import os

import numpy as np
import pytest

from conftest import GOLDEN, ORACLE, package, rel_err

K = np.load(os.path.join(GOLDEN, "kernel_cases.npz"))


def test_gemv_sym_bit_exact_vs_reference_golden(oracle):
    m = oracle.Matrix(1024, 2048, 64, 1, K["sym_packed"], K["sym_scales"], K["sym_zeros"])
    assert np.array_equal(oracle.port_gemv(m, K["sym_x"]), K["sym_y"])


def test_argmax_vs_reference_golden(oracle):
    m = oracle.Matrix(1024, 2048, 64, 1, K["sym_packed"], K["sym_scales"], K["sym_zeros"])
    idx, val = oracle.port_argmax(m, K["sym_x"])
    assert idx == int(K["sym_argmax"][0]) and np.float32(val) == K["sym_argmax_value"][0]


def test_kat_quantized_gemv_group8(oracle):
    # test_kernels.cpp:19-48: 7 x 24, group 8, asymmetric quantizeLowBit, tol 1e-5 vs dense.
    m = oracle.Matrix(7, 24, 8, 1, K["kat_packed"], K["kat_scales"], K["kat_zeros"])
    y = oracle.port_gemv(m, K["kat_x"])
    assert np.array_equal(y, K["kat_y"])
    assert np.abs(y - K["kat_dense_y"]).max() <= 1e-5


def test_kat_affine_v2(oracle):
    # test_kernels.cpp:50-77: hand-packed XQ4 v2 matrix, code * scale + zero, tol 1e-6.
    m = oracle.Matrix(2, 4, 4, 2, K["v2_packed"], K["v2_scales"], K["v2_zeros"])
    y = oracle.port_gemv(m, K["v2_x"])
    assert np.array_equal(y, K["v2_y"])
    dense = m.dequantize() @ K["v2_x"].astype(np.float64)
    assert np.abs(y - dense).max() <= 1e-6


def test_kat_rmsnorm(oracle):
    y = np.zeros(16, np.float32)
    oracle.port().xo_rmsnorm(K["rms_x"], K["rms_w"], 16, np.float32(1e-6), y)
    assert np.array_equal(y, K["rms_y"])


def test_kat_gated_delta_two_steps(oracle):
    # test_kernels.cpp:234-325 with A_log = -2.65625, dt_bias = -3.53125.
    L = oracle.port()
    state = np.zeros(6, np.float32)
    for s in range(2):
        beta = L.xo_sigmoid(np.float32(K["delta_b"][s]))
        gate = -np.exp(np.float32(-2.65625)) * L.xo_softplus(np.float32(K["delta_a"][s] + np.float32(-3.53125)))
        o = np.zeros(2, np.float32)
        L.xo_gated_delta_decode(np.ascontiguousarray(K["delta_q"][s]), np.ascontiguousarray(K["delta_k"][s]),
                                np.ascontiguousarray(K["delta_v"][s]), np.float32(beta), np.float32(gate), 3, 2,
                                state, o)
        assert np.array_equal(o, K["delta_out"][s])
    assert np.array_equal(state, K["delta_state"])


def test_kat_gqa_attention(oracle):
    # test_kernels.cpp:141-196; the runtime's attention (custom_model.cpp:871-928) normalises
    # probabilities before the V sum, attentionDecodeReference divides inside it: equal to 1e-6.
    o = np.zeros(12, np.float32)
    oracle.port().xo_attention_decode(K["attn_q"], K["attn_k"], K["attn_v"], 4, 2, 4, 3, o)
    assert np.abs(o - K["attn_out"]).max() <= 1e-6


def test_model_small_bit_exact_vs_reference_golden(oracle):
    g = np.load(os.path.join(GOLDEN, "model_small_s7.npz"))
    d = package("small", seed=7)
    p = oracle.PortModel(d)
    p.prefill(g["ids"])
    assert np.array_equal(p.hidden(), g["hidden_prefill"])
    toks = [p.decode_one() for _ in range(len(g["tokens"]))]
    assert toks == list(g["tokens"])
    assert np.array_equal(p.hidden(), g["hidden_after"])
    assert p.position == len(g["ids"]) + len(g["tokens"])


@pytest.mark.skipif(not ORACLE.ref_available(), reason="reference library not built here")
@pytest.mark.parametrize("quant", ["asym", "v2"])
def test_model_small_live_reference(oracle, quant):
    d = package("small", seed=3, quant=quant)
    ids = np.random.default_rng(3).integers(-5000, 9000, 9).astype(np.int32)  # includes folded ids
    r = oracle.RefSession(d)
    p = oracle.PortModel(d)
    r.prefill(ids)
    p.prefill(ids)
    assert np.array_equal(r.hidden(), p.hidden())
    assert [r.decode_one() for _ in range(3)] == [p.decode_one() for _ in range(3)]
    assert np.array_equal(r.hidden(), p.hidden())


@pytest.mark.skipif(not ORACLE.ref_available(), reason="reference library not built here")
def test_gemv_v2_live_reference(oracle):
    rng = np.random.default_rng(5)
    rows, cols = 1024, 4096
    m = oracle.Matrix(rows, cols, 64, 2, rng.integers(0, 256, rows * cols // 2, dtype=np.uint8),
                      rng.random(rows * cols // 64, dtype=np.float32) * 0.02,
                      rng.standard_normal(rows * cols // 64).astype(np.float32) * 0.1)
    x = rng.standard_normal(cols).astype(np.float32)
    assert np.array_equal(oracle.port_gemv(m, x), oracle.ref_gemv(m, x))


def test_dequantize_helper_matches_gemv(oracle):
    m = oracle.Matrix(1024, 2048, 64, 1, K["sym_packed"], K["sym_scales"], K["sym_zeros"])
    dense = m.dequantize().astype(np.float64) @ K["sym_x"].astype(np.float64)
    assert rel_err(K["sym_y"], dense) < 1e-5

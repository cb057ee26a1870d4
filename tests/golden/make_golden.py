"""Regenerate the golden fixtures in this directory from the reference library.

Runs the reference's own C++ code (oracle/_ref/libxqwen35_ref.so, compiled from the
reference sources by oracle/Makefile) on seeded inputs and on the inputs of the reference's
known-answer tests (customlib/tests/kernel_correctness/test_kernels.cpp), and stores inputs
and outputs as .npz files. The tests compare the oracle restatement and the CUDA path with
these files on machines where the reference tree is absent.

    python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import __graft_entry__  # noqa: E402

__graft_entry__.load_package()
from xqwen35_b200.packer import synthetic  # noqa: E402
import oracle as O  # noqa: E402


def kernel_cases():
    out = {}
    rng = np.random.default_rng(1234)
    # Seeded symmetric W4 matrix (benchmark distributions), 1024 x 2048, group 64 (a row
    # count at which the reference's WorkerPool uses all 8 threads; 2..7 threads can hang).
    rows, cols, g = 1024, 2048, 64
    packed = rng.integers(0, 256, size=(rows, cols // 2), dtype=np.uint8)
    scales = (np.abs(rng.standard_normal(rows * cols // g)) * 0.02).astype(np.float16).astype(np.float32)
    zeros = np.full(rows * cols // g, 8.0, np.float32)
    x = rng.standard_normal(cols).astype(np.float32)
    m = O.Matrix(rows, cols, g, 1, packed, scales, zeros)
    out.update(sym_packed=packed, sym_scales=scales, sym_zeros=zeros, sym_x=x, sym_y=O.ref_gemv(m, x))
    idx, val = O.ref_argmax(m, x)
    out.update(sym_argmax=np.array([idx], np.int32), sym_argmax_value=np.array([val], np.float32))
    # test_kernels.cpp:19-48 inputs: W = 0.7 sin(0.17 i), x = cos(0.11 i), 7 x 24, group 8.
    w = (np.sin(np.arange(7 * 24, dtype=np.float32) * np.float32(0.17)) * np.float32(0.7)).reshape(7, 24)
    x24 = np.cos(np.arange(24, dtype=np.float32) * np.float32(0.11)).astype(np.float32)
    q = O.ref_quantize(w.astype(np.float32), 8)
    out.update(kat_packed=q.packed, kat_scales=q.scales, kat_zeros=q.zeros, kat_x=x24, kat_y=O.ref_gemv(q, x24),
               kat_dense_y=(q.dequantize() @ x24.astype(np.float64)).astype(np.float32))
    # test_kernels.cpp:50-77 inputs: hand-packed affine (v2) 2 x 4 matrix, group 4.
    packed_v2 = np.array([(2 << 4) | 0, (15 << 4) | 7, (4 << 4) | 1, (8 << 4) | 6], np.uint8)
    mv2 = O.Matrix(2, 4, 4, 2, packed_v2, np.array([0.5, 0.25], np.float32), np.array([-1.0, 2.0], np.float32))
    xv2 = np.array([1.0, -2.0, 0.5, 3.0], np.float32)
    out.update(v2_packed=packed_v2, v2_scales=mv2.scales, v2_zeros=mv2.zeros, v2_x=xv2, v2_y=O.ref_gemv(mv2, xv2))
    # test_kernels.cpp:79-93 inputs: RMSNorm n = 16.
    xr = (np.float32(0.1) + np.arange(16, dtype=np.float32) * np.float32(0.03)).astype(np.float32)
    wr = (np.float32(1.0) + np.arange(16, dtype=np.float32) * np.float32(0.01)).astype(np.float32)
    yr = np.zeros(16, np.float32)
    O.ref().ref_rmsnorm(xr, wr, 16, np.float32(1e-6), yr)
    out.update(rms_x=xr, rms_w=wr, rms_y=yr)
    # test_kernels.cpp:234-325 inputs: two gated-delta steps with A_log -2.65625, dt_bias -3.53125.
    def l2(v):
        v = np.asarray(v, np.float32)
        return (v * (np.float32(1.0) / np.sqrt(np.sum(v * v, dtype=np.float32) + np.float32(1e-6)))).astype(np.float32)
    qs = [l2([0.4, -0.5, 0.6]), l2([-0.25, 0.35, 0.45])]
    ks = [l2([0.2, 0.1, -0.3]), l2([0.15, -0.4, 0.05])]
    vs = [np.array([0.7, -0.2], np.float32), np.array([-0.1, 0.55], np.float32)]
    a_proj = [np.float32(-0.35), np.float32(0.125)]
    b_proj = [np.float32(0.25), np.float32(-0.45)]
    L = O.port()
    state = np.zeros(6, np.float32)
    outs = []
    for s in range(2):
        beta = L.xo_sigmoid(b_proj[s])
        gate = -np.exp(np.float32(-2.65625)) * L.xo_softplus(np.float32(a_proj[s] + np.float32(-3.53125)))
        o = np.zeros(2, np.float32)
        O.ref().ref_gated_delta_decode(qs[s], ks[s], vs[s], np.float32(beta), np.float32(gate), 3, 2, state, o)
        outs.append(o.copy())
    out.update(delta_q=np.stack(qs), delta_k=np.stack(ks), delta_v=np.stack(vs), delta_a=np.array(a_proj),
               delta_b=np.array(b_proj), delta_out=np.stack(outs), delta_state=state)
    # test_kernels.cpp:141-196 inputs: GQA context 4, kv heads 2, q heads 4, dim 3.
    qa = np.sin(np.arange(1, 13, dtype=np.float32) * np.float32(0.13)).astype(np.float32)
    ka = np.cos(np.arange(2, 26, dtype=np.float32) * np.float32(0.17)).astype(np.float32)
    va = np.sin(np.arange(3, 27, dtype=np.float32) * np.float32(0.07)).astype(np.float32)
    oa = np.zeros(12, np.float32)
    O.ref().ref_attention_decode(qa, ka, va, 4, 2, 4, 3, oa)
    out.update(attn_q=qa, attn_k=ka, attn_v=va, attn_out=oa)
    np.savez(os.path.join(HERE, "kernel_cases.npz"), **out)


def model_small():
    d = os.path.join(os.environ.get("TMPDIR", "/tmp"), "xq_golden_small_s7")
    synthetic.make_package(d, synthetic.preset("small"), seed=7)
    ids = np.random.default_rng(7).integers(0, 4096, 12).astype(np.int32)
    r = O.RefSession(d)
    r.prefill(ids)
    h0 = r.hidden()
    toks = [r.decode_one() for _ in range(6)]
    h1 = r.hidden()
    np.savez(os.path.join(HERE, "model_small_s7.npz"), ids=ids, hidden_prefill=h0, tokens=np.array(toks, np.int32),
             hidden_after=h1)


if __name__ == "__main__":
    kernel_cases()
    model_small()
    print("golden fixtures written to", HERE)

"""DeltaNet, attention and RMSNorm kernels through the kernel C ABI vs the oracle.
Tolerances (max abs error relative to max |ref|): 1e-5 fp32 paths, 2e-3 with an fp16 KV cache."""
import os

import numpy as np
import pytest

from conftest import GOLDEN, PKG, rel_err

pytestmark = pytest.mark.gpu
K = np.load(os.path.join(GOLDEN, "kernel_cases.npz"))


def t(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def sync():
    import torch

    torch.cuda.synchronize()


def test_rmsnorm_kat():
    import torch

    y = torch.zeros(16, device="cuda")
    x, w = t(K["rms_x"]), t(K["rms_w"])  # keep the tensors alive across the call
    PKG.check(PKG.lib().xqk_rmsnorm(x.data_ptr(), w.data_ptr(), 16, 1e-6, y.data_ptr(), None), "rmsnorm")
    sync()
    assert np.abs(y.cpu().numpy() - K["rms_y"]).max() <= 1e-6


def oracle_delta(o, conv, ab, a_log, dt_bias, state, nk, nv, dk, dv):
    L = o.port()
    conv = conv.copy()
    q = conv[: nk * dk].copy()
    k = conv[nk * dk: 2 * nk * dk].copy()
    v = conv[2 * nk * dk:]
    L.xo_l2norm_heads(q, nk, dk)
    L.xo_l2norm_heads(k, nk, dk)
    out = np.zeros(nv * dv, np.float32)
    st = state.copy()
    for vh in range(nv):
        kh = vh // (nv // nk)
        beta = L.xo_sigmoid(float(ab[nv + vh]))
        gate = -np.exp(np.float32(a_log[vh])) * L.xo_softplus(float(ab[vh] + dt_bias[vh]))
        sv = st[vh * dk * dv:(vh + 1) * dk * dv].copy()
        ov = np.zeros(dv, np.float32)
        L.xo_gated_delta_decode(np.ascontiguousarray(q[kh * dk:(kh + 1) * dk]),
                                np.ascontiguousarray(k[kh * dk:(kh + 1) * dk]),
                                np.ascontiguousarray(v[vh * dv:(vh + 1) * dv]), np.float32(beta), np.float32(gate),
                                dk, dv, sv, ov)
        st[vh * dk * dv:(vh + 1) * dk * dv] = sv
        out[vh * dv:(vh + 1) * dv] = ov
    return out, st


@pytest.mark.parametrize("nk,nv", [(16, 32), (8, 16)])
def test_gated_delta_step_two_steps(oracle, nk, nv):
    rng = np.random.default_rng(nk)
    dk = dv = 128
    state = np.zeros(nv * dk * dv, np.float32)
    a_log = rng.uniform(-3, 0, nv).astype(np.float32)
    dt_bias = (rng.standard_normal(nv) - 3).astype(np.float32)
    sd = t(state)
    for step in range(3):
        conv = (rng.standard_normal(2 * nk * dk + nv * dv) * 2).astype(np.float32)
        ab = (rng.standard_normal(2 * nv) * 3).astype(np.float32)
        out_ref, state = oracle_delta(oracle, conv, ab, a_log, dt_bias, state, nk, nv, dk, dv)
        import torch

        od = torch.zeros(nv * dv, device="cuda")
        keep = [t(conv), t(ab), t(a_log), t(dt_bias)]
        PKG.check(PKG.lib().xqk_gated_delta_step(keep[0].data_ptr(), keep[1].data_ptr(), keep[2].data_ptr(),
                                                 keep[3].data_ptr(), sd.data_ptr(), od.data_ptr(), nk, nv, dk, dv,
                                                 None), "delta")
        sync()
        assert rel_err(od.cpu().numpy(), out_ref) <= 1e-5, step
        assert rel_err(sd.cpu().numpy(), state) <= 1e-5, step


def oracle_attention(o, qkv, qn, kn, kcache, vcache, pos, nq, nkv, hd, rot, theta, eps):
    L = o.port()
    q = np.concatenate([qkv[h * 2 * hd: h * 2 * hd + hd] for h in range(nq)]).astype(np.float32)
    gate = np.concatenate([qkv[h * 2 * hd + hd: (h + 1) * 2 * hd] for h in range(nq)]).astype(np.float32)
    k = qkv[2 * nq * hd: 2 * nq * hd + nkv * hd].copy()
    v = qkv[2 * nq * hd + nkv * hd:].copy()
    L.xo_head_rmsnorm(q, qn, nq, hd, np.float32(eps))
    L.xo_head_rmsnorm(k, kn, nkv, hd, np.float32(eps))
    L.xo_rope_partial(q, nq, hd, rot, pos, np.float32(theta))
    L.xo_rope_partial(k, nkv, hd, rot, pos, np.float32(theta))
    kc = kcache[: (pos + 1) * nkv * hd].copy()
    vc = vcache[: (pos + 1) * nkv * hd].copy()
    kc[pos * nkv * hd:] = k
    vc[pos * nkv * hd:] = v
    out = np.zeros(nq * hd, np.float32)
    L.xo_attention_decode(q, kc, vc, pos + 1, nkv, nq, hd, out)
    sig = np.array([L.xo_sigmoid(float(g)) for g in gate], np.float32)
    return out * sig, kc, vc


@pytest.mark.parametrize("pos,kv_fp16", [(0, 0), (37, 0), (511, 0), (767, 0), (511, 1)])
def test_attention_step(oracle, pos, kv_fp16):
    import torch

    rng = np.random.default_rng(pos)
    nq, nkv, hd, rot, cap = 16, 4, 256, 64, 1024
    theta, eps = 1e7, 1e-6
    qkv = (rng.standard_normal(2 * nq * hd + 2 * nkv * hd) * 3).astype(np.float32)
    qn = (1 + rng.standard_normal(hd) * 0.1).astype(np.float32)
    kn = (1 + rng.standard_normal(hd) * 0.1).astype(np.float32)
    kc = rng.standard_normal(cap * nkv * hd).astype(np.float32)
    vc = rng.standard_normal(cap * nkv * hd).astype(np.float32)
    if kv_fp16:
        kc = kc.astype(np.float16).astype(np.float32)
        vc = vc.astype(np.float16).astype(np.float32)
    ref, kref, vref = oracle_attention(oracle, qkv, qn, kn, kc, vc, pos, nq, nkv, hd, rot, theta, eps)
    dt = torch.float16 if kv_fp16 else torch.float32
    kd = torch.from_numpy(kc).to(dt).cuda()
    vd = torch.from_numpy(vc).to(dt).cuda()
    od = torch.zeros(nq * hd, device="cuda")
    keep = [t(qkv), t(qn), t(kn)]
    PKG.check(PKG.lib().xqk_attention_step(keep[0].data_ptr(), keep[1].data_ptr(), keep[2].data_ptr(), kd.data_ptr(),
                                           vd.data_ptr(), kv_fp16, cap, pos, nq, nkv, hd, rot, theta, eps,
                                           od.data_ptr(), None), "attention")
    sync()
    tol = 2e-3 if kv_fp16 else 1e-5
    assert rel_err(od.cpu().numpy(), ref) <= tol
    knew = kd.float().cpu().numpy()[pos * nkv * hd:(pos + 1) * nkv * hd]
    assert rel_err(knew, kref[pos * nkv * hd:]) <= (1e-3 if kv_fp16 else 1e-5)

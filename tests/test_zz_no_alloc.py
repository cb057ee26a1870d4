"""The allocation-free attention entry point (xqk_attention_step_noalloc).

It serves callers that cannot call cudaMalloc while they run, such as plugin hosts that
hand the library every buffer, code under a fixed device-memory budget, or paths where an
allocation would synchronise the device. Its scratch is a static device array, so these
tests check that it gives the same results as xqk_attention_step on two calls in a row
(the second call reuses scratch the first left behind) and that oversized requests are
refused. Tolerance: max abs difference relative to max |reference| <= 1e-5, the attention
tolerance of the other GPU tests. This file is collected last on purpose."""
import numpy as np
import pytest

from conftest import PKG, rel_err

pytestmark = pytest.mark.gpu


def _inputs(rng, nq, nkv, hd, cap):
    qkv = (rng.standard_normal(2 * nq * hd + 2 * nkv * hd) * 3).astype(np.float32)
    qn = (1 + rng.standard_normal(hd) * 0.1).astype(np.float32)
    kn = (1 + rng.standard_normal(hd) * 0.1).astype(np.float32)
    kc = rng.standard_normal(cap * nkv * hd).astype(np.float32)
    vc = rng.standard_normal(cap * nkv * hd).astype(np.float32)
    return qkv, qn, kn, kc, vc


@pytest.mark.parametrize("kv_fp16", [0, 1])
def test_noalloc_matches_allocating_entry_point_on_two_calls(kv_fp16):
    import torch

    L = PKG.lib()
    nq, nkv, hd, rot, cap, theta, eps = 16, 4, 256, 64, 1024, 1e7, 1e-6
    rng = np.random.default_rng(42 + kv_fp16)
    dt = torch.float16 if kv_fp16 else torch.float32
    for pos in (511, 512):  # two calls in a row on the shared static scratch
        qkv, qn, kn, kc, vc = _inputs(rng, nq, nkv, hd, cap)
        ins = [torch.from_numpy(a).cuda() for a in (qkv, qn, kn)]
        caches = {}
        outs = {}
        for name, fn in (("ref", L.xqk_attention_step), ("noalloc", L.xqk_attention_step_noalloc)):
            kd = torch.from_numpy(kc).to(dt).cuda()
            vd = torch.from_numpy(vc).to(dt).cuda()
            od = torch.full((nq * hd,), float("nan"), device="cuda")
            rc = fn(ins[0].data_ptr(), ins[1].data_ptr(), ins[2].data_ptr(), kd.data_ptr(), vd.data_ptr(), kv_fp16,
                    cap, pos, nq, nkv, hd, rot, theta, eps, od.data_ptr(), None)
            PKG.check(rc, name)
            torch.cuda.synchronize()
            outs[name] = od.cpu().numpy()
            caches[name] = (kd.float().cpu().numpy(), vd.float().cpu().numpy())
        assert np.isfinite(outs["noalloc"]).all()
        assert rel_err(outs["noalloc"], outs["ref"]) <= 1e-5
        assert np.array_equal(caches["noalloc"][0], caches["ref"][0])
        assert np.array_equal(caches["noalloc"][1], caches["ref"][1])


def test_noalloc_rejects_requests_beyond_its_scratch():
    import torch

    L = PKG.lib()
    hd, cap = 256, 64
    nq = nkv = 64  # 64 kv heads * 32 splits * 258 floats > 262144 floats of static scratch
    buf = torch.zeros(2 * nq * hd + 2 * nkv * hd, device="cuda")
    cache = torch.zeros(cap * nkv * hd, device="cuda")
    w = torch.ones(hd, device="cuda")
    out = torch.zeros(nq * hd, device="cuda")
    rc = L.xqk_attention_step_noalloc(buf.data_ptr(), w.data_ptr(), w.data_ptr(), cache.data_ptr(),
                                      cache.data_ptr(), 0, cap, 0, nq, nkv, hd, 64, 1e7, 1e-6, out.data_ptr(), None)
    assert rc == -1 and "static scratch holds" in PKG.last_error()

"""The whole decode path through the public C ABI (xq_create / xq_prefill / xq_decode_one /
xq_generate) vs the reference: greedy tokens must match exactly; the post-final-norm hidden
state within max rel err 1e-4 (fp32 KV cache) or 5e-3 (fp16 KV cache)."""
import ctypes as C
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN, PKG, package, rel_err

pytestmark = pytest.mark.gpu
G = np.load(os.path.join(GOLDEN, "model_small_s7.npz"))


@pytest.fixture(scope="module")
def small_session(small_pkg):
    s = PKG.Session(small_pkg, device=0)
    yield s
    s.close()


def test_small_model_matches_reference_golden(small_session):
    s = small_session
    s.prefill(G["ids"])
    assert rel_err(s.hidden(), G["hidden_prefill"]) <= 1e-4
    toks = [s.decode_one() for _ in range(len(G["tokens"]))]
    assert toks == list(G["tokens"])
    assert rel_err(s.hidden(), G["hidden_after"]) <= 1e-4


@pytest.mark.parametrize("mma", ["1", "0"])
def test_step_gemv_engines_match_reference_golden(small_pkg, monkeypatch, mma):
    """Both GEMV engines of the step kernel (integer tensor cores, and the dp4a row loop that
    XQ_STEP_MMA=0 selects) against the reference's golden outputs."""
    monkeypatch.setenv("XQ_STEP_MMA", mma)
    s = PKG.Session(small_pkg, device=0)
    try:
        info = json.loads(s.json("backend"))
        assert info["persistent_step_kernel"] and info["tensor_core_gemv"] == (mma == "1")
        s.prefill(G["ids"])
        assert rel_err(s.hidden(), G["hidden_prefill"]) <= 1e-4
        toks = [s.decode_one() for _ in range(len(G["tokens"]))]
        assert toks == list(G["tokens"])
        assert rel_err(s.hidden(), G["hidden_after"]) <= 1e-4
    finally:
        s.close()


def test_generate_equals_decode_loop(small_session):
    s = small_session
    out, m = s.generate(G["ids"], len(G["tokens"]))
    assert list(out) == list(G["tokens"])
    assert m.generated_tokens == len(G["tokens"]) and m.prompt_tokens == len(G["ids"])
    assert m.decode_tokens_per_second > 0 and m.prefill_tokens_per_second > 0
    assert rel_err(s.hidden(), G["hidden_after"]) <= 1e-4


def test_eager_and_graph_paths_agree(small_pkg):
    a = PKG.Session(small_pkg, device=0, use_graphs=True)
    b = PKG.Session(small_pkg, device=0, use_graphs=False)
    ids = np.arange(20, dtype=np.int32) * 37
    ta, _ = a.generate(ids, 5)
    tb, _ = b.generate(ids, 5)
    assert list(ta) == list(tb)
    assert np.array_equal(a.hidden(), b.hidden())


def test_status_codes_and_trace(small_pkg):
    s = PKG.Session(small_pkg, device=0)
    L = PKG.lib()
    t = C.c_int32()
    m = PKG.XqMetrics()
    m.struct_size = C.sizeof(m)
    assert L.xq_decode_one(s.h, C.byref(t), C.byref(m)) == PKG.XQ_ERR_NOT_READY  # session.cpp:345-349
    assert L.xq_prefill(s.h, None, 0, C.byref(m)) == PKG.XQ_ERR_INVALID_ARGUMENT
    ids = np.array([1, 2, 3], np.int32)
    out = np.zeros(2, np.int32)
    assert L.xq_generate(s.h, ids.ctypes.data_as(C.POINTER(C.c_int32)), 3, 4,
                         out.ctypes.data_as(C.POINTER(C.c_int32)), 2, C.byref(m)) == PKG.XQ_ERR_BUFFER_TOO_SMALL
    s.prefill(ids)
    assert L.xq_decode_one(s.h, None, C.byref(m)) == PKG.XQ_ERR_INVALID_ARGUMENT
    s.decode_one()
    n = C.c_size_t()
    small = np.zeros(4, np.float32)
    assert L.xq_get_hidden_state(s.h, small.ctypes.data_as(C.POINTER(C.c_float)), 4, C.byref(n)) == \
        PKG.XQ_ERR_BUFFER_TOO_SMALL and n.value == 2048
    buf = C.create_string_buffer(8)
    assert L.xq_get_backend_info(s.h, buf, 8) == PKG.XQ_ERR_BUFFER_TOO_SMALL
    trace = s.json("trace")
    names = {r["name"] for r in json.loads(trace)["rows"]}
    for n_ in ["prefill_token_custom", "prefill_kv_build_custom", "linear_attention_state_update_custom",
               "attention_score_custom", "attention_softmax_custom", "attention_v_reduce_custom", "lm_head_custom",
               "sampling_greedy_custom"]:  # the rows test_runtime.cpp:175-202 requires
        assert n_ in names
    assert "fallback_" not in trace
    m2 = s.metrics()
    assert m2.rss_kb > 0 and m2.pss_kb > 0  # host resident set; device memory of the session
    info = s.json("backend")
    assert "full_custom_decode=true" in info and "fallback_ops=none" in info
    dbg = json.loads(s.json("debug"))
    assert dbg["hidden"]["size"] == 2048 and len(dbg["lm_head_topk"]) == 10
    assert s.reset() == 0
    assert L.xq_decode_one(s.h, C.byref(t), C.byref(m)) == PKG.XQ_ERR_NOT_READY
    s.close()


def test_step_phase_trace_rows(small_pkg, monkeypatch):
    """With XQ_STEP_TRACE=1 the kernel trace carries one row per step-kernel phase kind with its
    device time, under names the reference's op_family rules classify."""
    monkeypatch.setenv("XQ_STEP_TRACE", "1")
    s = PKG.Session(small_pkg, device=0)
    try:
        if not json.loads(s.json("backend")).get("persistent_step_kernel"):
            pytest.skip("model not served by the step kernel")
        s.prefill(np.arange(9, dtype=np.int32))
        for _ in range(3):
            s.decode_one()
        rows = {r["name"]: r for r in json.loads(s.json("trace"))["rows"]}
        r = rows["linear_gate_proj_up_proj_swiglu_step_phase"]
        assert r["backend"] == "cuda_persistent_kernel" and r["op_family"] == "gate_proj"
        assert r["calls"] > 0 and r["total_ms"] > 0
        assert rows["lm_head_argmax_step_phase"]["op_family"] == "lm_head"
        assert rows["linear_attention_state_step_phase"]["op_family"] == "linear_attention_state"
        assert rows["decode_step_custom"]["backend"] == "cuda_persistent_kernel"
    finally:
        s.close()


def test_fp16_kv_cache_tolerance(small_pkg):
    s = PKG.Session(small_pkg, device=0, kv_fp16=True)
    s.prefill(G["ids"])
    assert rel_err(s.hidden(), G["hidden_prefill"]) <= 5e-3


def test_kv_cache_growth_past_initial_capacity(small_pkg, oracle):
    s = PKG.Session(small_pkg, device=0, max_context_tokens=64)
    ids = np.random.default_rng(1).integers(0, 4096, 100).astype(np.int32)
    s.prefill(ids)
    toks = [s.decode_one() for _ in range(3)]
    p = oracle.PortModel(small_pkg)
    p.prefill(ids)
    assert toks == [p.decode_one() for _ in range(3)]
    assert rel_err(s.hidden(), p.hidden()) <= 1e-4


def test_cfg1_two_layer_decode_step(oracle):
    # Config 1 shapes (hidden 4096, MLP 12288, 16/32 DeltaNet heads, 16/4 GQA heads of 256),
    # vocab 1024; a 96-token prefill then decode steps, against the oracle restatement.
    d = package("cfg1", seed=1)
    ids = np.random.default_rng(11).integers(0, 1024, 96).astype(np.int32)
    s = PKG.Session(d, device=0)
    s.prefill(ids)
    p = oracle.PortModel(d)
    p.prefill(ids)
    assert rel_err(s.hidden(), p.hidden()) <= 1e-4
    toks = [s.decode_one() for _ in range(2)]
    assert toks == [p.decode_one() for _ in range(2)]
    assert rel_err(s.hidden(), p.hidden()) <= 1e-4


def test_step_kernel_binary_is_sm100(small_session):
    """The loaded persistent step kernel was compiled for sm_100a (cudaFuncGetAttributes)."""
    info = json.loads(small_session.json("backend"))
    assert info["step_kernel_binary_version"] == 100

"""Host-side checks that need no GPU: the library loads, exports every entry point the
public headers declare, and the argument checks the reference performs before touching
the model return the reference's status codes."""
import ctypes as C
import os
import re

import numpy as np
import pytest

from conftest import PKG, ROOT, cuda_available, package


def declared_functions():
    names = []
    for h in ("xqwen35.h", "xq_kernels.h"):
        with open(os.path.join(ROOT, "include", h)) as f:
            src = f.read()
        names += re.findall(r"XQK?_API\s+[\w\s\*]+?\b(\w+)\s*\(", src)
    return names


def test_library_built_for_sm100a():
    """The build compiles every CUDA source for sm_100a only (checked on the build recipe; the
    GPU test test_step_kernel_binary_is_sm100 checks the loaded kernel's binary version)."""
    assert os.path.exists(PKG.LIB_PATH), "run __graft_entry__.build()"
    mk = open(os.path.join(PKG.CSRC, "Makefile")).read()
    arch = re.search(r"^ARCH\s*:=\s*(.*)$", mk, re.M).group(1).split()
    assert arch == ["-gencode", "arch=compute_100a,code=sm_100a"]
    assert "$(ARCH)" in re.search(r"^NVFLAGS\s*:=.*$", mk, re.M).group(0)


def test_exports_every_declared_symbol():
    L = PKG.lib()
    names = declared_functions()
    assert set(names) == set(PKG.ABI_SYMBOLS + PKG.KERNEL_SYMBOLS)
    for n in names:
        assert hasattr(L, n), n


def test_binding_declares_every_argument_list():
    """ctypes passes an undeclared pointer argument as a 32-bit int: every entry point that
    takes arguments must have its argtypes set by the Python binding."""
    L = PKG.lib()
    for h in ("xqwen35.h", "xq_kernels.h"):
        with open(os.path.join(ROOT, "include", h)) as f:
            src = f.read()
        for name, args in re.findall(r"XQK?_API\s+[\w\s\*]+?\b(\w+)\s*\(([^)]*)\)", src):
            if args.strip() not in ("", "void"):
                assert getattr(L, name).argtypes is not None, name


def test_null_arguments_follow_reference_status_codes():
    L = PKG.lib()
    out = C.c_void_p()
    assert L.xq_create(None, None, C.byref(out)) == PKG.XQ_ERR_INVALID_ARGUMENT
    assert L.xq_create(b"/nonexistent", None, None) == PKG.XQ_ERR_INVALID_ARGUMENT
    assert L.xq_prefill(None, None, 0, None) == PKG.XQ_ERR_INVALID_ARGUMENT
    assert L.xq_decode_one(None, None, None) == PKG.XQ_ERR_INVALID_ARGUMENT
    assert L.xq_generate(None, None, 0, 0, None, 0, None) == PKG.XQ_ERR_INVALID_ARGUMENT
    assert L.xq_reset(None) == PKG.XQ_ERR_INVALID_ARGUMENT
    assert L.xq_get_last_metrics(None, None) == PKG.XQ_ERR_INVALID_ARGUMENT
    n = C.c_size_t()
    assert L.xq_get_hidden_state(None, None, 0, C.byref(n)) == PKG.XQ_ERR_INVALID_ARGUMENT
    # snapshot entry points (no reference counterpart) follow the same conventions
    assert L.xq_snapshot_size(None, C.byref(n)) == PKG.XQ_ERR_INVALID_ARGUMENT
    assert L.xq_snapshot_save(None, None, 0, C.byref(n)) == PKG.XQ_ERR_INVALID_ARGUMENT
    assert L.xq_snapshot_restore(None, None, 0) == PKG.XQ_ERR_INVALID_ARGUMENT
    L.xq_destroy(None)


def test_vulkan_selftest_reports_unavailable():
    buf = C.create_string_buffer(2048)
    assert PKG.lib().xq_run_vulkan_w4a16_selftest(buf, len(buf)) == PKG.XQ_ERR_RUNTIME
    assert b'"pass":false' in buf.value


@pytest.mark.skipif(cuda_available(), reason="checks the no-GPU failure path")
def test_create_without_gpu_fails_loudly():
    d = package("small", seed=7)
    out = C.c_void_p()
    st = PKG.lib().xq_create(d.encode(), None, C.byref(out))
    assert st == PKG.XQ_ERR_MODEL and not out.value


def test_kernel_abi_rejects_bad_arguments():
    L = PKG.lib()
    h = C.c_void_p()
    assert L.xqk_matrix_create(None, None, None, 4, 4, 4, 1, 0, C.byref(h)) == -1
    assert L.xqk_gemv_w4a16(None, None, None, None) == -1
    assert L.xqk_attention_step(None, None, None, None, None, 0, 0, 0, 0, 0, 0, 0, 1.0, 1e-6, None, None) == -1


def test_synthetic_package_distributions():
    from xqwen35_b200.packer import synthetic

    d = package("small", seed=7)
    m = synthetic.read_xq4(os.path.join(d, "layers_0_mlp_gate_proj_weight.xq4"))
    assert m["version"] == 1 and m["group"] == 64 and m["rows"] == 2048 and m["cols"] == 2048
    assert np.all(m["zeros"] == 8.0)
    s = m["scales"]
    assert np.array_equal(s, s.astype(np.float16).astype(np.float32))
    codes = np.concatenate([m["packed"].reshape(-1) & 15, m["packed"].reshape(-1) >> 4])
    assert codes.min() == 0 and codes.max() == 15 and abs(codes.mean() - 7.5) < 0.05
    emb = np.fromfile(os.path.join(d, "embeddings_bf16.bin"), dtype=np.uint16)
    f = (emb.astype(np.uint32) << 16).view(np.float32)
    assert np.array_equal(f, f.astype(np.float16).astype(np.float32))  # fp16-representable


def test_package_generation_is_deterministic(tmp_path):
    from xqwen35_b200.packer import synthetic

    cfg = synthetic.preset("small")
    cfg.layer_types = ["linear_attention"]
    a = synthetic.make_package(str(tmp_path / "a"), cfg, seed=11)
    b = synthetic.make_package(str(tmp_path / "b"), cfg, seed=11)
    for name in sorted(os.listdir(a)):
        with open(os.path.join(a, name), "rb") as fa, open(os.path.join(b, name), "rb") as fb:
            assert fa.read() == fb.read(), name

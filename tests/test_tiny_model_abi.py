"""The reference's own tiny runtime-test model (hidden 4, head_dim 2, linear head dims 2, conv
kernel 2, vocab 8, group 4; customlib/tests/runtime_correctness/test_runtime.cpp:72-144, written
by tests/golden/make_tiny_fixture.py) served as a drop-in: a plain C program compiled against
include/xqwen35.h and linked to libxqwen35.so runs the reference test's call sequence and
checks (status codes, metrics, trace row names, backend info; test_runtime.cpp:148-211), and its
outputs must equal the reference library's on the same package: the greedy tokens exactly, the
hidden states within 1e-5 (shapes the fused kernels do not take run the generic-shape step on
the GPU). The CPU test pins the oracle restatement to the same reference outputs."""
import os
import shutil
import subprocess

import numpy as np
import pytest

from conftest import GOLDEN, PKG, ROOT, rel_err

TINY = os.path.join(GOLDEN, "tiny_model")
REF = np.load(os.path.join(GOLDEN, "tiny_model_ref.npz"))


def test_oracle_matches_reference_on_tiny_model(oracle):
    m = oracle.PortModel(TINY)
    m.prefill(REF["prompt"])
    assert rel_err(m.hidden(), REF["hidden_prefill"]) <= 1e-6
    assert m.decode_one() == int(REF["decode_token"])
    assert rel_err(m.hidden(), REF["hidden_decode"]) <= 1e-6
    m.prefill(REF["prompt"])
    assert [m.decode_one() for _ in range(2)] == list(REF["generate_tokens"])
    assert rel_err(m.hidden(), REF["hidden_generate"]) <= 1e-6
    m.close()


@pytest.mark.gpu
def test_c_host_runs_reference_runtime_test_on_tiny_model(tmp_path):
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    exe = str(tmp_path / "abi_tiny_model")
    lib_dir = os.path.dirname(PKG.LIB_PATH)
    subprocess.run([cc, "-std=c11", "-O1", "-Wall", "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "abi_tiny_model.c"), "-o", exe, "-L", lib_dir, "-lxqwen35",
                    f"-Wl,-rpath,{lib_dir}"], check=True)
    r = subprocess.run([exe, TINY], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    lines = {ln.split()[0]: ln.split()[1:] for ln in r.stdout.splitlines() if ln.strip()}
    assert "ok" in lines
    assert int(lines["decode_token"][0]) == int(REF["decode_token"])
    assert [int(v) for v in lines["generate_tokens"]] == list(REF["generate_tokens"])
    for k in ("hidden_prefill", "hidden_decode", "hidden_generate"):
        assert rel_err(np.array(lines[k], np.float32), REF[k]) <= 1e-5, k

"""The full 9B-shaped model (config 2 shapes: 32 layers, 3:1 DeltaNet:GQA, vocab 248320,
W4A16 g64) through the public C ABI against the reference library's own output on the same
seeded package (tests/golden/model_9b_s2024.npz, made by make_golden_9b.py): the hidden state
after prefill and after 8 greedy steps within max rel err 1e-4, the greedy tokens exactly. The
package (6.6 GB) is rebuilt from its seed where bench.py keeps it."""
import os

import numpy as np
import pytest

from conftest import GOLDEN, PKG, rel_err, synthetic

pytestmark = pytest.mark.gpu
PATH = os.path.join(GOLDEN, "model_9b_s2024.npz")


@pytest.mark.skipif(not os.path.exists(PATH), reason="9B golden file not generated")
def test_9b_package_matches_reference_golden():
    G = np.load(PATH)
    d = os.path.join(os.environ.get("XQ_BENCH_DIR", os.path.join(os.environ.get("TMPDIR", "/tmp"), "xq_bench")),
                     "qwen35_9b_s2024")
    synthetic.make_package(d, synthetic.preset("cfg2"), seed=2024)
    s = PKG.Session(d, device=0)
    try:
        s.prefill(G["ids"])
        assert rel_err(s.hidden(), G["hidden_prefill"]) <= 1e-4
        toks = [s.decode_one() for _ in range(len(G["tokens"]))]
        assert toks == list(G["tokens"])
        assert rel_err(s.hidden(), G["hidden_after"]) <= 1e-4
    finally:
        s.close()

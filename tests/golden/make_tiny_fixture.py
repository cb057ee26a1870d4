"""The reference's tiny runtime-test model (customlib/tests/runtime_correctness/test_runtime.cpp:
72-144: hidden 4, 2 layers (one Gated-DeltaNet, one full attention), head_dim 2, linear head
dims 2, conv kernel 2, vocab 8, group 4) written as a package under tests/golden/tiny_model/, and
the reference library's own outputs on it (prompt [1, 2, 3]: the hidden state after prefill,
the xq_decode_one token, then the xq_generate tokens and hidden state) in
tests/golden/tiny_model_ref.npz.

The matrices are quantized with the reference's own quantizeLowBit (4 bits, group 4; through
the oracle shim), the embeddings are bf16 by truncation, as the reference test writes them.

    python tests/golden/make_tiny_fixture.py      (needs oracle/_ref, the compiled reference)
"""
import json
import os
import struct
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle as O  # noqa: E402

DIR = os.path.join(HERE, "tiny_model")
PROMPT = np.array([1, 2, 3], np.int32)

MANIFEST = {"format": "xqwen35_custom_w4a16", "hidden_size": 4, "intermediate_size": 8, "vocab_size": 8,
            "num_hidden_layers": 2, "num_attention_heads": 2, "num_key_value_heads": 1, "head_dim": 2,
            "linear_key_head_dim": 2, "linear_value_head_dim": 2, "linear_num_key_heads": 1,
            "linear_num_value_heads": 2, "linear_conv_kernel_dim": 2, "rms_norm_eps": 0.000001,
            "rope_theta": 10000, "partial_rotary_factor": 1.0}


def patterned(rows, cols, scale):
    r = np.arange(rows)[:, None]
    c = np.arange(cols)[None, :]
    sign = np.where((r + c) % 2 == 0, 1.0, -1.0)
    return (sign * scale * (1.0 + ((r * 3 + c * 5) % 7))).astype(np.float32)


def write_vec(name, values):
    np.asarray(values, np.float32).tofile(os.path.join(DIR, name))


def write_xq4(name, rows, cols, scale):
    m = O.ref_quantize(patterned(rows, cols, scale), 4)
    with open(os.path.join(DIR, name), "wb") as f:
        f.write(struct.pack("<8sIIIIIQQQ", b"XQW4A16\0", 1, m.rows, m.cols, m.group, 4, m.packed.size,
                            m.scales.size, m.zeros.size))
        f.write(m.packed.tobytes())
        f.write(m.scales.astype("<f4").tobytes())
        f.write(m.zeros.astype("<f4").tobytes())


def make_package():
    os.makedirs(DIR, exist_ok=True)
    # the reference writes this manifest as one line with this key order
    with open(os.path.join(DIR, "xqwen35_manifest.json"), "w") as f:
        f.write(json.dumps(MANIFEST, separators=(",", ":")))
    emb = np.zeros((8, 4), np.float32)
    for t in range(8):
        for d in range(4):
            emb[t, d] = np.float32(0.05) * np.float32(t + 1) + (np.float32(1.0) if t == d else np.float32(0.0))
    (emb.view(np.uint32) >> 16).astype(np.uint16).tofile(os.path.join(DIR, "embeddings_bf16.bin"))
    write_vec("norm_weight.f32", np.ones(4))
    for layer in range(2):
        p = f"layers_{layer}_"
        write_vec(p + "input_layernorm_weight.f32", np.ones(4))
        write_vec(p + "post_attention_layernorm_weight.f32", np.ones(4))
        write_xq4(p + "mlp_gate_proj_weight.xq4", 8, 4, 0.02)
        write_xq4(p + "mlp_up_proj_weight.xq4", 8, 4, 0.015)
        write_xq4(p + "mlp_down_proj_weight.xq4", 4, 8, 0.01)
    write_xq4("layers_0_linear_attn_in_proj_qkv_weight.xq4", 8, 4, 0.03)
    write_xq4("layers_0_linear_attn_in_proj_a_weight.xq4", 2, 4, 0.02)
    write_xq4("layers_0_linear_attn_in_proj_b_weight.xq4", 2, 4, 0.025)
    write_xq4("layers_0_linear_attn_in_proj_z_weight.xq4", 4, 4, 0.03)
    write_xq4("layers_0_linear_attn_out_proj_weight.xq4", 4, 4, 0.02)
    write_vec("layers_0_linear_attn_norm_weight.f32", np.ones(2))
    write_vec("layers_0_linear_attn_conv1d_weight.f32", np.tile([0.25, 1.0], 8))
    write_vec("layers_0_linear_attn_A_log.f32", [-2.0, -2.2])
    write_vec("layers_0_linear_attn_dt_bias.f32", [0.0, 0.1])
    write_xq4("layers_1_self_attn_q_proj_weight.xq4", 8, 4, 0.025)
    write_xq4("layers_1_self_attn_k_proj_weight.xq4", 2, 4, 0.02)
    write_xq4("layers_1_self_attn_v_proj_weight.xq4", 2, 4, 0.03)
    write_xq4("layers_1_self_attn_o_proj_weight.xq4", 4, 4, 0.02)
    write_vec("layers_1_self_attn_q_norm_weight.f32", np.ones(2))
    write_vec("layers_1_self_attn_k_norm_weight.f32", np.ones(2))
    write_xq4("lm_head_weight.xq4", 8, 4, 0.04)


def main():
    make_package()
    s = O.RefSession(DIR, threads=1)
    s.prefill(PROMPT)
    h0 = s.hidden()
    t1 = s.decode_one()
    h1 = s.hidden()
    # xq_generate = prefill again + 2 decode steps (session.cpp:385-421)
    s.prefill(PROMPT)
    g = [s.decode_one() for _ in range(2)]
    h2 = s.hidden()
    s.close()
    np.savez(os.path.join(HERE, "tiny_model_ref.npz"), prompt=PROMPT, hidden_prefill=h0, decode_token=t1,
             hidden_decode=h1, generate_tokens=np.array(g, np.int32), hidden_generate=h2)
    print("decode", t1, "generate", g, "hidden", h0)


if __name__ == "__main__":
    main()

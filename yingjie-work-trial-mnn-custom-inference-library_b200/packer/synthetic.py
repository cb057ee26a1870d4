"""Seeded random-init model packages in the reference's on-disk format.

A package is a directory the reference's loader accepts unchanged
(customlib/runtime/custom_model.cpp:423-553):

* ``xqwen35_manifest.json``: dims read with substring search (custom_model.cpp:431-453);
* ``embeddings_bf16.bin``: ``[vocab][hidden]`` bf16;
* ``norm_weight.f32`` and per-layer ``*.f32`` vectors;
* XQ4 matrices: 8-byte magic ``XQW4A16\\0``, u32 version / rows / cols / group / bits,
  u64 packed_bytes / scale_count / zero_count, then the nibbles (row-major, even column in
  the low nibble), fp32 scales, fp32 zeros (custom_model.cpp:218-262; writer
  pack_qwen35_xq4_numpy.py:166-188, 248).

Value distributions follow the benchmark definitions: int4 values uniform in [-8, 7]
stored as XQ4 v1 codes ``v + 8`` with zero = 8; one fp16-representable scale per 64
weights drawn from |N(0, 0.02)|; norms N(0, 0.1) (the loader adds 1); conv weights
N(0, 0.5); A_log ~ U(-3, 0); dt_bias ~ N(-3, 1); embeddings N(0, 1) rounded to bf16 and
restricted to values exactly representable in fp16 as well.

Every file is generated from its own PCG64 stream keyed by (seed, file name) with a fixed
chunking, so a package is bit-identical on every machine with the same numpy.
"""
from __future__ import annotations

import dataclasses
import json
import os
import struct
import zlib
from typing import Dict, List

import numpy as np

XQ4_MAGIC = b"XQW4A16\x00"
_CHUNK_ROWS = 2048


@dataclasses.dataclass
class ModelConfig:
    hidden_size: int = 4096
    intermediate_size: int = 12288
    vocab_size: int = 248320
    num_attention_heads: int = 16
    num_key_value_heads: int = 4
    head_dim: int = 256
    linear_key_head_dim: int = 128
    linear_value_head_dim: int = 128
    linear_num_key_heads: int = 16
    linear_num_value_heads: int = 32
    linear_conv_kernel_dim: int = 4
    rms_norm_eps: float = 1e-6
    rope_theta: float = 10000000.0
    partial_rotary_factor: float = 0.25
    group_size: int = 64
    layer_types: List[str] = dataclasses.field(default_factory=list)

    @property
    def num_hidden_layers(self) -> int:
        return len(self.layer_types)

    @property
    def conv_dim(self) -> int:
        return 2 * self.linear_key_head_dim * self.linear_num_key_heads + (
            self.linear_value_head_dim * self.linear_num_value_heads)


def qwen35_9b(num_layers: int = 32, vocab_size: int = 248320) -> ModelConfig:
    """Qwen3.5-9B shapes: 3 Gated-DeltaNet layers then 1 full-attention layer, repeated."""
    types = ["full_attention" if (i % 4) == 3 else "linear_attention" for i in range(num_layers)]
    return ModelConfig(vocab_size=vocab_size, layer_types=types)


def preset(name: str) -> ModelConfig:
    """Named configurations.

    * ``cfg1``: one DeltaNet layer + one full-attention layer at 9B shapes, vocab 1024.
    * ``cfg2``: the full 32-layer 9B-shaped model with the real vocab (248320).
    * ``small``: the 9B layer pattern at reduced widths, for fast CPU checks. Its widths
      keep every reference GEMV either single-threaded or on all 8 pool threads: the
      reference's WorkerPool (xq_gemv_w4a16_neon.cpp:145-182) can hang when a call uses
      more than one but fewer than all of its threads. Like the 9B shapes it keeps
      heads * head_dim == hidden and value heads * 128 <= hidden, which the reference's
      scratch sizing assumes (custom_model.cpp:478-498).
    """
    if name == "cfg1":
        return ModelConfig(vocab_size=1024, layer_types=["linear_attention", "full_attention"])
    if name == "cfg2":
        return qwen35_9b()
    if name == "small":
        return ModelConfig(hidden_size=2048, intermediate_size=2048, vocab_size=4096,
                           num_attention_heads=8, num_key_value_heads=4, head_dim=256,
                           linear_key_head_dim=128, linear_value_head_dim=128,
                           linear_num_key_heads=8, linear_num_value_heads=16,
                           layer_types=["linear_attention", "linear_attention",
                                        "linear_attention", "full_attention"])
    raise ValueError(f"unknown preset {name!r}")


def _rng(seed: int, name: str) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(np.random.SeedSequence([seed, zlib.crc32(name.encode())])))


def _write_f32(path: str, values: np.ndarray) -> None:
    with open(path, "wb") as f:
        f.write(np.ascontiguousarray(values, dtype="<f4").tobytes())


def write_xq4(path: str, rows: int, cols: int, group: int, packed: np.ndarray, scales: np.ndarray,
              zeros: np.ndarray, version: int = 1) -> None:
    """Write one XQ4 matrix (header layout: customlib/runtime/custom_model.cpp:218-262)."""
    gpr = (cols + group - 1) // group
    packed = np.ascontiguousarray(packed, dtype=np.uint8).reshape(rows, (cols + 1) // 2)
    assert scales.size == rows * gpr and zeros.size == rows * gpr
    with open(path, "wb") as f:
        f.write(struct.pack("<8sIIIIIQQQ", XQ4_MAGIC, version, rows, cols, group, 4,
                            packed.size, scales.size, zeros.size))
        f.write(packed.tobytes())
        f.write(np.ascontiguousarray(scales, dtype="<f4").tobytes())
        f.write(np.ascontiguousarray(zeros, dtype="<f4").tobytes())


def read_xq4(path: str) -> Dict:
    with open(path, "rb") as f:
        head = f.read(struct.calcsize("<8sIIIIIQQQ"))
        magic, version, rows, cols, group, bits, nbytes, nscale, nzero = struct.unpack("<8sIIIIIQQQ", head)
        if magic[:7] != XQ4_MAGIC[:7]:
            raise ValueError(f"bad xq4 magic: {path}")
        packed = np.frombuffer(f.read(nbytes), dtype=np.uint8).reshape(rows, -1)
        scales = np.frombuffer(f.read(4 * nscale), dtype="<f4")
        zeros = np.frombuffer(f.read(4 * nzero), dtype="<f4")
    return dict(version=version, rows=rows, cols=cols, group=group, bits=bits, packed=packed,
                scales=scales, zeros=zeros)


def _gen_matrix(path: str, rows: int, cols: int, group: int, seed: int, quant: str) -> None:
    """quant: 'sym' (XQ4 v1, zero 8, fp16 scales), 'asym' (v1, integer zeros, fp32 scales),
    'v2' (XQ4 v2 affine: code * scale + zero with fp32 zero)."""
    rng = _rng(seed, os.path.basename(path))
    gpr = (cols + group - 1) // group
    version = 2 if quant == "v2" else 1
    with open(path, "wb") as f:
        f.write(struct.pack("<8sIIIIIQQQ", XQ4_MAGIC, version, rows, cols, group, 4,
                            rows * ((cols + 1) // 2), rows * gpr, rows * gpr))
        scales_all = np.empty((rows, gpr), dtype=np.float32)
        zeros_all = np.empty((rows, gpr), dtype=np.float32)
        for r0 in range(0, rows, _CHUNK_ROWS):
            nr = min(_CHUNK_ROWS, rows - r0)
            packed = rng.integers(0, 256, size=(nr, (cols + 1) // 2), dtype=np.uint8)
            if cols % 2:
                packed[:, -1] &= 0x0F
            s = np.abs(rng.standard_normal((nr, gpr), dtype=np.float32)) * np.float32(0.02)
            if quant == "sym":
                s = s.astype(np.float16).astype(np.float32)
                z = np.full((nr, gpr), 8.0, dtype=np.float32)
            elif quant == "asym":
                z = rng.integers(0, 16, size=(nr, gpr)).astype(np.float32)
            else:
                z = (rng.standard_normal((nr, gpr), dtype=np.float32) * np.float32(0.1)).astype(np.float32)
            scales_all[r0:r0 + nr] = s
            zeros_all[r0:r0 + nr] = z
            f.write(packed.tobytes())
        f.write(scales_all.astype("<f4").tobytes())
        f.write(zeros_all.astype("<f4").tobytes())


def bf16_round(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns, round to nearest even."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = (b + np.uint32(0x7FFF) + ((b >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)
    return r.astype(np.uint16)


def _gen_embeddings(path: str, vocab: int, hidden: int, seed: int) -> None:
    rng = _rng(seed, "embeddings_bf16.bin")
    with open(path, "wb") as f:
        for r0 in range(0, vocab, _CHUNK_ROWS):
            nr = min(_CHUNK_ROWS, vocab - r0)
            v = rng.standard_normal((nr, hidden), dtype=np.float32)
            v[np.abs(v) < np.float32(2.0 ** -14)] = 0.0  # keep every value fp16-representable
            f.write(bf16_round(v).tobytes())


def manifest_dict(cfg: ModelConfig, quant: str) -> Dict:
    return {
        "format": "xqwen35_custom_w4a16",
        "generator": "xqwen35_b200.packer.synthetic",
        "quantization": {"bits": 4, "group_size": cfg.group_size, "scheme": quant},
        "hidden_size": cfg.hidden_size,
        "intermediate_size": cfg.intermediate_size,
        "num_hidden_layers": cfg.num_hidden_layers,
        "num_attention_heads": cfg.num_attention_heads,
        "num_key_value_heads": cfg.num_key_value_heads,
        "head_dim": cfg.head_dim,
        "linear_key_head_dim": cfg.linear_key_head_dim,
        "linear_value_head_dim": cfg.linear_value_head_dim,
        "linear_num_key_heads": cfg.linear_num_key_heads,
        "linear_num_value_heads": cfg.linear_num_value_heads,
        "linear_conv_kernel_dim": cfg.linear_conv_kernel_dim,
        "vocab_size": cfg.vocab_size,
        "layer_types": cfg.layer_types,
        "rms_norm_eps": cfg.rms_norm_eps,
        "rope_theta": cfg.rope_theta,
        "partial_rotary_factor": cfg.partial_rotary_factor,
    }


def make_package(out_dir: str, cfg: ModelConfig, seed: int = 0, quant: str = "sym") -> str:
    """Write a complete package; skipped when ``out_dir`` already holds one made from the
    same (config, seed, quant), so repeated runs reuse it."""
    os.makedirs(out_dir, exist_ok=True)
    ident = json.dumps({"cfg": dataclasses.asdict(cfg), "seed": seed, "quant": quant}, sort_keys=True)
    stamp_path = os.path.join(out_dir, ".synthetic_stamp")
    if os.path.exists(stamp_path):
        with open(stamp_path) as f:
            if f.read() == ident:
                return out_dir
    g = cfg.group_size
    H, I = cfg.hidden_size, cfg.intermediate_size

    def mat(name, rows, cols):
        _gen_matrix(os.path.join(out_dir, name), rows, cols, g, seed, quant)

    def vec(name, values):
        _write_f32(os.path.join(out_dir, name), values)

    rng = _rng(seed, "vectors")
    with open(os.path.join(out_dir, "xqwen35_manifest.json"), "w") as f:
        json.dump(manifest_dict(cfg, quant), f, indent=2, sort_keys=True)
    _gen_embeddings(os.path.join(out_dir, "embeddings_bf16.bin"), cfg.vocab_size, H, seed)
    vec("norm_weight.f32", rng.standard_normal(H, dtype=np.float32) * np.float32(0.1))
    mat("lm_head_weight.xq4", cfg.vocab_size, H)
    kd = cfg.linear_key_head_dim * cfg.linear_num_key_heads
    vd = cfg.linear_value_head_dim * cfg.linear_num_value_heads
    for i, kind in enumerate(cfg.layer_types):
        p = f"layers_{i}_"
        vec(p + "input_layernorm_weight.f32", rng.standard_normal(H, dtype=np.float32) * np.float32(0.1))
        vec(p + "post_attention_layernorm_weight.f32",
            rng.standard_normal(H, dtype=np.float32) * np.float32(0.1))
        mat(p + "mlp_gate_proj_weight.xq4", I, H)
        mat(p + "mlp_up_proj_weight.xq4", I, H)
        mat(p + "mlp_down_proj_weight.xq4", H, I)
        if kind == "full_attention":
            qd = cfg.num_attention_heads * cfg.head_dim
            kvd = cfg.num_key_value_heads * cfg.head_dim
            mat(p + "self_attn_q_proj_weight.xq4", 2 * qd, H)
            mat(p + "self_attn_k_proj_weight.xq4", kvd, H)
            mat(p + "self_attn_v_proj_weight.xq4", kvd, H)
            mat(p + "self_attn_o_proj_weight.xq4", H, qd)
            vec(p + "self_attn_q_norm_weight.f32",
                rng.standard_normal(cfg.head_dim, dtype=np.float32) * np.float32(0.1))
            vec(p + "self_attn_k_norm_weight.f32",
                rng.standard_normal(cfg.head_dim, dtype=np.float32) * np.float32(0.1))
        else:
            nv = cfg.linear_num_value_heads
            mat(p + "linear_attn_in_proj_qkv_weight.xq4", 2 * kd + vd, H)
            mat(p + "linear_attn_in_proj_a_weight.xq4", nv, H)
            mat(p + "linear_attn_in_proj_b_weight.xq4", nv, H)
            mat(p + "linear_attn_in_proj_z_weight.xq4", vd, H)
            mat(p + "linear_attn_out_proj_weight.xq4", H, vd)
            vec(p + "linear_attn_norm_weight.f32",
                rng.standard_normal(cfg.linear_value_head_dim, dtype=np.float32) * np.float32(0.1))
            vec(p + "linear_attn_conv1d_weight.f32",
                rng.standard_normal(cfg.conv_dim * cfg.linear_conv_kernel_dim, dtype=np.float32)
                * np.float32(0.5))
            vec(p + "linear_attn_A_log.f32", rng.uniform(-3.0, 0.0, nv).astype(np.float32))
            vec(p + "linear_attn_dt_bias.f32", (rng.standard_normal(nv) - 3.0).astype(np.float32))
    with open(stamp_path, "w") as f:
        f.write(ident)
    return out_dir

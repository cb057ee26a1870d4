"""The tensor-core tile layout (xqk_mma_tiles; host only) and the arithmetic the tensor-core
kernels run on it, on the CPU.

1. The library's tiles equal an independent numpy construction of the documented layout,
   byte for byte, ragged last tile included.
2. A numpy emulation of the kernels' mma.sync m16n8k32 fragment math, reading only those tile
   bytes (codes unpacked from the nibbles of A-fragment words, x as three signed 8-bit digits
   of a 22-bit mantissa per 64-column group in B columns 0-2 / 3-5, accumulator start
   -8 * digit sum, per-column weights 256^d * 2^-S times the fp16 group scale), matches the
   oracle GEMV within 1e-5 of max |y|, and its integer sums equal sum (code - 8) * m exactly.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import PKG, rel_err

UNIT = 1088


def tiles_from_lib(packed, scales, rows, cols):
    L = PKG.lib()
    need = C.c_size_t()
    assert L.xqk_mma_tiles(packed.ctypes.data, scales.ctypes.data, rows, cols, None, 0, C.byref(need)) == -5
    out = np.zeros(need.value, np.uint8)
    got = C.c_size_t()
    assert L.xqk_mma_tiles(packed.ctypes.data, scales.ctypes.data, rows, cols, out.ctypes.data, out.size,
                           C.byref(got)) == 0
    assert got.value == need.value
    return out


def codes_of(packed, rows, cols):
    b = packed.reshape(rows, cols // 2)
    c = np.empty((rows, cols), np.uint8)
    c[:, 0::2] = b & 15
    c[:, 1::2] = b >> 4
    return c


def expected_tiles(packed, scales, rows, cols):
    """The layout as documented in include/xq_kernels.h, built with numpy indexing."""
    nt, pairs = (rows + 15) // 16, cols // 128
    code = np.full((nt * 16, cols), 8, np.uint8)
    code[:rows] = codes_of(packed, rows, cols)
    sc = np.zeros((nt * 16, cols // 64), np.float16)
    sc[:rows] = scales.reshape(rows, cols // 64).astype(np.float16)
    out = np.zeros((nt, pairs, UNIT), np.uint8)
    lane = np.arange(32)
    r, c0 = lane // 4, (lane % 4) * 4
    for t in range(nt):
        for p in range(pairs):
            for sl in range(4):
                col = 128 * p + 32 * sl + c0
                for j in range(4):
                    lo = code[16 * t + r, col + j] | (code[16 * t + r + 8, col + j] << 4)
                    hi = code[16 * t + r, col + 16 + j] | (code[16 * t + r + 8, col + 16 + j] << 4)
                    out[t, p, sl * 256 + 8 * lane + j] = lo
                    out[t, p, sl * 256 + 8 * lane + 4 + j] = hi
            s = np.stack([sc[16 * t:16 * t + 8, 2 * p], sc[16 * t:16 * t + 8, 2 * p + 1],
                          sc[16 * t + 8:16 * t + 16, 2 * p], sc[16 * t + 8:16 * t + 16, 2 * p + 1]], axis=1)
            out[t, p, 1024:] = s.reshape(-1).view(np.uint8)
    return out.reshape(-1)


def digits(x):
    """Per 64-column group: S with amax = f * 2^ex (f in [0.5, 1)), S = clamp(22 - ex), the
    round-to-nearest-even mantissa m = x * 2^S and its signed base-256 digits."""
    g = x.reshape(-1, 64).astype(np.float64)
    amax = np.abs(g).max(axis=1)
    ex = np.where(amax > 0, np.frexp(amax)[1], -126)
    S = np.clip(22 - ex, -100, 100)
    m = np.rint(g * np.exp2(S)[:, None]).astype(np.int64)
    u = m + 0x808080
    d = np.stack([((u >> (8 * k)) & 0xFF) - 128 for k in range(3)])  # [3][groups][64]
    assert np.array_equal(d[0] + 256 * d[1] + 65536 * d[2], m)
    return S, m, d


def emulate(tiles, x, rows, cols):
    """y from the tile bytes the way one warp's m16n8k32 loop computes it."""
    nt, pairs = (rows + 15) // 16, cols // 128
    T = tiles.reshape(nt, pairs, UNIT)
    S, m, d = digits(x)
    lane = np.arange(32)
    y = np.zeros(nt * 16)
    exact = np.zeros((nt * 16, cols // 64), np.int64)
    for t in range(nt):
        for p in range(pairs):
            A = np.zeros((16, 128), np.int64)  # codes of rows 16t..16t+15, columns 128p..128p+127
            for sl in range(4):
                w = T[t, p, sl * 256:sl * 256 + 256].reshape(32, 8).astype(np.int64)
                r, c0 = lane // 4, 32 * sl + (lane % 4) * 4
                for j in range(4):
                    A[r, c0 + j] = w[:, j] & 15
                    A[r + 8, c0 + j] = w[:, j] >> 4
                    A[r, c0 + 16 + j] = w[:, 4 + j] & 15
                    A[r + 8, c0 + 16 + j] = w[:, 4 + j] >> 4
            B = np.zeros((128, 8), np.int64)  # N columns: digits of group 2p (0-2), 2p+1 (3-5)
            for k in range(3):
                B[:64, k] = d[k, 2 * p]
                B[64:, 3 + k] = d[k, 2 * p + 1]
            start = np.zeros(8, np.int64)
            start[:6] = [-8 * d[k, 2 * p + g].sum() for g in range(2) for k in range(3)]
            D = A @ B + start  # the s32 accumulator of the pair (all sums exact)
            for g in range(2):
                exact[16 * t:16 * t + 16, 2 * p + g] = (D[:, 3 * g:3 * g + 3] * [1, 256, 65536]).sum(axis=1)
            sc = T[t, p, 1024:].view(np.float16).astype(np.float64).reshape(8, 4)
            s = np.concatenate([sc[:, :2], sc[:, 2:]])  # [16 rows][g0, g1]
            for n in range(6):
                g, k = n // 3, n % 3
                y[16 * t:16 * t + 16] += D[:, n] * (256.0 ** k) * 2.0 ** (-S[2 * p + g]) * s[:, g]
    code = codes_of_tiles_rows(T, rows, cols)
    ref_exact = ((code.astype(np.int64) - 8).reshape(-1, cols // 64, 64) * m[None]).sum(axis=2)
    assert np.array_equal(exact[:rows], ref_exact)
    return y[:rows]


def codes_of_tiles_rows(T, rows, cols):
    nt, pairs = T.shape[0], T.shape[1]
    code = np.zeros((nt * 16, cols), np.uint8)
    lane = np.arange(32)
    for t in range(nt):
        for p in range(pairs):
            for sl in range(4):
                w = T[t, p, sl * 256:sl * 256 + 256].reshape(32, 8)
                r, c0 = 16 * t + lane // 4, 128 * p + 32 * sl + (lane % 4) * 4
                for j in range(4):
                    code[r, c0 + j] = w[:, j] & 15
                    code[r + 8, c0 + j] = w[:, j] >> 4
                    code[r, c0 + 16 + j] = w[:, 4 + j] & 15
                    code[r + 8, c0 + 16 + j] = w[:, 4 + j] >> 4
    return code[:rows]


def seeded(rows, cols, seed):
    rng = np.random.default_rng(seed)
    packed = rng.integers(0, 256, rows * cols // 2, dtype=np.uint8)
    s = (np.abs(rng.standard_normal(rows * cols // 64)) * 0.02).astype(np.float16).astype(np.float32)
    x = rng.standard_normal(cols).astype(np.float32)
    x[::5] *= 1e-3
    x[3] = 0.0
    return packed, s, x


@pytest.mark.parametrize("rows,cols", [(37, 256), (16, 128), (5, 512), (8200, 128)])
def test_tiles_match_documented_layout(rows, cols):
    """(8200 rows: more than 512 tiles, built by several host threads.)"""
    packed, s, _ = seeded(rows, cols, rows)
    assert np.array_equal(tiles_from_lib(packed, s, rows, cols), expected_tiles(packed, s, rows, cols))


@pytest.mark.parametrize("rows,cols", [(37, 256), (21, 512)])
def test_fragment_math_matches_oracle(oracle, rows, cols):
    packed, s, x = seeded(rows, cols, 100 + rows)
    tiles = tiles_from_lib(packed, s, rows, cols)
    z = np.full(s.size, 8.0, np.float32)
    ref = oracle.port_gemv(oracle.Matrix(rows, cols, 64, 1, packed, s, z), x)
    assert rel_err(emulate(tiles, x, rows, cols), ref) <= 1e-5


def test_tile_entry_point_checks_arguments():
    L = PKG.lib()
    packed, s, _ = seeded(16, 128, 1)
    n = C.c_size_t()
    assert L.xqk_mma_tiles(packed.ctypes.data, s.ctypes.data, 16, 100, None, 0, C.byref(n)) == -1
    assert L.xqk_mma_tiles(None, s.ctypes.data, 16, 128, None, 0, C.byref(n)) == -1
    small = np.zeros(100, np.uint8)
    assert L.xqk_mma_tiles(packed.ctypes.data, s.ctypes.data, 16, 128, small.ctypes.data, small.size,
                           C.byref(n)) == -5
    assert n.value == UNIT

"""The arithmetic of the sc*q Q4_K GEMM variant, emulated on the CPU against the
oracle: the bit recipe that turns two packed nibbles into fp16 lanes, the exact
fp16 product sc*q, and the per-superblock decomposition
y = sum_sb d * sum(sc q x) - dmin * sum_j m_j (xs_hi + xs_lo)."""
from __future__ import annotations

import numpy as np

from oracle import gguf_oracle as O
from tests.helpers import TOL


def _byte_perm(x: int, y: int, sel: int) -> int:
    """CUDA __byte_perm (default mode): result byte i = byte (sel >> 4i) & 7 of y:x."""
    src = (y << 32) | x
    return sum(((src >> (8 * ((sel >> (4 * i)) & 7))) & 0xFF) << (8 * i) for i in range(4))


def test_nibble_lanes_bit_recipe():
    rng = np.random.default_rng(0)
    for word in [0, 0xFFFFFFFF, 0x12345678, 0xF0E1D2C3] + [int(v) for v in rng.integers(0, 2**32, 200)]:
        b = [(word >> (8 * i)) & 0xFF for i in range(4)]
        for sel, (b0, b1) in ((0x5140, (b[0], b[1])), (0x5342, (b[2], b[3]))):
            t = _byte_perm(word, 0x6464, sel)
            lo = t & 0xFF0FFF0F
            hi = ((t >> 4) & 0x000F000F) | 0x64006400
            assert lo & 0xFFFF == 0x6400 | (b0 & 15) and lo >> 16 == 0x6400 | (b1 & 15)
            assert hi & 0xFFFF == 0x6400 | (b0 >> 4) and hi >> 16 == 0x6400 | (b1 >> 4)
            # the fp16 value of 0x6400 | q is 1024 + q
            assert np.array([lo & 0xFFFF], np.uint16).view(np.float16)[0] == 1024 + (b0 & 15)


def test_sc_times_q_is_exact_in_fp16():
    q = np.arange(16, dtype=np.float64)[:, None]
    sc = np.arange(64, dtype=np.float64)[None, :]
    fused = (1024 + q) * sc + (-1024 * sc)        # exact, then one rounding (the hfma2)
    assert np.array_equal(fused.astype(np.float16).astype(np.float64), q * sc)
    assert np.array_equal((-1024 * sc).astype(np.float16).astype(np.float64), -1024 * sc)
    assert (q * sc).max() <= 945


def test_superblock_decomposition_matches_oracle():
    n, k, m = 48, 1024, 5
    raw = O.make_weights(n, k, O.Q4_K, seed=3)
    x16 = O.make_activations(m, k, seed=4).astype(np.float16).astype(np.float32)
    blk = raw.reshape(n, k // 256, 144)
    d = blk[:, :, 0:2].copy().view(np.float16)[..., 0].astype(np.float32)
    dmin = blk[:, :, 2:4].copy().view(np.float16)[..., 0].astype(np.float32)
    sc, mn = O.q4_k_scale_min(blk[:, :, 4:16].reshape(-1, 12))
    sc = sc.reshape(n, k // 256, 8).astype(np.float32)
    mn = mn.reshape(n, k // 256, 8).astype(np.float32)
    qs = blk[:, :, 16:144].reshape(n, k // 256, 4, 32)
    q = np.stack([qs & 15, qs >> 4], axis=3).reshape(n, k // 256, 8, 32).astype(np.float32)
    a = (sc[..., None] * q)                                   # the MMA's A operand, exact
    assert np.array_equal(a.astype(np.float16).astype(np.float32), a)
    xr = x16.reshape(m, k // 256, 8, 32)
    acc_q = np.einsum("nsjk,msjk->nms", a.astype(np.float64), xr.astype(np.float64))
    xs = xr.sum(axis=3, dtype=np.float32)                    # fp32 sub-block sums
    hi = xs.astype(np.float16).astype(np.float32)
    lo = (xs - hi).astype(np.float16).astype(np.float32)
    acc_m = np.einsum("nsj,msj->nms", mn.astype(np.float64), (hi + lo).astype(np.float64))
    y = np.einsum("ns,nms->mn", d.astype(np.float64), acc_q) - np.einsum("ns,nms->mn", dmin.astype(np.float64), acc_m)
    ref = O.matmul_ref(x16, raw, O.Q4_K, n, k)
    assert O.rel_err(y.astype(np.float32), ref) <= TOL * 0.01

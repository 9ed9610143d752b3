"""Generate the committed golden vectors for the GGUF block formats.

Run from the repository root in a container where gguf-py (the reference's
pinned dependency, ``pyproject.toml:14`` of maci0/vllm-webgpu; 0.19.0 here)
is importable:

    python tests/golden/make_golden.py

Every expected output below comes from gguf-py itself
(``gguf.quants.dequantize`` / ``gguf.quants.quantize``), never from this
repository's oracle, so the fixtures pin the oracle and the CUDA kernels to
the reference dependency. The fixtures are small (a few hundred KB total) and
need nothing but numpy to read.

Contents of ``golden_<qtype>.npz``:
  blocks_rand   random bytes with finite fp16 scale fields (bit-pattern sweep)
  deq_rand      gguf dequant of blocks_rand (fp32)
  blocks_edge   hand-built edge blocks: d = 0, +-subnormal, +-65504, every
                quant value, zero / max sub-scales, non-finite d (inf, nan)
  deq_edge      gguf dequant of blocks_edge (fp32; NaN where gguf gives NaN)
  mm_w, mm_x, mm_y32, mm_shape
                a small matmul: W (gguf-valid blocks, N x row_bytes), x
                (bf16-representable fp32, M x K) and y = x @ dequant(W).T in
                numpy fp32 -- the reference's fp32 dequantize-then-matmul
  quant_w, quant_q   (Q8_0, Q4_0 only) seeded fp32 weights and gguf's own
                quantize() bytes for them
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.abspath(os.path.join(HERE, "..", "..")))

import gguf  # noqa: E402
from gguf.quants import dequantize as g_deq, quantize as g_quant  # noqa: E402

from oracle import gguf_oracle as O  # noqa: E402  (only for the Q4_K/Q6_K packers)

# fp16 offsets of the scale fields inside each block
F16_FIELDS = {O.Q8_0: [0], O.Q4_0: [0], O.Q4_K: [0, 2], O.Q6_K: [208]}


def _set_f16(blk: np.ndarray, off: int, vals) -> None:
    blk[:, off:off + 2] = np.asarray(vals, np.float16).reshape(-1, 1).view(np.uint8)


def rand_blocks(qt: int, n: int, rng) -> np.ndarray:
    ts = O.type_size(qt)
    blk = rng.integers(0, 256, size=(n, ts), dtype=np.uint8)
    for off in F16_FIELDS[qt]:
        _set_f16(blk, off, rng.standard_normal(n) * rng.choice([1e-4, 1e-2, 1.0, 100.0], n))
    return blk


def edge_blocks(qt: int, rng) -> np.ndarray:
    ts = O.type_size(qt)
    rows = []
    specials = [0.0, -0.0, 6e-8, -6e-8, 6.1e-5, 65504.0, -65504.0, 1.0, -0.5]
    for s in specials:
        b = rng.integers(0, 256, size=(1, ts), dtype=np.uint8)
        for off in F16_FIELDS[qt]:
            _set_f16(b, off, [s])
        rows.append(b)
    # every quant value: walk payload bytes through 0..255
    for start in (0, 128):
        b = np.zeros((1, ts), np.uint8)
        payload = [i for i in range(ts) if all(not (o <= i < o + 2) for o in F16_FIELDS[qt])]
        for t, i in enumerate(payload):
            b[0, i] = (start + t * 37) & 0xFF
        for off in F16_FIELDS[qt]:
            _set_f16(b, off, [0.0123])
        rows.append(b)
    # all-zero and all-0xFF payloads
    for fill in (0x00, 0xFF):
        b = np.full((1, ts), fill, np.uint8)
        for off in F16_FIELDS[qt]:
            _set_f16(b, off, [0.5])
        rows.append(b)
    # non-finite scales (gguf propagates inf / nan)
    for s in (np.inf, -np.inf, np.nan):
        b = rng.integers(0, 256, size=(1, ts), dtype=np.uint8)
        _set_f16(b, F16_FIELDS[qt][0], [s])
        rows.append(b)
    return np.concatenate(rows, axis=0)


def main() -> None:
    rng = np.random.default_rng(20261201)
    for qt in (O.Q8_0, O.Q4_0, O.Q4_K, O.Q6_K):
        name = O.QTYPES[qt][0]
        gt = gguf.GGMLQuantizationType(qt)
        out = {}
        br = rand_blocks(qt, 64, rng)
        out["blocks_rand"] = br
        out["deq_rand"] = g_deq(br, gt).reshape(br.shape[0], -1)
        be = edge_blocks(qt, rng)
        out["blocks_edge"] = be
        with np.errstate(invalid="ignore", over="ignore"):
            out["deq_edge"] = g_deq(be, gt).reshape(be.shape[0], -1)
        # small matmul case
        n, k, m = 24, 512, 3
        w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
        if qt in (O.Q8_0, O.Q4_0):
            wq = g_quant(w, gt)
        else:
            wq = O.quantize(w, qt)
        x = rng.standard_normal((m, k)).astype(np.float32)
        x = (x.view(np.uint32) & np.uint32(0xFFFF0000)).view(np.float32)  # bf16-exact
        wd = g_deq(wq, gt).reshape(n, k)
        out["mm_w"] = np.ascontiguousarray(wq).reshape(n, -1)
        out["mm_x"] = x
        out["mm_y32"] = (x @ wd.T).astype(np.float32)
        out["mm_shape"] = np.array([m, n, k], np.int64)
        if qt in (O.Q8_0, O.Q4_0):
            qw = (rng.standard_normal((8, 256)) * 0.02).astype(np.float32)
            out["quant_w"] = qw
            out["quant_q"] = g_quant(qw, gt)
        path = os.path.join(HERE, f"golden_{name.lower()}.npz")
        np.savez_compressed(path, **out)
        print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()

"""Quantize fp32 weights to GGUF blocks with torch ops (runs on the GPU).

The reference only ever loads pre-quantized GGUF files or converts
safetensors bf16 -> f16 (vllm_webgpu/quant/gguf_loader.py:51-92). This module
lets the loader turn dense weights into the GGUF formats the B200 kernels
read, on the device, without a round trip through numpy:

* Q8_0 / Q4_0 follow gguf-py's own quantizers (gguf quants.py:381-393 and
  :222-238) operation for operation, so the bytes are identical to
  ``gguf.quants.quantize``.
* Q4_K / Q6_K: gguf-py 0.19.0 has no quantizer for these, so a simple
  per-sub-block min/max fit is used (documented in each function); the
  output is a valid GGUF block stream that any GGUF dequantizer decodes.

All arithmetic is fp32 with round-to-nearest-even (``torch.round``) or the
round-half-away-from-zero gguf uses for Q8_0, in the order written, so CPU
and CUDA tensors give the same bytes.
"""
from __future__ import annotations

import torch

from ..formats import Q4_0, Q4_K, Q6_K, Q8_0, QUANT_SIZES, GGUFQuantTensor, qtype_of, row_bytes


def _f16_bytes(v: torch.Tensor) -> torch.Tensor:
    """fp32 [n] -> fp16 -> 2 little-endian bytes per value, uint8 [n, 2]."""
    return v.to(torch.float16).contiguous().view(torch.uint8).reshape(-1, 2)


def _roundf(v: torch.Tensor) -> torch.Tensor:
    a = v.abs()
    fl = torch.floor(a)
    return torch.sign(v) * (fl + torch.floor(2 * (a - fl)))


def _q8_0(w: torch.Tensor) -> torch.Tensor:
    blk = w.reshape(-1, 32)
    d = blk.abs().amax(dim=1, keepdim=True) / 127.0
    inv = torch.where(d == 0, torch.zeros_like(d), 1.0 / d)
    q = _roundf(blk * inv).to(torch.int8).view(torch.uint8)
    return torch.cat([_f16_bytes(d.reshape(-1)), q], dim=1)


def _q4_0(w: torch.Tensor) -> torch.Tensor:
    blk = w.reshape(-1, 32)
    imax = blk.abs().argmax(dim=1, keepdim=True)
    mx = torch.gather(blk, 1, imax)
    d = mx / -8.0
    inv = torch.where(d == 0, torch.zeros_like(d), 1.0 / d)
    q = torch.trunc(blk * inv + 8.5).to(torch.uint8).clamp(0, 15)
    qs = q[:, :16] | (q[:, 16:] << 4)
    return torch.cat([_f16_bytes(d.reshape(-1)), qs], dim=1)


def _q4_k(w: torch.Tensor) -> torch.Tensor:
    """Sub-block of 32: offset m = max(0, -min), step = (max + m)/15; d =
    max(step)/63 and dmin = max(m)/63 stored as fp16; sc/m = rounded ratios
    (6 bits); q = round((w + dmin*m)/(d*sc)) clamped to 0..15."""
    sb = w.reshape(-1, 8, 32)
    n = sb.shape[0]
    lo = sb.amin(dim=2)
    hi = sb.amax(dim=2)
    off = torch.clamp(-lo, min=0.0)
    step = (hi + off) / 15.0
    d = (step.amax(dim=1) / 63.0).to(torch.float16)
    dmin = (off.amax(dim=1) / 63.0).to(torch.float16)
    d32 = d.float()[:, None]
    dm32 = dmin.float()[:, None]
    zero = torch.zeros((), dtype=torch.float32, device=w.device)
    sc = torch.where(d32 > 0, torch.round(step / d32), zero).clamp(0, 63).to(torch.uint8)
    mn = torch.where(dm32 > 0, torch.round(off / dm32), zero).clamp(0, 63).to(torch.uint8)
    dsc = (d32 * sc.float())[:, :, None]
    dmm = (dm32 * mn.float())[:, :, None]
    q = torch.where(dsc > 0, torch.round((sb + dmm) / dsc), zero).clamp(0, 15).to(torch.uint8)
    out = torch.zeros((n, 144), dtype=torch.uint8, device=w.device)
    out[:, 0:2] = _f16_bytes(d.float())
    out[:, 2:4] = _f16_bytes(dmin.float())
    s = torch.empty((n, 12), dtype=torch.uint8, device=w.device)
    s[:, 0:4] = (sc[:, 0:4] & 63) | ((sc[:, 4:8] >> 4) << 6)
    s[:, 4:8] = (mn[:, 0:4] & 63) | ((mn[:, 4:8] >> 4) << 6)
    s[:, 8:12] = (sc[:, 4:8] & 15) | ((mn[:, 4:8] & 15) << 4)
    out[:, 4:16] = s
    qs = q.reshape(n, 4, 2, 32)
    out[:, 16:144] = (qs[:, :, 0, :] | (qs[:, :, 1, :] << 4)).reshape(n, 128)
    return out


def _q6_k(w: torch.Tensor) -> torch.Tensor:
    """Sub-block of 16: step = -(signed max-magnitude weight)/32; d =
    max|step|/127 (fp16); int8 sc = round(step/d); q = round(w/(d*sc))
    clamped to -32..31, stored as q+32 split into 4 low + 2 high bits."""
    sb = w.reshape(-1, 16, 16)
    n = sb.shape[0]
    imax = sb.abs().argmax(dim=2, keepdim=True)
    amax = torch.gather(sb, 2, imax)[:, :, 0]
    step = -amax / 32.0
    d = (step.abs().amax(dim=1) / 127.0).to(torch.float16)
    d32 = d.float()[:, None]
    zero = torch.zeros((), dtype=torch.float32, device=w.device)
    sc = torch.where(d32 > 0, torch.round(step / d32), zero).clamp(-128, 127).to(torch.int8)
    dl = (d32 * sc.float())[:, :, None]
    q = (torch.where(dl != 0, torch.round(sb / dl), zero).clamp(-32, 31).to(torch.int16) + 32).to(torch.uint8)
    q = q.reshape(n, 2, 4, 32)  # (h, u, c)
    out = torch.zeros((n, 210), dtype=torch.uint8, device=w.device)
    ql = torch.stack([(q[:, :, 0] & 15) | ((q[:, :, 2] & 15) << 4),
                      (q[:, :, 1] & 15) | ((q[:, :, 3] & 15) << 4)], dim=2)  # (n, h, 2, 32)
    qh = torch.zeros((n, 2, 32), dtype=torch.uint8, device=w.device)
    for u in range(4):
        qh |= ((q[:, :, u] >> 4) & 3) << (2 * u)
    out[:, 0:128] = ql.reshape(n, 128)
    out[:, 128:192] = qh.reshape(n, 64)
    out[:, 192:208] = sc.view(torch.uint8)
    out[:, 208:210] = _f16_bytes(d.float())
    return out


_PACKERS = {Q8_0: _q8_0, Q4_0: _q4_0, Q4_K: _q4_k, Q6_K: _q6_k}


@torch.no_grad()
def quantize(w: torch.Tensor, qtype, row_chunk: int = 4096) -> GGUFQuantTensor:
    """Quantize a dense [N, K] weight (any float dtype, any device) to GGUF
    blocks on the same device. Rows are processed in chunks to bound the
    temporary memory."""
    qt = qtype_of(qtype)
    if w.dim() != 2:
        raise ValueError("expected a 2-D [N, K] weight")
    n, k = w.shape
    rb = row_bytes(qt, k)
    out = torch.empty((n, rb), dtype=torch.uint8, device=w.device)
    for r0 in range(0, n, row_chunk):
        r1 = min(n, r0 + row_chunk)
        chunk = w[r0:r1].to(torch.float32).contiguous()
        out[r0:r1] = _PACKERS[qt](chunk).reshape(r1 - r0, rb)
    return GGUFQuantTensor(out, qt, (n, k))


def random_weights(n: int, k: int, qtype, seed: int = 0, std: float = 0.02,
                   device="cuda") -> GGUFQuantTensor:
    """Seeded synthetic weights W ~ N(0, std) quantized to ``qtype`` on ``device``."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    out = None
    qt = qtype_of(qtype)
    rb = row_bytes(qt, k)
    out = torch.empty((n, rb), dtype=torch.uint8, device=device)
    step = 2048
    for r0 in range(0, n, step):
        r1 = min(n, r0 + step)
        w = torch.randn((r1 - r0, k), generator=g, device=device, dtype=torch.float32) * std
        out[r0:r1] = _PACKERS[qt](w).reshape(r1 - r0, rb)
    return GGUFQuantTensor(out, qt, (n, k))


__all__ = ["quantize", "random_weights", "QUANT_SIZES"]

"""GGUF block formats handled by the B200 path and the quantized-tensor type.

The reference loader uploads raw GGUF bytes and drops the tensor type and the
logical shape (vllm_webgpu/quant/gguf_loader.py:152-159); here both travel
with the bytes so the kernels can be dispatched by type.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

# GGMLQuantizationType ids (gguf constants.py:4059-4073)
Q4_0, Q8_0, Q4_K, Q6_K = 2, 8, 12, 14
F32, F16, BF16 = 0, 1, 30

# (name, weights per block, bytes per block) -- gguf constants.py:4231-4245
QUANT_SIZES = {
    Q4_0: ("Q4_0", 32, 18),
    Q8_0: ("Q8_0", 32, 34),
    Q4_K: ("Q4_K", 256, 144),
    Q6_K: ("Q6_K", 256, 210),
}
SUPPORTED = tuple(QUANT_SIZES)
BY_NAME = {v[0]: k for k, v in QUANT_SIZES.items()}


def qtype_of(q) -> int:
    """Accept an int id, a name ("Q4_K") or a gguf GGMLQuantizationType."""
    if isinstance(q, str):
        if q.upper() not in BY_NAME:
            raise ValueError(f"unsupported quantization type {q!r}")
        return BY_NAME[q.upper()]
    q = int(q)
    if q not in QUANT_SIZES:
        raise ValueError(f"unsupported quantization type {q}")
    return q


def row_bytes(qtype: int, k: int) -> int:
    name, bs, ts = QUANT_SIZES[qtype]
    if k % bs:
        raise ValueError(f"K={k} is not a multiple of the {name} block size {bs}")
    return k // bs * ts


@dataclass
class GGUFQuantTensor:
    """A GGUF-quantized [N, K] weight resident on a CUDA device.

    ``data`` is uint8 [N, K/block*type_size]: the GGUF blocks byte for byte,
    exactly as gguf.GGUFReader returns them.
    """

    data: torch.Tensor
    qtype: int
    shape: tuple[int, int]

    def __post_init__(self) -> None:
        self.qtype = qtype_of(self.qtype)
        n, k = self.shape
        rb = row_bytes(self.qtype, k)
        if self.data.dtype != torch.uint8 or tuple(self.data.shape) != (n, rb):
            raise ValueError(
                f"expected uint8 [{n}, {rb}] blocks for {QUANT_SIZES[self.qtype][0]} {self.shape}, "
                f"got {self.data.dtype} {tuple(self.data.shape)}")

    @property
    def n(self) -> int:
        return self.shape[0]

    @property
    def k(self) -> int:
        return self.shape[1]

    @property
    def device(self) -> torch.device:
        return self.data.device

    @property
    def nbytes(self) -> int:
        return self.data.numel()

    def to(self, device) -> "GGUFQuantTensor":
        return GGUFQuantTensor(self.data.to(device), self.qtype, self.shape)

    def rows(self, start: int, stop: int) -> "GGUFQuantTensor":
        """Output rows [start, stop) -- a column split of y = x W^T."""
        return GGUFQuantTensor(self.data[start:stop].contiguous(), self.qtype, (stop - start, self.k))

    def cols(self, start: int, stop: int) -> "GGUFQuantTensor":
        """Input columns [start, stop) -- a row split of y = x W^T (block aligned)."""
        _, bs, ts = QUANT_SIZES[self.qtype]
        if start % bs or stop % bs:
            raise ValueError(f"K split [{start}, {stop}) is not aligned to the {bs}-weight block")
        b0, b1 = start // bs * ts, stop // bs * ts
        return GGUFQuantTensor(self.data[:, b0:b1].contiguous(), self.qtype, (self.n, stop - start))

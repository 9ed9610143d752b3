"""Host-side routing between the decode GEMV and the GEMM (CPU only): which
kernel kind a shape gets is faked, the policy on top of it is checked."""
from __future__ import annotations

import pytest
import torch


def _w(qt: int, n: int = 256, k: int = 4096):
    from vllm_webgpu_b200.formats import GGUFQuantTensor, row_bytes
    return GGUFQuantTensor(torch.zeros((n, row_bytes(qt, k)), dtype=torch.uint8), qt, (n, k))


@pytest.mark.parametrize("qt,m,kind,expect", [
    (12, 1, 2, True),    # Q4_K on the integer GEMV
    (12, 4, 1, True),    # Q4_K on the fp16 GEMV
    (12, 8, 0, False),   # Q4_K where only the streaming GEMV fits -> fused-dequant GEMM
    (2, 8, 0, True),     # Q4_0: the GEMV stays (no fused GEMM for it)
    (8, 8, 0, True),     # Q8_0: likewise
    (14, 3, 0, True),    # Q6_K: likewise
    (14, 1, -3, False),  # Q6_K rows no decode GEMV can stage (ERR_ALIGN) -> GEMM
    (12, 9, 2, False),   # above the GEMV's 8 tokens
    (12, 0, 2, False),
])
def test_gemv_preferred_policy(monkeypatch, qt, m, kind, expect):
    from vllm_webgpu_b200 import ops
    calls = []

    def fake_kernel(mm, w, x_dtype=torch.bfloat16):
        calls.append(mm)
        return kind

    monkeypatch.setattr(ops, "gemv_kernel", fake_kernel)
    assert ops.gemv_preferred(m, _w(qt)) is expect
    if not 1 <= m <= ops.GEMV_MAX_M:
        assert calls == []  # the device is only asked about decode shapes


def test_kernel_kind_codes_match_header():
    """The Python kind codes are the header's GGUFMM_GEMV_* values."""
    import os
    import re
    from vllm_webgpu_b200 import ops
    hdr = open(os.path.join(os.path.dirname(__file__), "..", "include", "ggufmm.h")).read()
    vals = dict(re.findall(r"GGUFMM_GEMV_(STREAM|F16|INT8)\s*=\s*(\d+)", hdr))
    assert (int(vals["STREAM"]), int(vals["F16"]), int(vals["INT8"])) == (ops.GEMV_STREAM, ops.GEMV_F16,
                                                                         ops.GEMV_INT8)


def test_model_grouping_needs_cuda_inputs():
    """The model's grouped projection path declines host tensors (the caller then
    takes the per-projection path, which reports the missing device)."""
    from vllm_webgpu_b200.models.llama import LlamaB200Model
    model = LlamaB200Model(None, device="cpu")
    x = torch.zeros((2, 4096), dtype=torch.bfloat16)
    bufs = [torch.empty((2, 256)), torch.empty((2, 256))]
    assert model._fused(x, [_w(12), _w(12)], bufs) is False

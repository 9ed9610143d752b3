"""ggufmm_gemm_noalloc: the GEMM for callers that cannot allocate device memory.

Some callers of this library have no way to get device memory when they call
it -- their host owns the GPU's memory through a fixed pool and exposes no
allocator over the FFI, or they must not allocate once they are serving -- so
they cannot supply the workspace ggufmm_gemm needs. ggufmm_gemm_noalloc uses a
scratch array inside the library instead. These tests call it through the C
ABI (ctypes, raw device pointers) and check it against ggufmm_gemm on the same
inputs, twice in a row (the second call reuses the scratch the first one
left behind). The file name sorts last so a stop-at-first-failure run has
already run every other test; it also passes alone in a fresh process.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import gguf_oracle as O
from tests.helpers import TOL

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 64 << 20  # GGUFMM_NOALLOC_SCRATCH_BYTES in include/ggufmm.h


def _lib():
    from vllm_webgpu_b200 import _lib
    return _lib.lib()


def _problem(qt, m, n, k, seed):
    raw = O.make_weights(n, k, qt, seed=seed)
    q = torch.from_numpy(raw).cuda()
    x = torch.from_numpy(O.make_activations(m, k, seed=seed + 1)).to(torch.bfloat16).cuda()
    return raw, q, x


def _with_workspace(q, qt, n, k, x, m):
    lib = _lib()
    ws_bytes = lib.ggufmm_gemm_workspace_size(qt, m, n, k)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    y = torch.empty((m, n), dtype=torch.float32, device="cuda")
    st = lib.ggufmm_gemm(q.data_ptr(), qt, n, k, x.data_ptr(), 2, m, k, y.data_ptr(), 0, n,
                         ws.data_ptr(), ws_bytes, torch.cuda.current_stream().cuda_stream)
    assert st == 0
    return y


def _no_alloc(q, qt, n, k, x, m):
    y = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    st = _lib().ggufmm_gemm_noalloc(q.data_ptr(), qt, n, k, x.data_ptr(), 2, m, k, y.data_ptr(), 0, n,
                                    torch.cuda.current_stream().cuda_stream)
    assert st == 0
    return y


@pytest.mark.parametrize("qt,m,n,k", [(O.Q4_K, 64, 2048, 4096), (O.Q6_K, 300, 1024, 4096),
                                      (O.Q8_0, 17, 4096, 2048), (O.Q4_0, 128, 777, 1024)])
def test_noalloc_matches_workspace_gemm_twice(cuda, qt, m, n, k):
    for call in range(2):
        raw, q, x = _problem(qt, m, n, k, seed=10 * call + qt)
        ref_ws = _with_workspace(q, qt, n, k, x, m)
        got = _no_alloc(q, qt, n, k, x, m)
        torch.cuda.synchronize()
        got, ref_ws = got.cpu().numpy(), ref_ws.cpu().numpy()
        assert np.isfinite(got).all()
        assert O.rel_err(got, ref_ws.astype(np.float64)) <= TOL
        assert O.rel_err(got, O.matmul_ref(x.float().cpu().numpy(), raw, qt, n, k)) <= TOL


def test_noalloc_rejects_problems_beyond_the_scratch(cuda):
    from vllm_webgpu_b200 import _lib as L
    n, k, m = 8192, 4096, 16  # 64 MiB of fp16 weights alone: over the limit
    assert n * k * 2 + m * k * 2 > SCRATCH_BYTES
    q = torch.zeros((n, k // 256 * 144), dtype=torch.uint8, device="cuda")
    x = torch.zeros((m, k), dtype=torch.bfloat16, device="cuda")
    y = torch.zeros((m, n), dtype=torch.float32, device="cuda")
    st = _lib().ggufmm_gemm_noalloc(q.data_ptr(), O.Q4_K, n, k, x.data_ptr(), 2, m, k, y.data_ptr(), 0, n, None)
    assert st == L.ERR_WORKSPACE
    torch.cuda.synchronize()
    assert torch.count_nonzero(y).item() == 0  # nothing was launched

"""The C ABI: the library loads, exports every declared symbol and rejects bad
arguments on the host before touching a GPU (CPU only)."""
from __future__ import annotations

import ctypes

import pytest

from tests.helpers import header_functions


@pytest.fixture(scope="module")
def lib():
    from vllm_webgpu_b200 import _lib
    return _lib.load()


def test_header_declares_the_entry_points():
    names = header_functions()
    for must in ("ggufmm_dequantize", "ggufmm_gemv", "ggufmm_gemm", "ggufmm_mul_mat",
                 "ggufmm_gemm_workspace_size", "ggufmm_version"):
        assert must in names


def test_every_declared_symbol_is_exported(lib):
    from vllm_webgpu_b200 import _lib
    for name in header_functions():
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_geometry(lib):
    assert lib.ggufmm_version() >= 100
    assert [lib.ggufmm_block_size(q) for q in (2, 8, 12, 14)] == [32, 32, 256, 256]
    assert [lib.ggufmm_type_size(q) for q in (2, 8, 12, 14)] == [18, 34, 144, 210]
    assert lib.ggufmm_block_size(3) == 0 and lib.ggufmm_type_size(99) == 0


def test_workspace_size(lib):
    assert lib.ggufmm_gemm_workspace_size(12, 512, 14336, 4096) == 14336 * 4096 * 2 + 512 * 4096 * 2
    # M = 2048: 896 tiles of 256 tokens on 148 SMs leave 8 in the last wave, each cut
    # in 8 K slices whose fp32 partial tiles (256 x 128) follow the fp16 operands
    assert lib.ggufmm_gemm_workspace_size(12, 2048, 14336, 4096) == (14336 * 4096 * 2 + 2048 * 4096 * 2
                                                                     + 8 * 8 * 256 * 128 * 4)
    assert lib.ggufmm_gemm_workspace_size(12, 1, 10, 100) == 0  # K not a block multiple
    assert lib.ggufmm_gemm_workspace_size(99, 1, 10, 256) == 0


def _gemv(lib, q=1 << 20, qt=12, n=16, k=256, x=1 << 20, xt=2, m=1, ldx=256, y=1 << 20, yt=0, ldy=16):
    return lib.ggufmm_gemv(q, qt, n, k, x, xt, m, ldx, y, yt, ldy, None)


def test_host_side_validation(lib):
    from vllm_webgpu_b200 import _lib as L
    assert _gemv(lib, q=None) == L.ERR_ARG
    assert _gemv(lib, qt=3) == L.ERR_QTYPE
    assert _gemv(lib, k=100) == L.ERR_SHAPE
    assert _gemv(lib, m=9) == L.ERR_SHAPE
    assert _gemv(lib, m=0) == L.ERR_SHAPE
    assert _gemv(lib, ldx=128) == L.ERR_SHAPE
    assert _gemv(lib, xt=7) == L.ERR_DTYPE
    assert _gemv(lib, q=(1 << 20) + 8) == L.ERR_ALIGN
    assert lib.ggufmm_dequantize(None, 12, 1, 256, 1 << 20, 0, None) == L.ERR_ARG
    assert lib.ggufmm_dequantize(1 << 20, 12, 1, 256, 1 << 20, 2, None) == L.ERR_DTYPE
    assert lib.ggufmm_gemm(1 << 20, 12, 16, 256, 1 << 20, 2, 32, 256, 1 << 20, 0, 16, None, 0, None) == L.ERR_WORKSPACE
    assert b"block size" in lib.ggufmm_status_string(L.ERR_SHAPE)


def test_status_maps_to_reference_exceptions():
    from vllm_webgpu_b200 import _lib as L
    with pytest.raises(ValueError):
        L.check(L.ERR_SHAPE, "x")
    with pytest.raises(L.GGUFMMError):
        L.check(L.ERR_CUDA, "x")
    L.check(L.OK, "x")


def test_ops_refuse_cpu_tensors():
    import torch
    from vllm_webgpu_b200 import ops
    from vllm_webgpu_b200.formats import GGUFQuantTensor
    w = GGUFQuantTensor(torch.zeros((4, 144), dtype=torch.uint8), 12, (4, 256))
    with pytest.raises(ValueError, match="CUDA"):
        ops.gemv(torch.zeros((1, 256)), w)
    with pytest.raises(ValueError, match="CUDA"):
        ops.dequantize(w)


def test_swiglu_and_allreduce_host_validation(lib):
    """The fused SwiGLU and all-reduce entry points reject bad arguments on the
    host, before any device query or launch."""
    from vllm_webgpu_b200 import _lib as L
    P = 1 << 20

    def sw(qg=P, qu=P, qt=12, n=16, k=256, m=1):
        return lib.ggufmm_gemv_swiglu(qg, qu, qt, n, k, P, 2, m, k, P, 0, n, None)

    assert sw(qu=None) == L.ERR_ARG
    assert sw(qg=None) == L.ERR_ARG
    assert sw(qt=3) == L.ERR_QTYPE
    assert sw(m=9) == L.ERR_SHAPE
    assert sw(qu=P + 8) == L.ERR_ALIGN

    bufs = (ctypes.c_void_p * 2)(P, P + 4096)

    def ar(world=2, rank=0, m=1, m_max=8, epoch=1, b=bufs):
        return lib.ggufmm_gemv_allreduce(P, 12, 16, 256, P, 2, m, 256, P, 0, 16, b, world, rank, m_max, epoch, None)

    assert ar(b=None) == L.ERR_ARG
    assert ar(world=1) == L.ERR_ARG
    assert ar(world=9) == L.ERR_ARG
    assert ar(rank=2) == L.ERR_ARG
    assert ar(m=4, m_max=2) == L.ERR_ARG
    assert ar(epoch=0) == L.ERR_ARG
    assert ar(b=(ctypes.c_void_p * 2)(P, P + 8)) == L.ERR_ALIGN
    # exchange buffer: 2 parities x world x m_max x n fp32, then 2 x world x row-block flags
    # 4 KB of per-CTA generation counters + [2 parities][2 sources][8 tokens][8192] 8-byte tagged words
    assert lib.ggufmm_gemv_allreduce_buffer_bytes(8192, 8, 2) == 4096 + 2 * 2 * 8 * 8192 * 8
    assert lib.ggufmm_gemv_allreduce_buffer_bytes(8192, 9, 2) == 0
    assert lib.ggufmm_gemv_allreduce_buffer_bytes(8192, 1, 1) == 0


def test_gemv_kernel_query_host_validation(lib):
    """ggufmm_gemv_kernel rejects bad shapes, qtypes and dtypes before any device
    query; on a host without a sm_100 device a valid shape reports a device or
    CUDA error, never a kernel kind."""
    from vllm_webgpu_b200 import _lib as L
    assert lib.ggufmm_gemv_kernel(3, 4096, 4096, 1, 2) == L.ERR_QTYPE
    assert lib.ggufmm_gemv_kernel(12, 4096, 4096, 9, 2) == L.ERR_SHAPE
    assert lib.ggufmm_gemv_kernel(12, 4096, 4096, 0, 2) == L.ERR_SHAPE
    assert lib.ggufmm_gemv_kernel(12, 4096, 4000, 1, 2) == L.ERR_SHAPE
    assert lib.ggufmm_gemv_kernel(12, 0, 4096, 1, 2) == L.ERR_SHAPE
    assert lib.ggufmm_gemv_kernel(12, 4096, 4096, 1, 7) == L.ERR_DTYPE
    import torch
    if not torch.cuda.is_available():
        assert lib.ggufmm_gemv_kernel(12, 4096, 4096, 1, 2) < 0



def test_gemm_grouped_host_validation(lib):
    """ggufmm_gemm_grouped rejects bad arguments before touching the device."""
    from vllm_webgpu_b200 import _lib as L
    P = 1 << 20
    qs = (ctypes.c_void_p * 2)(P, P)
    ns = (ctypes.c_int64 * 2)(256, 128)
    ys = (ctypes.c_void_p * 2)(P, P)
    ld = (ctypes.c_int64 * 2)(256, 128)

    def gg(nseg=2, q=qs, n=ns, qt=12, k=256, m=16, y=ys, ldy=ld, ws=P, wsb=1 << 30):
        return lib.ggufmm_gemm_grouped(nseg, q, n, qt, k, P, 2, m, k, y, 0, ldy, ws, wsb, None)

    assert gg(q=None) == L.ERR_ARG
    assert gg(nseg=0) == L.ERR_SHAPE
    assert gg(nseg=5) == L.ERR_SHAPE
    assert gg(qt=3) == L.ERR_QTYPE
    assert gg(k=100) == L.ERR_SHAPE
    assert gg(ws=None) == L.ERR_WORKSPACE
    assert gg(wsb=1024) == L.ERR_WORKSPACE



def test_gemv_residual_host_validation(lib):
    """ggufmm_gemv_residual rejects bad arguments before touching the device."""
    from vllm_webgpu_b200 import _lib as L
    P = 1 << 20

    def gr(r=P, m=1, ldr=16, qt=12, yd=0):
        return lib.ggufmm_gemv_residual(P, qt, 16, 256, P, 2, m, 256, P, yd, 16, r, ldr, None)

    assert gr(r=None) == L.ERR_ARG
    assert gr(m=9) == L.ERR_SHAPE
    assert gr(ldr=15) == L.ERR_SHAPE
    assert gr(qt=3) == L.ERR_QTYPE
    assert gr(r=P + 2) == L.ERR_ALIGN

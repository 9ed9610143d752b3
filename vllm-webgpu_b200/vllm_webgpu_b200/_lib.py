"""ctypes binding of libggufmm.so (the C ABI declared in include/ggufmm.h).

The library is built in-tree by ``vllm-webgpu_b200/build.py`` (or
``__graft_entry__.build()``). There is no fallback: if the shared library is
missing or cannot be loaded, importing the ops raises ``ImportError`` so a GPU
run can never silently take a CPU or eager-PyTorch path.
"""
from __future__ import annotations

import ctypes
import os

# GGUFMM_LIBRARY may point at another build of the same library (e.g. a debug build).
_LIB_PATH = os.environ.get("GGUFMM_LIBRARY") or os.path.join(
    os.path.dirname(os.path.abspath(__file__)), "lib", "libggufmm.so")

# status codes (include/ggufmm.h, enum ggufmm_status)
OK = 0
ERR_QTYPE = -1
ERR_SHAPE = -2
ERR_ALIGN = -3
ERR_DTYPE = -4
ERR_WORKSPACE = -5
ERR_CUDA = -6
ERR_ARG = -7
ERR_DEVICE = -8

# dtype codes (enum ggufmm_dtype)
F32, F16, BF16 = 0, 1, 2

# every symbol the header declares: name -> (restype, argtypes)
_VP, _I, _I64, _SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t
SIGNATURES = {
    "ggufmm_version": (_I, []),
    "ggufmm_block_size": (_I, [_I]),
    "ggufmm_type_size": (_I, [_I]),
    "ggufmm_status_string": (ctypes.c_char_p, [_I]),
    "ggufmm_last_cuda_error": (_I, []),
    "ggufmm_device_status": (_I, [_I, _VP]),
    "ggufmm_set_wait_limit": (_I, [ctypes.c_uint32]),
    "ggufmm_dequantize": (_I, [_VP, _I, _I64, _I64, _VP, _I, _VP]),
    "ggufmm_embedding": (_I, [_VP, _I, _I64, _I64, _VP, _I64, _VP, _I, _I64, _VP]),
    "ggufmm_stage_copy": (_I, [_VP, _VP, _SZ, _VP]),
    "ggufmm_gemv": (_I, [_VP, _I, _I64, _I64, _VP, _I, _I64, _I64, _VP, _I, _I64, _VP]),
    "ggufmm_gemv_grouped": (_I, [_I, _VP, _VP, _I, _I64, _VP, _I, _I64, _I64, _VP, _I, _VP, _VP]),
    "ggufmm_gemm_grouped": (_I, [_I, _VP, _VP, _I, _I64, _VP, _I, _I64, _I64, _VP, _I, _VP, _VP, _SZ, _VP]),
    "ggufmm_gemv_residual": (_I, [_VP, _I, _I64, _I64, _VP, _I, _I64, _I64, _VP, _I, _I64, _VP, _I64, _VP]),
    "ggufmm_gemv_kernel": (_I, [_I, _I64, _I64, _I64, _I]),
    "ggufmm_gemv_swiglu": (_I, [_VP, _VP, _I, _I64, _I64, _VP, _I, _I64, _I64, _VP, _I, _I64, _VP]),
    "ggufmm_gemv_allreduce_buffer_bytes": (_SZ, [_I64, _I64, _I]),
    "ggufmm_gemv_allreduce": (_I, [_VP, _I, _I64, _I64, _VP, _I, _I64, _I64, _VP, _I, _I64, _VP, _I, _I, _I64,
                                   ctypes.c_uint32, _VP]),
    "ggufmm_allreduce_buffer_bytes": (_SZ, [_I64, _I]),
    "ggufmm_allreduce": (_I, [_VP, _VP, _I64, _VP, _I, _I, _VP, _VP]),
    "ggufmm_peer_barrier": (_I, [_VP, _I, _I, _VP]),
    "ggufmm_gemm_allgather": (_I, [_VP, _I, _I64, _I64, _VP, _I, _I64, _I64, _VP, _I, _I64, _I, _I64, _VP, _SZ, _VP]),
    "ggufmm_gemm_workspace_size": (_SZ, [_I, _I64, _I64, _I64]),
    "ggufmm_gemm": (_I, [_VP, _I, _I64, _I64, _VP, _I, _I64, _I64, _VP, _I, _I64, _VP, _SZ, _VP]),
    "ggufmm_mul_mat": (_I, [_VP, _I, _I64, _I64, _VP, _I, _I64, _I64, _VP, _I, _I64, _VP, _SZ, _VP]),
    "ggufmm_gemm_ffn_workspace_size": (_SZ, [_I, _I64, _I64, _I64, _I]),
    "ggufmm_ffn_epilogue": (_I, [_VP, _I64, _I64, _I, _VP, _I64, _VP, _I, _I64, _VP]),
    "ggufmm_gemm_swiglu": (_I, [_VP, _VP, _I, _I64, _I64, _VP, _I, _I64, _I64, _VP, _I, _I64, _VP, _SZ, _VP]),
    "ggufmm_gemm_residual": (_I, [_VP, _I, _I64, _I64, _VP, _I, _I64, _I64, _VP, _I, _I64, _VP, _I64, _VP, _SZ, _VP]),
    "ggufmm_gemm_noalloc": (_I, [_VP, _I, _I64, _I64, _VP, _I, _I64, _I64, _VP, _I, _I64, _VP]),
}


def library_path() -> str:
    return _LIB_PATH


def load() -> ctypes.CDLL:
    """Load the library and declare every entry point's signature."""
    if not os.path.exists(_LIB_PATH):
        raise ImportError(
            f"libggufmm.so not found at {_LIB_PATH}; build it with "
            "`python vllm-webgpu_b200/build.py` (there is no CPU fallback)")
    lib = ctypes.CDLL(_LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        _lib = load()
    return _lib


class GGUFMMError(RuntimeError):
    """A CUDA-side failure reported by libggufmm."""


class GGUFMMValueError(ValueError):
    """An argument the library refused before launching anything; ``status`` is
    the GGUFMM_ERR_* code (so callers can tell an alignment refusal, which a
    slower path may serve, from a caller-side shape or dtype bug)."""

    def __init__(self, msg: str, status: int):
        super().__init__(msg)
        self.status = status


def is_align_refusal(exc: BaseException) -> bool:
    """True when ``exc`` is the library's refusal of misaligned operands."""
    return isinstance(exc, GGUFMMValueError) and exc.status == ERR_ALIGN


def check(status: int, what: str) -> None:
    """Map a status code to the exception the reference would raise.

    Shape/qtype/dtype problems are ValueError (the reference raises ValueError
    for bad dimensions, vllm_webgpu/models/llama.py:45-54); CUDA failures are
    GGUFMMError (a RuntimeError).
    """
    if status == OK:
        return
    msg = lib().ggufmm_status_string(status).decode()
    if status == ERR_CUDA:
        raise GGUFMMError(f"{what}: {msg} (cudaError {lib().ggufmm_last_cuda_error()})")
    if status == ERR_DEVICE:
        raise GGUFMMError(f"{what}: {msg}")
    raise GGUFMMValueError(f"{what}: {msg} (status {status})", status)

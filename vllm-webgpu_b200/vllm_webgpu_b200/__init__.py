"""vllm_webgpu_b200 -- B200 (sm_100a) GGUF block-quantized matmul behind the
quant / linear-layer / platform API of maci0/vllm-webgpu.

``register()`` mirrors the reference's vLLM platform-plugin entry point
(vllm_webgpu/__init__.py:23-42): it returns the platform class path when a
B200-class CUDA device is present, else None.
"""
from __future__ import annotations

__version__ = "0.1.0"


def register() -> str | None:
    from .platform import B200Platform
    if B200Platform.is_available():
        return "vllm_webgpu_b200.platform.B200Platform"
    return None


def __getattr__(name: str):
    if name == "B200Platform":
        from .platform import B200Platform
        return B200Platform
    if name in ("ops", "formats", "platform", "quant", "models", "tp"):
        import importlib
        return importlib.import_module(f"{__name__}.{name}")
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")


__all__ = ["register", "B200Platform", "__version__"]

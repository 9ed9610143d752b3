"""vLLM out-of-tree platform for the B200 path; the same classmethods as the
reference's ``WebGPUPlatform`` (vllm_webgpu/platform.py:55-147) with CUDA
answers: real device count and capability instead of the (1, "8.0") shim,
``set_device`` on any index instead of device 0 only, real synchronisation.
"""
from __future__ import annotations

import logging

logger = logging.getLogger(__name__)


def _base():
    try:
        from vllm.platforms.interface import Platform
        return Platform
    except Exception:  # vLLM absent or incompatible: a plain base keeps the API testable
        return object


def _capability_cls():
    try:
        from vllm.platforms.interface import DeviceCapability
        return DeviceCapability
    except Exception:
        class DeviceCapability:  # noqa: D401 - minimal stand-in
            def __init__(self, major=0, minor=0):
                self.major, self.minor = major, minor
        return DeviceCapability


def _enum():
    try:
        from vllm.platforms.interface import PlatformEnum
        return PlatformEnum.OOT
    except Exception:
        return "OOT"


_DeviceCapability = _capability_cls()
SUPPORTED_QUANTIZATIONS = ("gguf", "q4_0", "q8_0", "q4_k", "q4_k_m", "q6_k", "auto")


class B200Platform(_base()):
    _enum = _enum()
    device_name: str = "cuda"
    device_type: str = "cuda"
    dispatch_key: str = "CUDA"

    @classmethod
    def is_available(cls) -> bool:
        try:
            import torch
            return torch.cuda.is_available() and any(
                torch.cuda.get_device_capability(i)[0] == 10 for i in range(torch.cuda.device_count()))
        except Exception:
            return False

    @classmethod
    def get_device_name(cls, device_id: int = 0) -> str:
        import torch
        return torch.cuda.get_device_name(device_id) if torch.cuda.is_available() else "B200 (absent)"

    @classmethod
    def get_device_count(cls) -> int:
        import torch
        return torch.cuda.device_count() if torch.cuda.is_available() else 0

    @classmethod
    def get_device_capability(cls, device_id: int = 0):
        import torch
        major, minor = torch.cuda.get_device_capability(device_id) if torch.cuda.is_available() else (0, 0)
        return _DeviceCapability(major=major, minor=minor)

    @classmethod
    def get_device_total_memory(cls, device_id: int = 0) -> int:
        import torch
        return torch.cuda.get_device_properties(device_id).total_memory if torch.cuda.is_available() else 0

    @classmethod
    def get_device_available_memory(cls, device_id: int = 0) -> int:
        import torch
        if not torch.cuda.is_available():
            return 0
        free, _ = torch.cuda.mem_get_info(device_id)
        return free

    @classmethod
    def check_and_update_config(cls, vllm_config) -> None:
        # Multi-GPU is real here (the reference forced a uni executor and
        # disabled custom all-reduce, platform.py:106-113): keep vLLM's choices.
        return None

    @classmethod
    def is_pin_memory_available(cls) -> bool:
        return True

    @classmethod
    def set_device(cls, device_id: int) -> None:
        import torch
        if device_id < 0 or device_id >= cls.get_device_count():
            raise ValueError(f"B200 device {device_id} does not exist ({cls.get_device_count()} visible)")
        torch.cuda.set_device(device_id)

    @classmethod
    def current_device(cls) -> int:
        import torch
        return torch.cuda.current_device() if torch.cuda.is_available() else 0

    @classmethod
    def synchronize(cls, device_id: int = 0) -> None:
        import torch
        if torch.cuda.is_available():
            torch.cuda.synchronize(device_id)

    @classmethod
    def verify_quantization(cls, quant: str) -> None:
        if quant is not None and quant.lower() not in SUPPORTED_QUANTIZATIONS:
            raise ValueError(f"quantization {quant!r} is not supported on the B200 path "
                             f"(supported: {', '.join(SUPPORTED_QUANTIZATIONS)})")

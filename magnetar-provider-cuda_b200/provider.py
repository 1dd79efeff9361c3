"""``CudaProvider``: device discovery, health and the Kernel Registry advertisements.

Mirrors ``src/provider.rs:56-324`` (graceful unavailability, Available / Degraded /
Unavailable health, ``execution_api()``) and ``src/advertisements.rs:140-289`` (kernel
names, operator families, dtypes, rank constraints and features) for the operators this
provider implements.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import List, Optional, Tuple

from . import _native as N
from ._native import CudaError

CUDA_PROVIDER_NAME = "magnetar:provider/cuda"
CUDA_KERNEL_FAMILY = "Cuda"
CUDA_CONFORMANCE_PROFILE = "cuda-conformance-v1"


@dataclass(frozen=True)
class KernelAdvertisement:
    """One advertised kernel (``KernelAdvertisement``)."""

    name: str
    operator: str
    family: str
    provider: str
    device: str
    input_dtypes: Tuple[str, ...] = ("f32",)
    output_dtypes: Tuple[str, ...] = ("f32",)
    layouts: Tuple[str, ...] = ("contiguous",)
    memory_classes: Tuple[str, ...] = ("device",)
    rank: Optional[int] = None
    features: Tuple[str, ...] = ()
    cancellation: str = "timeout-only"
    kernel_family: str = CUDA_KERNEL_FAMILY
    conformance_profile: str = CUDA_CONFORMANCE_PROFILE
    version: str = "1.0.0"


def _baseline(name, family, device, provider, features=()):
    # src/advertisements.rs:57-80: rank-2 constraint for matmul, rope, attention, softmax.
    rank = 2 if name in ("matmul", "rope", "attention", "softmax") else None
    return KernelAdvertisement(name=name, operator=name, family=family, provider=provider, device=device,
                               rank=rank, features=tuple(features))


def _half(base, family, device, provider):
    # src/advertisements.rs:109-132: same operator, f16/bf16 kernel "<op>-half".
    return KernelAdvertisement(name=f"{base}-half", operator=base, family=family, provider=provider,
                               device=device, input_dtypes=("f16", "bf16"), output_dtypes=("f16", "bf16"))


def cuda_kernel_advertisements(device: str, provider: str = CUDA_PROVIDER_NAME) -> List[KernelAdvertisement]:
    """The implemented kernel set for one device (``cuda_kernel_advertisements``)."""
    return [
        _baseline("matmul", "LinearAlgebra", device, provider),
        _baseline("matmul-bias", "LinearAlgebra", device, provider),
        _baseline("matmul-residual", "LinearAlgebra", device, provider),
        _baseline("silu-mul", "Activation", device, provider),
        _baseline("gated-matmul", "LinearAlgebra", device, provider),
        _baseline("activation", "Activation", device, provider),
        _baseline("embedding", "Tensor", device, provider, ["embedding-scale"]),
        _baseline("rmsnorm", "Normalization", device, provider, ["rmsnorm-per-head", "rmsnorm-without-weight"]),
        _baseline("rope", "PositionEncoding", device, provider,
                  ["rope-banded-frequency-scaling", "rope-partial-rotary", "rope-yarn-frequency-scaling"]),
        _baseline("attention", "Attention", device, provider,
                  ["attention-key-count", "attention-scale", "attention-value-head-dimension", "key-count"]),
        _baseline("softmax", "Activation", device, provider),
        _baseline("silu", "Activation", device, provider),
        _baseline("gelu", "Activation", device, provider),  # the tanh approximation
        _baseline("add", "Tensor", device, provider),
        _baseline("mul", "Tensor", device, provider),
        _baseline("residual-add", "Tensor", device, provider),
        _baseline("row-scale", "Tensor", device, provider),
        _baseline("concat", "Tensor", device, provider, ["heads"]),  # rows, or heads (axis = "heads")
        _baseline("batched-matmul", "LinearAlgebra", device, provider),
        _baseline("kv-write", "Tensor", device, provider),  # f32 stores, in place
        _half("add", "Tensor", device, provider),
        _half("mul", "Tensor", device, provider),
    ]


class CudaProvider:
    """A provider bound to one GPU (``CudaProvider::for_device``).

    Construction never raises: with no usable device (no driver, no GPU, not sm_100) the
    provider is Unavailable and ``execution_api()`` is None (``src/provider.rs:149-192``).
    """

    def __init__(self, ordinal: int = 0, name: str = CUDA_PROVIDER_NAME):
        self.ordinal = ordinal
        self.name = name
        self.device_id = f"cuda:{ordinal}"
        self._kernels = None
        self._executor = None
        self._error: Optional[str] = None
        try:
            from .kernels import CudaKernels
            from .executor import CudaExecutor
            self._kernels = CudaKernels(ordinal)
            self._executor = CudaExecutor(self._kernels)
        except CudaError as e:
            self._error = str(e)
        except OSError as e:  # the native library could not be loaded at all
            self._error = f"DeviceUnavailable: {e}"

    @classmethod
    def new(cls) -> "CudaProvider":
        return cls(0)

    @classmethod
    def for_device(cls, ordinal: int, name: str = CUDA_PROVIDER_NAME) -> "CudaProvider":
        return cls(ordinal, name)

    def is_available(self) -> bool:
        return self._executor is not None

    def health(self) -> str:
        """"Available", "Degraded" (device present, kernels unusable) or "Unavailable"."""
        if self._executor is not None:
            return "Available"
        if self._error and "DeviceUnavailable" not in self._error:
            return "Degraded"
        return "Unavailable"

    def unavailable_reason(self) -> Optional[str]:
        return self._error

    def execution_api(self):
        return self._executor

    def kernels(self):
        return self._kernels

    def advertisements(self) -> List[KernelAdvertisement]:
        if not self.is_available():
            return []
        return cuda_kernel_advertisements(self.device_id, self.name)

    def device_metadata(self) -> dict:
        """``cuda_device_descriptor`` (``src/device.rs:41-92``) with its pressure bucket."""
        if self._kernels is None:
            return {"id": self.device_id, "available": False}
        info = self._kernels.info()
        free = info["free_bytes"] / max(1, info["total_bytes"])
        pressure = "low" if free > 0.5 else "medium" if free > 0.2 else "high"
        return {"id": self.device_id, "available": True, "name": info["name"], "sm": info["sm"],
                "sm_count": info["sm_count"], "total_bytes": info["total_bytes"], "dtypes": ["f32"],
                "layouts": ["contiguous"], "memory_pressure": pressure}

    def close(self) -> None:
        if self._executor is not None:
            self._executor.close()
        if self._kernels is not None:
            self._kernels.close()
        self._executor = self._kernels = None


def device_count() -> int:
    n = ctypes.c_int()
    N.check(N.lib().mg_device_count(ctypes.byref(n)))
    return n.value

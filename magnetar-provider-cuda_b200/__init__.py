"""Magnetar CUDA execution provider for B200 (sm_100a).

A drop-in for the operator path of astorise/Magnetar-provider-CUDA: the same provider /
executor / kernel surface (``CudaProvider``, ``CudaExecutor``, ``CudaKernels``) over the
precompiled native library ``lib/libmagnetar_cuda.so`` (C ABI in ``include/magnetar_cuda.h``).
There is no CPU fallback: without the library every call raises.
"""
from ._native import CudaError, build, lib
from .executor import CudaExecutor, KernelInvocation, KernelResult
from .kernels import CudaKernels, DeviceBuffer
from .provider import CudaProvider, KernelAdvertisement, cuda_kernel_advertisements, device_count

__all__ = [
    "CudaError", "CudaExecutor", "CudaKernels", "CudaProvider", "DeviceBuffer", "KernelAdvertisement",
    "KernelInvocation", "KernelResult", "build", "cuda_kernel_advertisements", "device_count", "lib",
]

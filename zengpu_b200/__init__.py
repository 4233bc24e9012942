"""zengpu_b200 - B200 (sm_100a) backend for ZenGPU's compute hot path.

Layers (all over libzengpu_b200.so, include/zengpu_b200.h):
  api      - ZenGPU's DeviceArray / BufferPool / ElementwiseKernels /
             GemmKernel / Blas API and the GpuDevice compute subset
  kernels  - the same kernels on torch CUDA tensors, stream ordered
  dist     - M-row sharding over one process per GPU: B packed on its owner
             and carried rank to rank by the copy engines while every rank's
             GEMM runs (ChainedGemm, the default), or broadcast over NCCL
             (ShardedGemm)
"""
from .api import (  # noqa: F401
    Backend, BindingMismatch, Blas, BufferPool, BufferUsage, CudaDevice, DeviceArray,
    DeviceLost, Dispatch, DType, ElementwiseKernels, GemmKernel, GemmMode, GpuError,
    InvalidUsage, KernelWait, Level1Kernels, MemoryUsage, MissingUsage, NoDevice,
    OutOfMemory, PipelineCreation, ShaderCompile, ShaderKind, StaleHandle, Submission,
    Timeout, Unsupported, UnsupportedFeatures, device_count, download, download_async, f32,
    i32, size_class, u32, upload)
from ._lib import LIB_PATH, load as load_library  # noqa: F401

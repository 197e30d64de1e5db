"""Host side of the math-plus CUDA device backend (B200): the Python twin of the TypeScript
``createCudaDevice()`` facade, over the C ABI of libmathplus_cuda.so (include/mathplus_cuda.h)."""
from . import _ffi  # noqa: F401
from .backend import CudaBackend, CudaTensor, HostTensor, host  # noqa: F401
from .device import (ArrayDevice, CudaDevice, DeviceArray, create_cuda_device,  # noqa: F401
                     createCudaDevice, cuda_unavailable_reason)

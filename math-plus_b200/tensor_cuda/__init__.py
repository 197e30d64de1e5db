"""Host side of the math-plus CUDA device backend (B200): the Python twin of the TypeScript
`createCudaDevice()` facade, over the C ABI of libmathplus_cuda.so."""
from . import _ffi  # noqa: F401

"""triton_llm (B200) -- sm_100a kernels and GPU allocator behind a C ABI.

Drop-in for the reference package of the same name: ``triton_llm.gpu`` is
the allocator, ``triton_llm.kernels`` the kernel library. The kernels are
hand-written CUDA in libtllm.so, reached through ctypes; nothing here uses
Triton, PyTorch or a CPU fallback.
"""

from . import gpu

__all__ = ["gpu"]

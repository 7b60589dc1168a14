"""TempLit B200 backend: a CUDA (sm_100a) runtime for JTPuffer/TempLit.

The product is native: ``include/my_cuda`` (cuda::Runtime and
Storage<cuda::CUDA, T>, C++20, the drop-in for metal::Runtime), the kernel
library behind ``include/templit_cuda.h`` and the GPT training step behind
``include/templit_gpt.h``.  This package only locates and loads the built
libraries (``capi``) for tests, the benchmark and callers that drive the
backend from Python.
"""
from .capi import BUILD_DIR, cuda_lib, gpt_lib, library_path  # noqa: F401

__all__ = ["BUILD_DIR", "cuda_lib", "gpt_lib", "library_path"]

"""ctypes binding of libllmgpu.so, the B200-native training step of llm-cpp.

Mirrors the reference's own ctypes binding style (python/llm_cpp/__init__.py):
a plain CDLL with declared argtypes over an `extern "C"` ABI.
"""
from ._lib import load, LIB_PATH, PKG_ROOT  # noqa: F401

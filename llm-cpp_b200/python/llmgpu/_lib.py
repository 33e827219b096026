"""Loader for libllmgpu.so (built in-tree by `make -C llm-cpp_b200`).

There is no fallback: if the shared library is missing, importing the binding
raises, so a product path can never silently run on the CPU.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
PKG_ROOT = os.path.abspath(os.path.join(_HERE, "..", ".."))
LIB_PATH = os.path.join(PKG_ROOT, "libllmgpu.so")

_lib = None

c_int, c_ll, c_vp, c_float, c_size_t = (ctypes.c_int, ctypes.c_longlong, ctypes.c_void_p,
                                       ctypes.c_float, ctypes.c_size_t)


def _declare(lib):
    lib.llmgpu_op_num_sms.argtypes = []
    lib.llmgpu_op_num_sms.restype = c_int
    lib.llmgpu_op_gemm_pair_slots.argtypes = []
    lib.llmgpu_op_gemm_pair_slots.restype = c_int
    lib.llmgpu_op_gemm.argtypes = [c_vp, c_ll, c_int, c_vp, c_ll, c_int, c_int, c_int, c_int,
                                   c_int, c_vp, c_ll, c_int, c_vp, c_ll, c_vp, c_ll, c_int, c_vp,
                                   c_int, c_ll, c_int, c_vp, c_vp]
    lib.llmgpu_op_gemm.restype = c_int
    lib.llmgpu_op_embed.argtypes = [c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_vp]
    lib.llmgpu_op_embed_bwd_work.argtypes = [c_int, c_int, c_int]
    lib.llmgpu_op_embed_bwd_work.restype = c_ll
    lib.llmgpu_op_embed_bwd.argtypes = [c_vp, c_vp, c_vp, c_vp] + [c_int] * 5 + [c_vp, c_vp]
    lib.llmgpu_op_norm_fwd.argtypes = [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_int, c_int, c_int,
                                       c_vp]
    lib.llmgpu_op_norm_bwd.argtypes = [c_vp] * 12 + [c_int, c_int, c_int, c_vp]
    lib.llmgpu_op_norm_bwd_work.argtypes = [c_int, c_int]
    lib.llmgpu_op_norm_bwd_work.restype = c_ll
    lib.llmgpu_op_cross_entropy.argtypes = [c_vp, c_int, c_int, c_int, c_vp, c_vp, c_float,
                                            c_float, c_vp]
    lib.llmgpu_op_attention_fwd.argtypes = [c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int, c_vp,
                                            c_vp]
    lib.llmgpu_op_attention_bwd.argtypes = [c_vp] * 6 + [c_int, c_int, c_int, c_int, c_vp, c_vp,
                                                         c_vp]
    lib.llmgpu_op_attention_fwd_ws.argtypes = [c_vp, c_vp, c_vp, c_int, c_int, c_int, c_int,
                                               c_vp, c_vp, c_vp]
    lib.llmgpu_op_attention_bwd_work.argtypes = [c_int, c_int, c_int, c_int]
    lib.llmgpu_op_attention_bwd_work.restype = c_ll
    lib.llmgpu_op_swiglu_fwd.argtypes = [c_vp, c_vp, c_int, c_int, c_vp]
    lib.llmgpu_op_swiglu_bwd.argtypes = [c_vp, c_vp, c_vp, c_int, c_int, c_vp]
    lib.llmgpu_op_gemm_grouped.argtypes = [c_vp, c_ll, c_int, c_vp, c_ll, c_int, c_int, c_int,
                                           c_int, c_int, c_vp, c_ll, c_int, c_vp, c_ll, c_vp,
                                           c_int, c_int, c_ll, c_ll, c_vp, c_vp]
    lib.llmgpu_op_moe_route.argtypes = [c_vp] * 5 + [c_int, c_vp] + [c_int] * 5 + [c_vp] * 5
    lib.llmgpu_op_moe_dispatch.argtypes = [c_vp, c_int, c_int, c_int, c_int, c_vp, c_vp, c_vp,
                                           c_vp]
    for n in ("llmgpu_op_embed", "llmgpu_op_norm_fwd", "llmgpu_op_norm_bwd",
              "llmgpu_op_cross_entropy", "llmgpu_op_attention_fwd", "llmgpu_op_attention_bwd",
              "llmgpu_op_attention_fwd_ws",
              "llmgpu_op_swiglu_fwd", "llmgpu_op_swiglu_bwd", "llmgpu_op_gemm_grouped",
              "llmgpu_op_moe_route", "llmgpu_op_moe_dispatch"):
        getattr(lib, n).restype = c_int
    try:
        from . import _abi_decl
        _abi_decl.declare(lib)
    except ImportError:
        pass


def load(path=None):
    """Load (once) and return the ctypes handle of libllmgpu.so."""
    global _lib
    if _lib is not None:
        return _lib
    p = path or os.environ.get("LLMGPU_LIB", LIB_PATH)
    if not os.path.exists(p):
        raise FileNotFoundError(
            f"libllmgpu.so not found at {p}; build it with `make -C llm-cpp_b200` "
            "(there is no CPU fallback)")
    lib = ctypes.CDLL(p)
    _declare(lib)
    _lib = lib
    return lib

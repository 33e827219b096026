"""CPU checks of the C ABI: the shared library loads and exports every function that
include/*.h declares; context creation without a usable sm_100 device fails cleanly with a
message instead of falling back to the CPU."""
import ctypes
import os
import re

import pytest

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
HEADERS = [os.path.join(ROOT, "include", h) for h in sorted(os.listdir(os.path.join(ROOT, "include")))
           if h.endswith(".h")]


def _declared():
    names = []
    for h in HEADERS:
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        src = re.sub(r"//[^\n]*", "", src)
        for m in re.finditer(r"\b(llmgpu_\w+)\s*\(", src):
            names.append(m.group(1))
    return sorted(set(names))


def test_headers_declare_functions():
    names = _declared()
    assert "llmgpu_train_step" in names and "llmgpu_op_gemm" in names
    assert len(names) > 30


def test_library_exports_every_declared_symbol():
    from llmgpu import load
    lib = load()
    missing = [n for n in _declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_create_without_device_fails_cleanly():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    from llmgpu.trainer import LlmgpuError, Trainer, make_config
    with pytest.raises(LlmgpuError) as e:
        Trainer(make_config(vocab_size=64, n_layers=1, n_heads=1, n_embd=32, block_size=16), 1, 16)
    assert str(e.value)


def test_invalid_config_rejected_before_device_use():
    from llmgpu import load
    from llmgpu.trainer import make_config
    lib = load()
    bad = make_config(vocab_size=64, n_layers=1, n_heads=3, n_embd=32, block_size=16)
    h = lib.llmgpu_create(ctypes.byref(bad), 1, 16, 0, 1, None)
    assert not h
    assert lib.llmgpu_last_error(None)

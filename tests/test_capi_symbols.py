"""CPU tests of the C ABI boundary: the built library loads without a GPU and
exports every function include/aestrix_cuda.h declares; the ctypes binding
declares the same set; argument validation that needs no device."""
import os
import re

from aestrix_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _header_functions():
    with open(os.path.join(ROOT, "include", "aestrix_cuda.h")) as f:
        text = f.read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(aex_[a-z0-9_]+)\s*\(", text)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.lib()
    declared = _header_functions()
    assert len(declared) >= 15
    missing = [s for s in declared if not hasattr(lib, s)]
    assert not missing, f"declared in aestrix_cuda.h but not exported: {missing}"


def test_ctypes_binding_covers_the_header():
    assert sorted(_lib.declared_symbols()) == _header_functions()


def test_abi_version_and_null_ctx_errors():
    lib = _lib.lib()
    assert lib.aex_abi_version() == 1
    # NULL context: the call fails cleanly with INVALID_ARG, nothing launched.
    assert lib.aex_joint_attention(None, None, None) == _lib.AEX_ERR_INVALID_ARG
    assert lib.aex_sync(None, None, 0) == _lib.AEX_ERR_INVALID_ARG
    assert lib.aex_joint_attention_scratch_bytes(None) == 0


def test_ctx_create_without_a_gpu_reports_an_error():
    import ctypes as C

    import torch

    if torch.cuda.is_available():
        return
    h = C.c_void_p()
    rc = _lib.lib().aex_ctx_create(0, C.byref(h))
    assert rc != _lib.AEX_OK and not h.value
    assert _lib.lib().aex_last_error_string(None)

"""The C-ABI library loads and exports every symbol include/har_cuda.h
declares; host-side argument checking fails closed (CPU only, no compute)."""
import ctypes as C
import os
import re

import pytest

import har_cuda

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    text = open(os.path.join(ROOT, "include", "har_cuda.h")).read()
    return sorted(set(re.findall(r"\b(har_cuda_[a-z0-9_]+)\s*\(", text)))


def test_header_lists_match_binding():
    assert sorted(har_cuda.EXPORTS) == header_symbols()


def test_library_exports_every_declared_symbol():
    lib = har_cuda.load_library()
    for name in header_symbols():
        assert hasattr(lib, name), name


def test_library_is_sm100a_only_build():
    # the product library must not contain a CPU implementation: no oracle symbols
    lib = har_cuda.load_library()
    assert not hasattr(lib, "haro_q4k_matvec")
    assert lib.har_cuda_abi_version() == 1


def test_null_context_is_an_error_not_a_crash():
    lib = har_cuda.load_library()
    assert lib.har_cuda_ctx_destroy(None) == har_cuda.ERR_ARG
    assert lib.har_cuda_synchronize(None, 10) == har_cuda.ERR_ARG
    assert lib.har_cuda_q4k_gemv(None, None, 0, None, 0, 1, None) == har_cuda.ERR_ARG
    assert lib.har_cuda_moe_ffn(None, None, None, 1, 1, None, None, None, 0) == har_cuda.ERR_ARG
    assert lib.har_cuda_launch_count(None) == -1
    buf = C.create_string_buffer(16)
    assert lib.har_cuda_last_error(None, buf, 16) == har_cuda.ERR_ARG


def test_ctx_create_without_gpu_fails_closed():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    lib = har_cuda.load_library()
    h = C.c_void_p()
    st = lib.har_cuda_ctx_create(0, C.byref(h))
    assert st != har_cuda.OK and not h.value
    with pytest.raises(har_cuda.HarCudaError):
        har_cuda.Context(0, use_torch_stream=False)

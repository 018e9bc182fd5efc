"""CPU checks of the C ABI library: it loads, exports every symbol the header
declares, and fails cleanly (no GPU in this container)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "kestrel_cuda.h")


def header_symbols():
    txt = open(HEADER).read()
    return sorted(set(re.findall(r"^KC_API [^(]*?\b(kc_\w+)\(", txt, flags=re.M)))


def test_header_declares_the_boundary():
    syms = header_symbols()
    for s in ("kc_init", "kc_free", "kc_upload_experts", "kc_upload_router", "kc_upload_dense", "kc_moe_ffn",
              "kc_matmul", "kc_last_error"):
        assert s in syms


def test_library_exports_every_header_symbol():
    from kestrel_b200 import cuda
    lib = cuda.load_library()
    for s in header_symbols():
        assert hasattr(lib, s), s
    assert sorted(cuda.SIGNATURES) == header_symbols()


def test_init_fails_cleanly_without_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from kestrel_b200 import cuda
    h = ctypes.c_void_p()
    rc = cuda.lib().kc_init(0, ctypes.byref(h))
    assert rc == 4 and h.value is None
    assert b"no CUDA device" in cuda.lib().kc_last_error(None)
    with pytest.raises(cuda.KestrelCudaError):
        cuda.Context(0)


def test_null_context_is_rejected():
    from kestrel_b200 import cuda
    assert cuda.lib().kc_sync(None) == 1
    assert cuda.lib().kc_moe_ffn_dev(None, 0, None, 0, None, None, None) == 1


def test_array_addresses_passed_to_the_library():
    """The binding passes numpy arrays by address through the buffer protocol
    when it can, else through ndarray.ctypes: both give the array's first
    element for writable, read-only, offset, strided and empty arrays."""
    import numpy as np
    from kestrel_b200.cuda import _ptr
    a = np.arange(48, dtype=np.float32).reshape(6, 8)
    ro = np.frombuffer(bytes(range(64)), dtype=np.uint8)
    cases = [a, a[2:], a[:, 3:], a[:, ::2], ro, ro[5:], np.empty(0, np.float32),
             np.zeros((3, 4), np.int32, order="F")]
    for x in cases:
        assert _ptr(x) == x.__array_interface__["data"][0]
    assert _ptr(None) is None

"""CPU tests of the C ABI boundary: the library loads without a GPU, exports
every function include/b2moe.h declares, and rejects invalid arguments with
MLX-style messages before touching the device."""
from __future__ import annotations

import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "b2moe.h")


def declared_functions():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^B2_API\s+[\w\s\*]+?\b(b2_\w+)\s*\(", src, flags=re.M)))


@pytest.fixture(scope="module")
def L():
    import b2moe

    return b2moe.lib()


def test_header_declares_the_boundary():
    names = declared_functions()
    for must in ("b2_quantized_matmul", "b2_gather_qmm", "b2_fp_quantize", "b2_fp_dequantize",
                 "b2_moe_router_topk", "b2_moe_gather_sort", "b2_moe_combine", "b2_moe_block_forward"):
        assert must in names


def test_library_exports_every_declared_symbol(L):
    missing = [n for n in declared_functions() if not hasattr(L, n)]
    assert not missing, missing


def test_version(L):
    import b2moe

    assert "sm_100a" in b2moe.version()


def _err(L):
    return L.b2_last_error().decode()


def test_qmm_rejects_k_not_multiple_of_group(L):
    rc = L.b2_quantized_matmul(ctypes.c_void_p(16), 0, ctypes.c_void_p(16), ctypes.c_void_p(16),
                               ctypes.c_void_p(16), ctypes.c_int64(1), ctypes.c_int64(8), ctypes.c_int64(20), None)
    assert rc == 1
    assert "[quantized_matmul]" in _err(L) and "divisible" in _err(L)


def test_qmm_rejects_null(L):
    rc = L.b2_quantized_matmul(None, 0, None, None, None, ctypes.c_int64(1), ctypes.c_int64(8),
                               ctypes.c_int64(32), None)
    assert rc == 1 and "null" in _err(L)


def test_gather_requires_indices_or_matching_batch(L):
    p = ctypes.c_void_p(16)
    rc = L.b2_gather_qmm(p, 0, p, p, None, p, ctypes.c_int64(4), ctypes.c_int64(2), ctypes.c_int64(8),
                         ctypes.c_int64(1), ctypes.c_int64(8), ctypes.c_int64(32), 0, p, None)
    assert rc == 1 and "lhs_indices" in _err(L)


def test_topk_rejects_bad_k(L):
    p = ctypes.c_void_p(16)
    rc = L.b2_moe_router_topk(p, None, 0, ctypes.c_int64(1), ctypes.c_int64(8), 9, 1, p, p, None)
    assert rc == 1 and "k must be" in _err(L)


def test_error_handler_receives_message(L):
    got = []
    CB = ctypes.CFUNCTYPE(None, ctypes.c_char_p, ctypes.c_void_p)
    cb = CB(lambda msg, data: got.append(msg.decode()))
    L.b2_set_error_handler(cb, None)
    try:
        L.b2_moe_router_topk(None, None, 0, ctypes.c_int64(1), ctypes.c_int64(8), 2, 1, None, None, None)
    finally:
        L.b2_set_error_handler(None, None)
    assert got and "[router_topk]" in got[0]


def test_python_front_end_mirrors_mlx_param_errors():
    import b2moe

    with pytest.raises(ValueError, match="group size 16"):
        b2moe._nvfp4_params("quantized_matmul", 64, 4, "nvfp4", None)
    with pytest.raises(ValueError, match="bits to be 4"):
        b2moe._nvfp4_params("quantize", 16, 3, "nvfp4", None)
    with pytest.raises(ValueError, match="biases must be null"):
        b2moe._nvfp4_params("gather_qmm", 16, 4, "nvfp4", object())


def test_block_workspace_query_needs_no_gpu():
    import b2moe

    b = b2moe._Block()
    b.hidden, b.ffn, b.n_experts, b.top_k = 2048, 768, 128, 8
    n1 = b2moe.lib().b2_moe_block_workspace_size(ctypes.byref(b), 1)
    n2 = b2moe.lib().b2_moe_block_workspace_size(ctypes.byref(b), 2048)
    assert 0 < n1 < n2

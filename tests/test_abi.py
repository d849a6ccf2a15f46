"""The C ABI library loads and exports every entry point of include/qk_b200.h (no GPU)."""

import ctypes
import re

import pytest

from conftest import ROOT


def header_symbols():
    text = (ROOT / "include" / "qk_b200.h").read_text()
    return sorted(set(re.findall(r"\b(qk_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    from qk_b200 import _lib

    lib = _lib.load()
    declared = header_symbols()
    assert len(declared) >= 20
    for name in declared:
        assert hasattr(lib, name), name
    assert set(declared) == set(_lib.SIGNATURES), "ctypes signatures must cover the header"


def test_version_and_launch_counter():
    import qk_b200

    assert qk_b200.version().startswith("qk_b200") and "sm_100a" in qk_b200.version()
    assert qk_b200.launch_count() >= 0
    assert qk_b200.library_path().endswith("libqk_b200.so")


def test_tiled_sizes_match_layout_statement():
    from oracle import layout
    from qk_b200 import _lib

    lib = _lib.load()
    for qtype, code in (("Q6_K", 14), ("Q4_K", 12), ("Q8_0", 8), ("Q5_K", 13), ("Q5_1", 7)):
        for rows, width in ((1, 1), (17, 263), (512, 2048), (2048, 512)):
            assert lib.qk_tiled_bytes(code, rows, width) == layout.tiled_bytes(qtype, rows, width)
    assert lib.qk_tiled_bytes(6, 16, 256) == -1  # Q5_0: no tiled layout


def test_argument_validation_happens_before_any_launch():
    from qk_b200 import _lib

    lib = _lib.load()
    null = ctypes.c_void_p(0)
    assert lib.qk_dequantize_rows(null, 99, 1, 256, 0, null, null) == _lib.QK_ERR_UNSUPPORTED_TYPE
    assert "unsupported" in _lib.last_error()
    assert lib.qk_dequantize_rows(null, 14, 1, 0, 0, null, null) == _lib.QK_ERR_INVALID_ARGUMENT
    assert lib.qk_quant_gemm(null, 1, 256, null, 6, 16, null, null, 0, null) == _lib.QK_ERR_UNSUPPORTED_TYPE
    assert lib.qk_quant_gemm(ctypes.c_void_p(16), 4, 256, ctypes.c_void_p(16), 14, 16, ctypes.c_void_p(16), null, 0, null) == _lib.QK_ERR_WORKSPACE
    assert lib.qk_quant_gemm_workspace_bytes(65, 263, 7) == 80 * 512 * 2 + 2 * 65 * 7 * 4
    assert lib.qk_router_topk_logits(null, null, 1, 4, 5, null, null, null, null) == _lib.QK_ERR_INVALID_ARGUMENT
    desc = _lib.MoeDesc(14, 12, 14, 2048, 512, 64, 0, 4)  # gate and up differ
    assert lib.qk_moe_forward(ctypes.byref(desc), *([null] * 6), 1, 1, null, null, 0, null) == _lib.QK_ERR_UNSUPPORTED_TYPE
    desc = _lib.MoeDesc(14, 14, 13, 2048, 512, 64, 0, 4)  # Q5_K down
    assert lib.qk_moe_forward(ctypes.byref(desc), *([null] * 6), 1, 1, null, null, 0, null) == _lib.QK_ERR_UNSUPPORTED_TYPE
    desc = _lib.MoeDesc(7, 7, 7, 2048, 512, 64, 0, 4)  # Q5_1 gate/up
    assert lib.qk_moe_forward(ctypes.byref(desc), *([null] * 6), 1, 1, null, null, 0, null) == _lib.QK_ERR_UNSUPPORTED_TYPE
    desc = _lib.MoeDesc(13, 13, 7, 2560, 640, 64, 0, 4)  # the Q4 checkpoint's Q5_K / Q5_1 mix
    assert lib.qk_moe_workspace_bytes(ctypes.byref(desc), 8) > 0
    assert lib.qk_moe_forward(ctypes.byref(desc), *([ctypes.c_void_p(16)] * 6), 1, 1,
                              ctypes.c_void_p(16), null, 0, null) == _lib.QK_ERR_WORKSPACE
    desc = _lib.MoeDesc(14, 14, 14, 2048, 96, 64, 0, 4)  # a k-quant down needs I % 256
    assert lib.qk_moe_forward(ctypes.byref(desc), *([null] * 6), 1, 1, null, null, 0, null) == _lib.QK_ERR_INVALID_ARGUMENT
    desc = _lib.MoeDesc(14, 14, 8, 2048, 96, 64, 0, 4)   # a Q8_0 down takes I % 32
    assert lib.qk_moe_workspace_bytes(ctypes.byref(desc), 8) > 8 * 4 * (256 + 2048) * 2
    desc = _lib.MoeDesc(14, 14, 14, 2048, 512, 64, 0, 4)
    assert lib.qk_moe_workspace_bytes(ctypes.byref(desc), 8) > 8 * 4 * (512 + 2048) * 2
    # missing workspace is refused before launching
    assert lib.qk_moe_forward(ctypes.byref(desc), *([ctypes.c_void_p(16)] * 6), 1, 1,
                              ctypes.c_void_p(16), null, 0, null) == _lib.QK_ERR_WORKSPACE
    assert lib.qk_kv_q8_append(null, null, 1, null, null, null, null, null, null, 1, 8, 2, 24, null) == _lib.QK_ERR_INVALID_ARGUMENT


def test_status_codes_raise_reference_exception_types():
    from qk_b200 import _lib

    with pytest.raises(ValueError):
        _lib.check(_lib.QK_ERR_INVALID_ARGUMENT)
    with pytest.raises(RuntimeError):
        _lib.check(_lib.QK_ERR_TIMEOUT)

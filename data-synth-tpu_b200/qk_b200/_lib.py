"""ctypes binding of ``libqk_b200.so`` (the C ABI declared in ``include/qk_b200.h``).

The shared library is the product; this module only loads it, declares the
signatures and turns status codes into the exceptions the reference raises for the
same contract violations (``ValueError``/``TypeError``). There is no fallback: if
the library is missing, importing any operator fails loudly.
"""

import ctypes
import os
from pathlib import Path

_HERE = Path(__file__).resolve().parent
LIBRARY_PATH = Path(os.environ.get("QK_B200_LIB", _HERE / "libqk_b200.so"))

QK_OK = 0
QK_ERR_INVALID_ARGUMENT = 1
QK_ERR_UNSUPPORTED_TYPE = 2
QK_ERR_NONFINITE_SCALE = 3
QK_ERR_CUDA = 4
QK_ERR_TIMEOUT = 5
QK_ERR_WORKSPACE = 6

QK_OUT_F32 = 0
QK_OUT_BF16 = 1
QK_DECODE_FUSED = 0x100

QK_NUM_EXP, QK_NUM_SIGMOID, QK_NUM_DIVIDE, QK_NUM_SOFTMAX, QK_NUM_SILU_BF16 = range(5)

_p = ctypes.c_void_p
_i = ctypes.c_int
_i64 = ctypes.c_int64
_sz = ctypes.c_size_t


class MoeDesc(ctypes.Structure):
    """``qk_moe_desc`` of include/qk_b200.h."""

    _fields_ = [
        ("gate_type", _i),
        ("up_type", _i),
        ("down_type", _i),
        ("hidden", _i),
        ("intermediate", _i),
        ("num_experts", _i),
        ("first_expert", _i),
        ("top_k", _i),
        ("compute", _i),
    ]


QK_COMPUTE_BF16, QK_COMPUTE_INT8_Q8 = 0, 1


# name -> (restype, argtypes)
SIGNATURES = {
    "qk_version": (ctypes.c_char_p, []),
    "qk_last_error": (ctypes.c_char_p, []),
    "qk_launch_count": (ctypes.c_uint64, []),
    "qk_dequantize_rows": (_i, [_p, _i, _i64, _i64, _i, _p, _p]),
    "qk_tiled_bytes": (_i64, [_i, _i64, _i64]),
    "qk_repack_rows": (_i, [_p, _i, _i64, _i64, _p, _p, _p]),
    "qk_unpack_rows": (_i, [_p, _i, _i64, _i64, _p, _p]),
    "qk_dequantize_tiled": (_i, [_p, _i, _i64, _i64, _i, _p, _p]),
    "qk_q6_soa_to_rows": (_i, [_p, _p, _i64, _i64, _p, _p]),
    "qk_quant_gemm_workspace_bytes": (_sz, [_i64, _i64, _i64]),
    "qk_quant_gemm": (_i, [_p, _i64, _i64, _p, _i, _i64, _p, _p, _sz, _p]),
    "qk_q8_matmul_workspace_bytes": (_sz, [_i64, _i64, _i64]),
    "qk_q8_matmul": (_i, [_p, _i64, _i64, _p, _i64, _i, _p, _p, _sz, _p]),
    "qk_router_topk": (_i, [_p, _p, _p, _i, _i, _i, _i, _p, _p, _p, _p]),
    "qk_router_topk_logits": (_i, [_p, _p, _i, _i, _i, _p, _p, _p, _p]),
    "qk_router_logits": (_i, [_p, _p, _i, _i, _i, _p, _p]),
    "qk_linear_bf16_workspace_bytes": (_sz, [_i64, _i64, _i64]),
    "qk_linear_bf16": (_i, [_p, _i64, _i64, _p, _i64, _p, _p, _sz, _p]),
    "qk_linear_bf16_check": (_i, [_p, _p]),
    "qk_router_select_shared": (_i, [_p, _p, _i, _i, _i, _p, _p, _i, _i, _i, _p, _p, _p]),
    "qk_moe_workspace_bytes": (_sz, [ctypes.POINTER(MoeDesc), _i]),
    "qk_moe_forward": (
        _i,
        [ctypes.POINTER(MoeDesc), _p, _p, _p, _p, _p, _p, _i, _i, _p, _p, _sz, _p],
    ),
    "qk_moe_forward_profiled": (
        _i,
        [ctypes.POINTER(MoeDesc), _p, _p, _p, _p, _p, _p, _i, _i, _p, _p, _sz, _p, _p],
    ),
    "qk_moe_forward_tp_partial": (
        _i,
        [ctypes.POINTER(MoeDesc), _p, _p, _p, _p, _p, _p, _i, _p, _p, _sz, _p],
    ),
    "qk_moe_forward_tp_combine": (_i, [ctypes.POINTER(MoeDesc), _p, _p, _i, _i, _p, _p, _sz, _p]),
    "qk_cast_f32_bf16": (_i, [_p, _p, _i64, _p]),
    "qk_moe_check": (_i, [_p, _p]),
    "qk_kv_q8_quantize": (_i, [_p, _i, _i64, _i, _i, _p, _p, _p]),
    "qk_kv_q8_append": (_i, [_p, _p, _i, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _p]),
    "qk_kv_q8_append_chunk": (_i, [_p, _p, _i, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _p]),
    "qk_kv_q8_gather_scales": (_i, [_p, _p, _i, _i, _i, _i, _p, _p]),
    "qk_kv_q8_read": (_i, [_p, _p, _p, _i, _i, _i, _i, _i, _i, _p, _p]),
    "qk_kv_q8_attention_workspace_bytes": (_sz, [_i, _i, _i, _i, _i]),
    "qk_kv_q8_decode_attention": (
        _i,
        [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _i, _p, _p, _sz, _p],
    ),
    "qk_kv_q8_decode_attention_partial": (
        _i,
        [_p, _p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _i, _p, _p, _sz, _p],
    ),
    "qk_kv_q8_attention_combine": (_i, [_p, _i, _i, _i, _i, _p, _p, _p]),
    "qk_qsa_block_scores": (_i, [_p, _p, _p, _i, _i, _i, _i, _i, _p, _p]),
    "qk_qsa_select": (_i, [_p, _p, _i, _i, _i, _i, _p, _p, _p]),
    "qk_qsa_update_keys": (
        _i,
        [_p, _p, _p, _p, _p, ctypes.c_float, _p, _p, _i, _i, _i, _i, _i, _p, _p, _p, _p],
    ),
    "qk_qsa_query": (_i, [_p, _p, _p, ctypes.c_float, _p, _p, _i, _i, _i, _i, _p, _p]),
    "qk_checked_argmax": (_i, [_p, _i, _i, _i64, _p, _p]),
    "qk_rms_norm": (_i, [_p, _p, _i, _i, ctypes.c_float, _p, _p]),
    "qk_qk_norm_rope": (
        _i,
        [_p, _p, _p, _p, _p, _i, _i, _i, _i, _i, ctypes.c_float, _p, _p, _p, _p, _p],
    ),
    "qk_residual_add": (_i, [_p, _p, _i64, _p, _p]),
    "qk_residual_rms_norm": (_i, [_p, _p, _p, _i, _i, ctypes.c_float, _p, _p, _p]),
    "qk_append_shared_route": (_i, [_p, _p, _i, _i, _p, _p, _i, _i, _p, _p, _p]),
    "qk_append_shared_route_ep": (_i, [_p, _p, _i, _i, _p, _p, _i, _i, _i, _p, _p, _p]),
    "qk_ep_plan": (_i, [_p, _p, _i, _i, _i, _i, _p, _p, _p, _p, _p, _p]),
    "qk_gather_rows": (_i, [_p, _p, _i64, _i64, _p, _p]),
    "qk_ep_combine": (_i, [_p, _p, _p, _p, _i, _i, _i, _i, _p, _p]),
    "qk_kv_q8_attention_check": (_i, [_p]),
    "qk_numerics": (_i, [_i, _p, _p, _p, _i64, _i, _p]),
    "qk_ep_p2p_bytes": (_sz, [_i, _i, _i, _i]),
    "qk_ep_p2p_reset": (_i, [_p, _p]),
    "qk_ep_p2p_status": (_i, [_p, _p]),
    "qk_ep_p2p_dispatch": (_i, [_p, _p, _i, _i, _i, _i, _i, _i, _p, _p, _p, _i, _p]),
    "qk_ep_p2p_expert": (
        _i,
        [ctypes.POINTER(MoeDesc), _p, _p, _p, _p, _p, _i, _i, _i, _p, _sz, _p],
    ),
    "qk_ep_p2p_expert_profiled": (
        _i,
        [ctypes.POINTER(MoeDesc), _p, _p, _p, _p, _p, _i, _i, _i, _p, _sz, _p, _p],
    ),
    "qk_ep_p2p_combine": (_i, [_p, _i, _i, _i, _i, _i, _i, _p, _p, _i, _p, _p]),
    "qk_device_alloc": (_i, [_sz, ctypes.POINTER(_p)]),
    "qk_device_free": (_i, [_p]),
    "qk_ipc_get_handle": (_i, [_p, _p]),
    "qk_ipc_open_handle": (_i, [_p, ctypes.POINTER(_p)]),
    "qk_ipc_close_handle": (_i, [_p]),
    "qk_kv_q8_decode_attention_noalloc": (
        _i,
        [_p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _i, _p, _p],
    ),
}

_lib = None


def load():
    """Load the library once and declare every exported signature."""
    global _lib
    if _lib is None:
        if not LIBRARY_PATH.exists():
            raise ImportError(
                f"{LIBRARY_PATH} is missing: build it with `python data-synth-tpu_b200/build.py`"
            )
        lib = ctypes.CDLL(str(LIBRARY_PATH))
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = lib
    return _lib


def last_error():
    return (load().qk_last_error() or b"").decode(errors="replace")


def check(status):
    """Raise the reference's exception type for a non-zero status."""
    if status == QK_OK:
        return
    message = last_error()
    if status in (QK_ERR_INVALID_ARGUMENT, QK_ERR_UNSUPPORTED_TYPE, QK_ERR_NONFINITE_SCALE,
                  QK_ERR_WORKSPACE):
        raise ValueError(message)
    raise RuntimeError(f"qk_b200 status {status}: {message}")


def call(name, *args):
    check(getattr(load(), name)(*args))


def ptr(tensor):
    """Device (or host) address of a tensor, or None."""
    return None if tensor is None else ctypes.c_void_p(tensor.data_ptr())


def stream_handle(device=None):
    import torch

    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def launch_count():
    return int(load().qk_launch_count())

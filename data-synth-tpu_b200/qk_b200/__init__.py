"""qk_b200: B200-native (sm_100a) packed-quant routed-MoE FFN and Q8 KV-cache kernels.

Drop-in host mirror of the reference runtime's operator surface for its hot path
(AhmadSaeedZaidi/data-synth-tpu ``kaggle/qwen38_tpu`` and ``kaggle/packed_q6``): GGUF
row decode, tiled repack, packed projection, router top-k, expert-parallel SwiGLU FFN
and the Q8 KV cache append/gather/decode attention. All compute runs in
``libqk_b200.so`` (C ABI in ``include/qk_b200.h``); there is no CPU fallback.
"""

from . import _lib
from ._lib import launch_count

__version__ = "0.1.0"


def version():
    return _lib.load().qk_version().decode()


def library_path():
    return str(_lib.LIBRARY_PATH)


__all__ = ["launch_count", "library_path", "version"]

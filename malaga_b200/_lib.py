"""ctypes bindings of libmalaga_b200.so (include/malaga_b200.h).

The CUDA library is the only compute path: if it is missing or fails to load,
every call raises. There is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmalaga_b200.so")

MGB_OK, MGB_ERR_INVALID, MGB_ERR_OOM, MGB_ERR_CUDA, MGB_ERR_IO, MGB_ERR_UNSUPPORTED = range(6)

# Every symbol the header declares, with (restype, argtypes).
_vp, _u32, _i, _u64 = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_int, ctypes.c_uint64


class Options(ctypes.Structure):
    _fields_ = [("use_graphs", ctypes.c_int), ("graph_cache_bytes", ctypes.c_uint64),
                ("fail_alloc_after", ctypes.c_int)]


class ModelInfo(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint32) for n in (
        "vocab_size", "d_model", "encoder_layers", "decoder_layers", "encoder_heads", "decoder_heads",
        "encoder_ffn", "decoder_ffn", "max_position_embeddings", "max_length", "pad_token_id", "eos_token_id",
        "decoder_start_token_id", "bos_token_id", "scale_embedding")] + [
        ("weight_bytes", ctypes.c_uint64), ("decoder_step_bytes", ctypes.c_uint64),
        ("lm_head_bytes", ctypes.c_uint64)]


SIGNATURES = {
    "mgb_default_options": (None, [ctypes.POINTER(Options)]),
    "mgb_open": (_i, [ctypes.c_char_p, _i, ctypes.POINTER(Options), ctypes.POINTER(_vp)]),
    "mgb_close": (None, [_vp]),
    "mgb_last_error": (ctypes.c_char_p, []),
    "mgb_model_info_get": (_i, [_vp, ctypes.POINTER(ModelInfo)]),
    "mgb_encode": (_i, [_vp, _vp, _vp, _u32, _u32, ctypes.POINTER(_vp)]),
    "mgb_batch_free": (None, [_vp]),
    "mgb_batch_cross": (_i, [_vp, _vp, _u32, _i, _vp]),
    "mgb_greedy": (_i, [_vp, _vp, _u32, _u32, _u32, _i, _vp, _vp]),
    "mgb_shortlist_find": (_i, [_vp, ctypes.c_char_p]),
    "mgb_greedy_shortlist": (_i, [_vp, _vp, _u32, _i, _u32, _u32, _i, _vp, _vp]),
    "mgb_beam": (_i, [_vp, _vp, _u32, _u32, ctypes.c_float, _u32, _vp, _vp]),
    "mgb_log_softmax_topk": (_i, [_vp, _vp, _u32, _u32, _u32, _vp, _vp]),
    "mgb_greedy_logits": (_i, [_vp, _vp, _u32, _u32, _i, _vp, _vp]),
    "mgb_clear_cache": (_i, [_vp]),
    "mgb_cuda_stream": (_vp, [_vp]),
    "mgb_kernel_launches": (_u64, [_vp]),
    "mgb_profile_step": (_i, [_vp, _vp, _u32, _u32, ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_float)]),
    "mgb_argmax_noalloc": (_i, [_vp, _u32, _u32, _vp, _vp, _vp]),
}


class MgbError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code

    @property
    def is_oom(self) -> bool:
        # translator.rs:338-340 matches this substring in the error text
        return "OUT_OF_MEMORY" in str(self)


_lib = None


def load(build_if_missing: bool = False):
    """Loads the engine library (building it first only when asked)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        if not build_if_missing:
            raise OSError(f"{LIB_PATH} is missing: build it with `python -m malaga_b200.build`")
        from .build import build_lib
        build_lib()
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(code: int) -> None:
    if code != MGB_OK:
        raise MgbError(code, load().mgb_last_error().decode(errors="replace"))

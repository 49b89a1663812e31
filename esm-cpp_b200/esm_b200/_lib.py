"""ctypes bindings of libesm_b200.so (the C ABI declared in include/esm_b200.h).

The library is built in-tree by esm-cpp_b200/build.py.  Loading fails loudly
when it is missing: there is no CPU fallback behind this package.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libesm_b200.so"

STATUS = {
    0: "OK", 1: "INVALID_ARGUMENT", 2: "OUT_OF_RANGE", 3: "NOT_FOUND", 4: "IO",
    5: "SHAPE_MISMATCH", 6: "INTERNAL", 7: "CUDA", 8: "TIMEOUT", 9: "NO_DEVICE",
}

ACT_PER_TENSOR = 0
ACT_PER_TOKEN = 1


class EsmCudaError(RuntimeError):
    """A C-ABI call returned a non-OK status."""

    def __init__(self, code: int, func: str, msg: str):
        super().__init__(f"{func}: {STATUS.get(code, code)}: {msg}")
        self.code = code


class Config(C.Structure):
    _fields_ = [
        ("num_layers", C.c_int), ("hidden_size", C.c_int), ("num_heads", C.c_int),
        ("head_dim", C.c_int), ("intermediate_size", C.c_int), ("vocab_size", C.c_int),
        ("layer_norm_eps", C.c_float), ("mask_token_id", C.c_int),
        ("weights_quantized", C.c_int), ("act_quant", C.c_int),
    ]


_FP = C.POINTER(C.c_float)
_I8P = C.POINTER(C.c_int8)


class LayerWeights(C.Structure):
    _fields_ = [
        ("attn_ln_w", _FP), ("attn_ln_b", _FP),
        ("q_w", _FP), ("k_w", _FP), ("v_w", _FP), ("out_w", _FP), ("fc1_w", _FP), ("fc2_w", _FP),
        ("q_wq", _I8P), ("k_wq", _I8P), ("v_wq", _I8P), ("out_wq", _I8P), ("fc1_wq", _I8P),
        ("fc2_wq", _I8P),
        ("q_ws", _FP), ("k_ws", _FP), ("v_ws", _FP), ("out_ws", _FP), ("fc1_ws", _FP),
        ("fc2_ws", _FP),
        ("q_b", _FP), ("k_b", _FP), ("v_b", _FP), ("out_b", _FP), ("fc1_b", _FP), ("fc2_b", _FP),
        ("ffn_ln_w", _FP), ("ffn_ln_b", _FP),
    ]


def torch_stream_handle(device: int) -> C.c_void_p:
    """The cudaStream_t of torch's current stream on `device` for
    esmcu_set_stream.  torch's default stream is the legacy default stream,
    whose handle is 0 -- which esmcu_set_stream reads as "the context's own
    stream" -- so it is passed as cudaStreamLegacy (0x1), the explicit handle
    of that same stream."""
    import torch

    h = torch.cuda.current_stream(device).cuda_stream
    return C.c_void_p(h if h else 1)


class LayerBuffers(LayerWeights):
    """esmcu_layer_buffers: the same fields, written by esmcu_model_get_layer."""


_lib = None

_VP = C.c_void_p
MATH_DEFAULT, MATH_AVX512 = 0, 1  # esmcu_math_mode
MATH_MODES = {"default": MATH_DEFAULT, "avx512": MATH_AVX512}

_SIGS = {
    "esmcu_last_error": (C.c_char_p, []),
    "esmcu_version": (C.c_char_p, []),
    "esmcu_device_count": (C.c_int, [C.POINTER(C.c_int)]),
    "esmcu_open": (C.c_int, [C.c_int, C.POINTER(_VP)]),
    "esmcu_close": (C.c_int, [_VP]),
    "esmcu_set_stream": (C.c_int, [_VP, _VP]),
    "esmcu_get_stream": (_VP, [_VP]),
    "esmcu_synchronize": (C.c_int, [_VP]),
    "esmcu_bounded_wait_selftest": (C.c_int, [_VP, C.c_int, C.POINTER(C.c_int)]),
    "esmcu_set_math_mode": (C.c_int, [_VP, C.c_int]),
    "esmcu_get_math_mode": (C.c_int, [_VP, C.POINTER(C.c_int)]),
    "esmcu_malloc": (C.c_int, [_VP, C.c_size_t, C.POINTER(_VP)]),
    "esmcu_free": (C.c_int, [_VP, _VP]),
    "esmcu_memcpy_h2d": (C.c_int, [_VP, _VP, _VP, C.c_size_t]),
    "esmcu_memcpy_d2h": (C.c_int, [_VP, _VP, _VP, C.c_size_t]),
    "esmcu_linear": (C.c_int, [_VP, _VP, _VP, _VP, _VP, C.c_int, C.c_int, C.c_int]),
    "esmcu_linear_int8": (C.c_int, [_VP, _VP, _VP, _VP, _VP, _VP, C.c_int, C.c_int, C.c_int,
                                    C.c_int]),
    "esmcu_linear_int8_noalloc": (C.c_int, [_VP, _VP, _VP, _VP, _VP, _VP, C.c_int, C.c_int,
                                            C.c_int, C.c_int]),
    "esmcu_quantize_activations": (C.c_int, [_VP, _VP, C.c_int, C.c_int, _VP, C.c_int, _VP,
                                             C.c_int]),
    "esmcu_quantize_weights": (C.c_int, [_VP, _VP, C.c_int, C.c_int, _VP, _VP]),
    "esmcu_gemm_int8_s32": (C.c_int, [_VP, _VP, C.c_int, _VP, C.c_int, _VP, C.c_int, C.c_int,
                                      C.c_int]),
    "esmcu_layernorm": (C.c_int, [_VP, _VP, _VP, _VP, C.c_float, _VP, C.c_int, C.c_int]),
    "esmcu_gelu": (C.c_int, [_VP, _VP, _VP, C.c_size_t]),
    "esmcu_residual_add_inplace": (C.c_int, [_VP, _VP, _VP, C.c_size_t]),
    "esmcu_scale_inplace": (C.c_int, [_VP, _VP, C.c_size_t, C.c_float]),
    "esmcu_rope_build_tables": (C.c_int, [C.c_int, C.c_int, _VP, _VP]),
    "esmcu_rope_apply_varlen": (C.c_int, [_VP, _VP, _VP, _VP, _VP, C.c_int, C.c_int, C.c_int]),
    "esmcu_attention_varlen": (C.c_int, [_VP, _VP, _VP, _VP, _VP, C.c_int, C.c_int, C.c_int,
                                         _VP]),
    "esmcu_plan_batches": (C.c_int, [_VP, C.c_int, C.c_float, C.c_int, _VP, _VP]),
    "esmcu_batch_view_check": (C.c_int, [C.c_int, C.c_int, _VP, C.c_int, C.c_int]),
    "esmcu_model_create": (C.c_int, [_VP, C.POINTER(Config), C.POINTER(_VP)]),
    "esmcu_model_destroy": (C.c_int, [_VP]),
    "esmcu_model_config": (C.c_int, [_VP, C.POINTER(Config)]),
    "esmcu_model_set_embeddings": (C.c_int, [_VP, _VP]),
    "esmcu_model_set_layer": (C.c_int, [_VP, C.c_int, C.POINTER(LayerWeights)]),
    "esmcu_model_set_head_int8": (C.c_int, [_VP, _VP, _VP]),
    "esmcu_model_set_first_block_fc1_fp16": (C.c_int, [_VP, C.c_int]),
    "esmcu_model_set_head": (C.c_int, [_VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP]),
    "esmcu_model_forward_packed": (C.c_int, [_VP, _VP, _VP, C.c_int, _VP, C.c_int, _VP]),
    "esmcu_model_forward_scheduled": (C.c_int, [_VP, _VP, _VP, _VP, C.c_int, C.c_float, C.c_int,
                                                _VP]),
    "esmcu_model_forward_packed_device": (C.c_int, [_VP, _VP, _VP, C.c_int, _VP, C.c_int, _VP]),
    "esmcu_model_forward_hidden_states": (C.c_int, [_VP, _VP, _VP, C.c_int, _VP, C.c_int, _VP, _VP]),
    "esmcu_model_masked_marginals": (C.c_int, [_VP, _VP, _VP, _VP, _VP, C.c_int, C.c_float, C.c_int,
                                               _VP]),
    "esmcu_forward_scheduled_multi": (C.c_int, [_VP, C.c_int, _VP, _VP, _VP, C.c_int, C.c_float,
                                                C.c_int, _VP]),
    "esmcu_model_observe_packed": (C.c_int, [_VP, _VP, C.c_int, _VP, C.c_int, C.c_float, _VP]),
    "esmcu_model_forward_observed": (C.c_int, [_VP, _VP, _VP, C.c_int, _VP, C.c_int, _VP]),
    "esmcu_model_apply_smoothquant": (C.c_int, [_VP, _VP, C.c_float]),
    "esmcu_model_quantize_weights": (C.c_int, [_VP, C.c_int]),
    "esmcu_model_get_layer": (C.c_int, [_VP, C.c_int, C.POINTER(LayerBuffers)]),
    "esmcu_model_get_head_int8": (C.c_int, [_VP, _VP, _VP]),
    "esmcu_observer_create": (C.c_int, [C.POINTER(_VP)]),
    "esmcu_observer_destroy": (C.c_int, [_VP]),
    "esmcu_observer_clear": (C.c_int, [_VP]),
    "esmcu_observer_observe": (C.c_int, [_VP, C.c_char_p, _VP, C.c_size_t]),
    "esmcu_observer_num_sites": (C.c_int, [_VP]),
    "esmcu_observer_site": (C.c_int, [_VP, C.c_int, C.c_float, C.POINTER(C.c_char_p),
                                      C.POINTER(C.c_float), C.POINTER(C.c_size_t)]),
    "esmcu_observer_percentile": (C.c_int, [_VP, C.c_char_p, C.c_float, C.POINTER(C.c_float)]),
    "esmcu_model_set_profiling": (C.c_int, [_VP, C.c_int]),
    "esmcu_model_profile": (C.c_int, [_VP, C.POINTER(C.c_char_p), _VP, C.c_int]),
    "esmcu_model_last_launch_count": (C.c_int, [_VP]),
}


def lib():
    """Loads libesm_b200.so once; raises if it has not been built."""
    global _lib
    if _lib is None:
        path = os.environ.get("ESM_B200_LIB", str(LIB_PATH))
        if not Path(path).exists():
            raise ImportError(
                f"{path} is missing: build it with `python esm-cpp_b200/build.py` "
                "(the CUDA path has no fallback)")
        L = C.CDLL(path)
        for name, (res, args) in _SIGS.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def exported_symbols() -> list[str]:
    return sorted(_SIGS)


def check(rc: int, func: str = "esmcu") -> None:
    if rc != 0:
        msg = lib().esmcu_last_error()
        raise EsmCudaError(rc, func, msg.decode() if msg else "")


def call(name: str, *args) -> int:
    """Calls esmcu_<name> and raises EsmCudaError on a non-OK status."""
    rc = getattr(lib(), name)(*args)
    check(rc, name)
    return rc

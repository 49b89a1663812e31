"""esm_b200: B200-native packed-varlen ESM-2 encoder forward (W8A8
SmoothQuant INT8), a drop-in for the hot path of esm.cpp.

    from esm_b200 import Model
    m = Model.load("esm2_650m_q8.gguf")          # or load_from_safetensors
    logits = m.forward_scheduled([ids0, ids1])   # list of [L_i, 33] float32

The compute runs in libesm_b200.so (hand-written sm_100a CUDA behind the C
ABI of include/esm_b200.h); this package is the host-side mirror of the
reference's Python API.
"""
from ._lib import ACT_PER_TENSOR, ACT_PER_TOKEN, EsmCudaError, lib  # noqa: F401
from .model import (CLS_ID, EOS_ID, MASK_ID, PAD_ID, VOCAB_SIZE, ActivationObserver,  # noqa: F401
                    Config, Model, forward_scheduled_multi)
from .streaming import StreamingScheduler  # noqa: F401

__version__ = "0.1.0"


def version() -> str:
    return lib().esmcu_version().decode()


def current_isa() -> str:
    """esm_cpp.current_isa (the ISA the reference's kernels dispatch to): here
    always the one target these kernels are built for."""
    return "sm_100a"


def host_isa() -> str:
    """esm_cpp.host_isa: the best ISA the machine offers; for this engine
    the same as current_isa (there is no other path)."""
    return "sm_100a"


def device_count() -> int:
    import ctypes

    n = ctypes.c_int(0)
    rc = lib().esmcu_device_count(ctypes.byref(n))
    return n.value if rc == 0 else 0

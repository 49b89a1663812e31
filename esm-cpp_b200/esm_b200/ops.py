"""The kernel facade (include/esm_b200.h, section 1) over torch CUDA tensors.

Each function mirrors one esm::kernels function of the reference
(include/esm_cpp/kernels.h) with device tensors instead of host pointers.
PyTorch provides device memory and the stream; every computation runs in
libesm_b200.so.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib

_ctx = {}


def context(device: int = 0):
    """A per-device esmcu_context bound to torch's current stream (so the ops
    are stream-ordered with the torch work around them)."""
    if device not in _ctx:
        h = C.c_void_p()
        _lib.call("esmcu_open", device, C.byref(h))
        _ctx[device] = h
    h = _ctx[device]
    _lib.call("esmcu_set_stream", h, _lib.torch_stream_handle(device))
    return h


def _p(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _dev(t):
    return t.device.index or 0


def set_math_mode(mode: str, device: int = 0) -> None:
    """esmcu_set_math_mode on the facade's context of `device`: "default"
    (tensor-core / fused kernels) or "avx512" (LayerNorm, GELU and attention
    reproduce the reference's default x86 kernels bit for bit)."""
    _lib.call("esmcu_set_math_mode", context(device), _lib.MATH_MODES[mode])


def synchronize(device: int = 0):
    _lib.call("esmcu_synchronize", context(device))


def linear(A, W, bias=None):
    """kernels::Linear: A [M,K] f32, W [N,K] f32 -> [M,N]."""
    import torch

    M, K = A.shape
    N = W.shape[0]
    out = torch.empty((M, N), dtype=torch.float32, device=A.device)
    _lib.call("esmcu_linear", context(_dev(A)), _p(A), _p(W), _p(bias), _p(out), M, N, K)
    return out


def linear_int8(A, Wq, w_scales, bias=None, act_quant: int = _lib.ACT_PER_TENSOR):
    """kernels::LinearInt8 (W8A8): A [M,K] f32, Wq [N,K] int8, w_scales [N]."""
    import torch

    M, K = A.shape
    N = Wq.shape[0]
    out = torch.empty((M, N), dtype=torch.float32, device=A.device)
    _lib.call("esmcu_linear_int8", context(_dev(A)), _p(A), _p(Wq), _p(w_scales), _p(bias),
              _p(out), M, N, K, act_quant)
    return out


def quantize_activations(A, act_quant: int = _lib.ACT_PER_TENSOR):
    """-> (q int8 [M, ldq], scales f32 [1] or [M]); ldq = K rounded up to 16."""
    import torch

    M, K = A.shape
    ldq = (K + 15) // 16 * 16
    q = torch.empty((M, ldq), dtype=torch.int8, device=A.device)
    s = torch.empty((M if act_quant == _lib.ACT_PER_TOKEN else 1,), dtype=torch.float32, device=A.device)
    _lib.call("esmcu_quantize_activations", context(_dev(A)), _p(A), M, K, _p(q), ldq, _p(s), act_quant)
    return q, s


def quantize_weights(W):
    """quant::Quantize on the device: W [N, K] float32 -> (q int8 [N, K],
    scales float32 [N]), bit-identical to prep.quantize_weight."""
    import torch

    W = W.contiguous()
    N, K = W.shape
    q = torch.empty((N, K), dtype=torch.int8, device=W.device)
    s = torch.empty((N,), dtype=torch.float32, device=W.device)
    _lib.call("esmcu_quantize_weights", context(_dev(W)), _p(W), N, K, _p(q), _p(s))
    return q, s


def gemm_int8_s32(q, Wq):
    """int32 acc [M,N] = q [M,K] . Wq [N,K]^T on the tensor cores."""
    import torch

    M, K = q.shape
    N = Wq.shape[0]
    acc = torch.empty((M, N), dtype=torch.int32, device=q.device)
    _lib.call("esmcu_gemm_int8_s32", context(_dev(q)), _p(q), q.stride(0), _p(Wq), Wq.stride(0),
              _p(acc), M, N, K)
    return acc


def layernorm(x, gamma, beta, eps: float = 1e-5):
    import torch

    rows, d = x.shape
    out = torch.empty_like(x)
    _lib.call("esmcu_layernorm", context(_dev(x)), _p(x), _p(gamma), _p(beta), float(eps), _p(out), rows, d)
    return out


def gelu(x):
    import torch

    out = torch.empty_like(x)
    _lib.call("esmcu_gelu", context(_dev(x)), _p(x), _p(out), x.numel())
    return out


def residual_add_inplace(y, x):
    _lib.call("esmcu_residual_add_inplace", context(_dev(y)), _p(y), _p(x), y.numel())
    return y


def scale_inplace(x, s: float):
    _lib.call("esmcu_scale_inplace", context(_dev(x)), _p(x), x.numel(), float(s))
    return x


def rope_build_tables(seq_len: int, head_dim: int):
    """kernels::RopeBuildTables on the host -> (cos, sin) numpy [L, dh]."""
    c = np.zeros((seq_len, head_dim), np.float32)
    s = np.zeros((seq_len, head_dim), np.float32)
    _lib.call("esmcu_rope_build_tables", seq_len, head_dim, c.ctypes.data, s.ctypes.data)
    return c, s


def rope_apply_varlen(x, cos_t, sin_t, cu_seqlens, num_heads: int, head_dim: int):
    B = cu_seqlens.numel() - 1
    _lib.call("esmcu_rope_apply_varlen", context(_dev(x)), _p(x), _p(cos_t), _p(sin_t),
              _p(cu_seqlens), B, num_heads, head_dim)
    return x


def attention_varlen(q, k, v, cu_seqlens, num_heads: int, head_dim: int):
    import torch

    out = torch.empty_like(q)
    B = cu_seqlens.numel() - 1
    _lib.call("esmcu_attention_varlen", context(_dev(q)), _p(q), _p(k), _p(v), _p(cu_seqlens), B,
              num_heads, head_dim, _p(out))
    return out


def plan_batches(lengths, imbalance_threshold: float = 1.2, max_batch_size: int = 256):
    """PlanBatches on the host -> list of index groups."""
    lens = np.ascontiguousarray(lengths, np.int32)
    n = lens.shape[0]
    order = np.zeros(max(n, 1), np.int32)
    sizes = np.zeros(max(n, 1), np.int32)
    g = _lib.lib().esmcu_plan_batches(lens.ctypes.data, n, float(imbalance_threshold),
                                      int(max_batch_size), order.ctypes.data, sizes.ctypes.data)
    if g < 0:
        _lib.check(1, "esmcu_plan_batches")
    out, pos = [], 0
    for i in range(g):
        out.append(order[pos:pos + sizes[i]].tolist())
        pos += sizes[i]
    return out


def batch_view_check(T: int, n_masks: int, cu_seqlens, batch_size: int) -> None:
    cu = np.ascontiguousarray(cu_seqlens, np.int32)
    _lib.call("esmcu_batch_view_check", T, n_masks, cu.ctypes.data, cu.shape[0], batch_size)

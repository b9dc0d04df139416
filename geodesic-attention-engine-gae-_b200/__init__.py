"""gae_b200 -- B200-native fused "Waller" attention (host side).

This package is the host-language mirror of the reference crate `ate`
(RegularJoe-CEO/Geodesic-Attention-Engine-GAE-, rust_src/src/lib.rs:20-30)
over the C ABI of libgae.so (include/gae.h).  Functions keep the crate's
names, argument meaning and failure behaviour (the crate panics on bad input;
here a GAEError is raised).  All attention compute runs in the library's CUDA
kernels; there is no CPU fallback: importing works without a GPU, but every
compute call needs libgae.so and a CUDA device and raises otherwise.

Device-tensor entry points (torch tensors on a CUDA device):
    attention(q, k, v, causal=..., ...)      -> tcgen05 kernel (bf16/f16) or fp32 kernel
    lse_merge_(o_acc, lse_acc, o_part, lse_part)
    quantize_rows_int8(x), attention_int8(...), int8_logits(...)
Host drop-ins of the crate (numpy / sequences of float, fp32):
    waller_operator, waller_operator_parallel, standard_attention
Scalar helpers of the crate (pure host logic, not the hot path):
    OnlineSoftmax, OnlineSoftmaxVec, WelfordState, gelu, silu, relu,
    GAEConfig, TransformerConfig
"""
from __future__ import annotations

import ctypes as C
import math
import os
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
# GAE_LIB selects another build of the library (e.g. the diagnostics variant
# lib/libgae_trace.so); the default is lib/libgae.so.
LIB_PATH = os.environ.get("GAE_LIB") or os.path.join(_HERE, "lib", "libgae.so")

GAE_OK = 0
_STATUS = {0: "GAE_OK", 1: "GAE_ERR_INVALID_ARG", 2: "GAE_ERR_UNSUPPORTED", 3: "GAE_ERR_CUDA",
           4: "GAE_ERR_OOM", 5: "GAE_ERR_COMM", 6: "GAE_ERR_TIMEOUT"}
DTYPE_F32, DTYPE_BF16, DTYPE_F16 = 0, 1, 2


class GAEError(RuntimeError):
    """A libgae.so entry point returned a non-OK status."""

    def __init__(self, status: int, detail: str):
        super().__init__(f"{_STATUS.get(status, status)}: {detail}")
        self.status = status


class AttnArgs(C.Structure):
    """Mirror of gae_attn_args (include/gae.h)."""
    _fields_ = [
        ("q", C.c_void_p), ("k", C.c_void_p), ("v", C.c_void_p), ("o", C.c_void_p),
        ("lse", C.c_void_p),
        ("batch", C.c_int64), ("heads", C.c_int64), ("seq_q", C.c_int64),
        ("seq_kv", C.c_int64), ("head_dim", C.c_int64),
        ("q_stride", C.c_int64 * 3), ("k_stride", C.c_int64 * 3),
        ("v_stride", C.c_int64 * 3), ("o_stride", C.c_int64 * 3),
        ("dtype", C.c_int), ("causal", C.c_int), ("scale", C.c_float),
        ("q_offset", C.c_int64), ("kv_offset", C.c_int64),
    ]


class AttnBwdArgs(C.Structure):
    """Mirror of gae_attn_bwd_args (include/gae.h)."""
    _fields_ = [
        ("q", C.c_void_p), ("k", C.c_void_p), ("v", C.c_void_p), ("o", C.c_void_p),
        ("dout", C.c_void_p), ("lse", C.c_void_p), ("dq", C.c_void_p), ("dk", C.c_void_p),
        ("dv", C.c_void_p),
        ("batch", C.c_int64), ("heads", C.c_int64), ("seq_q", C.c_int64),
        ("seq_kv", C.c_int64), ("head_dim", C.c_int64),
        ("q_stride", C.c_int64 * 3), ("k_stride", C.c_int64 * 3), ("v_stride", C.c_int64 * 3),
        ("o_stride", C.c_int64 * 3), ("do_stride", C.c_int64 * 3), ("dq_stride", C.c_int64 * 3),
        ("dk_stride", C.c_int64 * 3), ("dv_stride", C.c_int64 * 3),
        ("dtype", C.c_int), ("causal", C.c_int), ("scale", C.c_float),
        ("workspace", C.c_void_p), ("workspace_bytes", C.c_size_t),
    ]


class AttnInt8Args(C.Structure):
    """Mirror of gae_attn_int8_args (include/gae.h)."""
    _fields_ = [
        ("q", C.c_void_p), ("k", C.c_void_p), ("q_scale", C.c_void_p), ("k_scale", C.c_void_p),
        ("v", C.c_void_p), ("o", C.c_void_p), ("lse", C.c_void_p),
        ("batch_heads", C.c_int64), ("seq", C.c_int64), ("head_dim", C.c_int64),
        ("causal", C.c_int), ("scale", C.c_float),
    ]


_lib = None


def lib():
    """Loads libgae.so (built by build.py).  Raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise GAEError(3, f"libgae.so not found at {LIB_PATH}; run build.py")
    L = C.CDLL(LIB_PATH)
    vp, i64, sz = C.c_void_p, C.c_int64, C.c_size_t
    L.gae_status_string.restype = C.c_char_p
    L.gae_status_string.argtypes = [C.c_int]
    L.gae_last_error.argtypes = [C.c_char_p, sz]
    L.gae_version.restype = C.c_char_p
    L.gae_device_status.argtypes = [C.c_int]
    host = [vp, vp, vp, sz, sz, C.c_float, C.c_int, vp]
    L.gae_waller_operator_f32_host.argtypes = host
    L.gae_waller_operator_parallel_f32_host.argtypes = host
    L.gae_standard_attention_f32_host.argtypes = host
    L.gae_attn_fwd.argtypes = [C.POINTER(AttnArgs), vp]
    L.gae_attn_bwd.argtypes = [C.POINTER(AttnBwdArgs), vp]
    L.gae_attn_bwd_workspace_bytes.restype = sz
    L.gae_attn_bwd_workspace_bytes.argtypes = [i64, i64, i64, i64]
    L.gae_attn_int8_fwd.argtypes = [C.POINTER(AttnInt8Args), vp]
    L.gae_int8_logits.argtypes = [vp, vp, i64, i64, i64, i64, vp, vp]
    L.gae_quantize_rows_int8.argtypes = [vp, C.c_int, i64, i64, vp, vp, vp]
    L.gae_lse_merge.argtypes = [vp, vp, vp, vp, i64, i64, i64, i64, C.c_int, C.c_int, vp]
    L.gae_layer_workspace_bytes.restype = sz
    L.gae_layer_workspace_bytes.argtypes = [i64, i64, i64, i64]
    L.gae_layer_fwd.argtypes = [vp, vp, vp]
    L.gae_layer_stack_fwd.argtypes = [vp, vp, C.c_int, vp]
    L.gae_layer_fwd_static.argtypes = [vp, vp, vp]
    L.gae_layernorm_fwd.argtypes = [vp, vp, vp, vp, vp, vp, i64, i64, C.c_float, vp]
    L.gae_linear_fwd.argtypes = [vp, vp, vp, vp, vp, i64, i64, i64, C.c_int, vp]
    L.gae_symphony_workspace_bytes.restype = sz
    L.gae_symphony_workspace_bytes.argtypes = [i64, i64]
    L.gae_symphony_fwd.argtypes = [vp, vp, vp, vp, vp, vp, vp, i64, i64, vp, vp, vp, sz, vp]
    L.gae_layernorm_f32_host.argtypes = [vp, vp, vp, sz, C.c_float, vp]
    L.gae_layernorm_batched_f32_host.argtypes = [vp, vp, vp, sz, sz, C.c_float, vp]
    L.gae_mlp_block_f32_host.argtypes = [vp, vp, vp, vp, vp, sz, sz, sz, vp]
    L.gae_fused_mlp_layernorm_f32_host.argtypes = [vp] * 8 + [sz, sz, C.c_float, sz, vp]
    L.gae_transformer_block_forward_f32_host.argtypes = [vp, vp, sz, vp]
    L.gae_crate_linear_f32.argtypes = [vp, vp, vp, vp, vp, i64, i64, i64, C.c_int, C.c_int, vp]
    L.gae_crate_layernorm_f32.argtypes = [vp, vp, vp, vp, i64, i64, C.c_float, vp]
    L.gae_ring_unique_id.argtypes = [vp]
    L.gae_ring_ctx_create.argtypes = [vp, C.c_int, C.c_int, C.c_double, C.POINTER(C.c_void_p)]
    L.gae_ring_ctx_create_from_comm.argtypes = [vp, C.c_double, C.POINTER(C.c_void_p)]
    L.gae_ring_attn_fwd.argtypes = [vp, C.POINTER(AttnArgs), C.c_int, vp]
    L.gae_ring_ctx_destroy.argtypes = [vp]
    L.gae_debug_ring_plan.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, i64, vp,
                                      C.POINTER(C.c_int)]
    L.gae_debug_attn_trace.argtypes = [vp, C.c_int]
    L.gae_debug_wait_timeout.argtypes = [C.c_uint64, vp]
    L.gae_debug_attn_int8_logits.argtypes = [C.POINTER(AttnInt8Args), vp, vp]
    _lib = L
    return L


def _check(status: int):
    if status != GAE_OK:
        buf = C.create_string_buffer(512)
        lib().gae_last_error(buf, 512)
        raise GAEError(status, buf.value.decode(errors="replace"))


def version() -> str:
    return lib().gae_version().decode()


def device_status(reset: bool = True):
    """Raises GAEError(GAE_ERR_TIMEOUT) if a kernel recorded a bounded-wait failure."""
    _check(lib().gae_device_status(1 if reset else 0))


# ---------------------------------------------------------------- torch glue
def _torch():
    import torch
    return torch


def _stream_ptr(stream=None):
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def _dtype_code(t):
    torch = _torch()
    if t.dtype == torch.bfloat16:
        return DTYPE_BF16
    if t.dtype == torch.float16:
        return DTYPE_F16
    if t.dtype == torch.float32:
        return DTYPE_F32
    raise GAEError(1, f"unsupported dtype {t.dtype}")


def _bhsd(t, name):
    if t.dim() != 4:
        raise GAEError(1, f"{name} must be [batch, heads, seq, head_dim]")
    if t.stride(-1) != 1:
        raise GAEError(1, f"{name} must have a contiguous head_dim")
    if not t.is_cuda:
        raise GAEError(1, f"{name} must be a CUDA tensor")
    return (t.stride(0), t.stride(1), t.stride(2))


def attention(q, k, v, *, causal: bool = False, scale: float | None = None, q_offset: int = 0,
              kv_offset: int = 0, out=None, lse=None, return_lse: bool = False, stream=None):
    """Fused exact attention on device tensors [B, H, N, D] (strided views allowed).

    bf16/f16 -> tcgen05 tensor-core kernel (head_dim 64/128); fp32 -> fp32
    CUDA-core kernel.  The Waller operator of rust_src/src/waller_operator.rs:8-59
    generalised to batches, both masks and ring-block offsets.
    """
    torch = _torch()
    B, H, Nq, D = q.shape
    Nkv = k.shape[2]
    if k.shape != (B, H, Nkv, D) or v.shape != (B, H, Nkv, D):
        raise GAEError(1, "k and v must be [B, H, Nkv, D] matching q")
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise GAEError(1, "q, k, v must share a dtype")
    if out is None:
        out = torch.empty((B, H, Nq, D), dtype=q.dtype, device=q.device)
    if return_lse and lse is None:
        lse = torch.empty((B, H, Nq), dtype=torch.float32, device=q.device)
    if lse is not None and (not lse.is_contiguous() or lse.dtype != torch.float32):
        raise GAEError(1, "lse must be a contiguous fp32 tensor [B, H, Nq]")
    a = _attn_args(q, k, v, out, lse, causal, scale, q_offset, kv_offset)
    _check(lib().gae_attn_fwd(C.byref(a), _stream_ptr(stream)))
    return (out, lse) if return_lse else out


def _attn_args(q, k, v, out, lse, causal, scale, q_offset=0, kv_offset=0):
    """gae_attn_args for device tensors [B, H, N, D] (strided views)."""
    B, H, Nq, D = q.shape
    a = AttnArgs()
    a.q, a.k, a.v, a.o = q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr()
    a.lse = lse.data_ptr() if lse is not None else None
    a.batch, a.heads, a.seq_q, a.seq_kv, a.head_dim = B, H, Nq, k.shape[2], D
    a.q_stride[:] = _bhsd(q, "q")
    a.k_stride[:] = _bhsd(k, "k")
    a.v_stride[:] = _bhsd(v, "v")
    a.o_stride[:] = _bhsd(out, "out")
    a.dtype = _dtype_code(q)
    a.causal = 1 if causal else 0
    a.scale = (1.0 / math.sqrt(D)) if scale is None else float(scale)
    a.q_offset, a.kv_offset = int(q_offset), int(kv_offset)
    return a


def attention_backward(q, k, v, out, dout, lse, *, causal: bool = False, scale: float | None = None,
                       dq=None, dk=None, dv=None, workspace=None, stream=None):
    """Gradients (dq, dk, dv) of attention(q, k, v, causal, scale) = out given
    dout, from the forward's lse ([B, H, Nq] fp32, return_lse=True).  bf16/f16
    tensors [B, H, N, D] (strided views allowed), head_dim 64/128; causal
    needs Nq == Nkv.  The reference is inference-only: this is the training
    caller of its operator (gae_attn_bwd)."""
    torch = _torch()
    B, H, Nq, D = q.shape
    Nkv = k.shape[2]
    if k.shape != (B, H, Nkv, D) or v.shape != k.shape or out.shape != q.shape or dout.shape != q.shape:
        raise GAEError(1, "attention_backward: shape mismatch")
    if len({t.dtype for t in (q, k, v, out, dout)}) != 1:
        raise GAEError(1, "attention_backward: q, k, v, out, dout must share a dtype")
    if lse.dtype != torch.float32 or not lse.is_contiguous() or lse.numel() != B * H * Nq:
        raise GAEError(1, "attention_backward: lse must be contiguous fp32 [B, H, Nq]")
    dq = torch.empty_like(q, memory_format=torch.contiguous_format) if dq is None else dq
    dk = torch.empty_like(k, memory_format=torch.contiguous_format) if dk is None else dk
    dv = torch.empty_like(v, memory_format=torch.contiguous_format) if dv is None else dv
    if workspace is None:
        workspace = torch.empty(lib().gae_attn_bwd_workspace_bytes(B, H, Nq, D), dtype=torch.uint8,
                                device=q.device)
    a = AttnBwdArgs()
    a.q, a.k, a.v, a.o, a.dout = (t.data_ptr() for t in (q, k, v, out, dout))
    a.lse = lse.data_ptr()
    a.dq, a.dk, a.dv = dq.data_ptr(), dk.data_ptr(), dv.data_ptr()
    a.batch, a.heads, a.seq_q, a.seq_kv, a.head_dim = B, H, Nq, Nkv, D
    for name, t in (("q", q), ("k", k), ("v", v), ("o", out), ("do", dout), ("dq", dq), ("dk", dk),
                    ("dv", dv)):
        getattr(a, name + "_stride")[:] = _bhsd(t, name)
    a.dtype = _dtype_code(q)
    a.causal = 1 if causal else 0
    a.scale = (1.0 / math.sqrt(D)) if scale is None else float(scale)
    a.workspace, a.workspace_bytes = workspace.data_ptr(), workspace.numel()
    _check(lib().gae_attn_bwd(C.byref(a), _stream_ptr(stream)))
    return dq, dk, dv


def _attention_function():
    torch = _torch()

    class AttentionFunction(torch.autograd.Function):
        """torch.autograd wrapper: forward = gae_attn_fwd (saves the LSE),
        backward = gae_attn_bwd."""

        @staticmethod
        def forward(ctx, q, k, v, causal, scale):
            out, lse = attention(q, k, v, causal=causal, scale=scale, return_lse=True)
            ctx.save_for_backward(q, k, v, out, lse)
            ctx.causal, ctx.scale = causal, scale
            return out

        @staticmethod
        def backward(ctx, dout):
            q, k, v, out, lse = ctx.saved_tensors
            dq, dk, dv = attention_backward(q, k, v, out, dout.contiguous(), lse, causal=ctx.causal,
                                            scale=ctx.scale)
            return dq, dk, dv, None, None

    return AttentionFunction


_ATTN_FN = None


def attention_autograd(q, k, v, *, causal: bool = False, scale: float | None = None):
    """attention() that records a backward (training use)."""
    global _ATTN_FN
    if _ATTN_FN is None:
        _ATTN_FN = _attention_function()
    return _ATTN_FN.apply(q, k, v, causal, scale)


def lse_merge_(o_acc, lse_acc, o_part, lse_part, stream=None):
    """In-place log-sum-exp merge of a partial result into an accumulator.

    o_acc/o_part: contiguous [..., D] (dtypes may differ, e.g. an fp32
    accumulator fed bf16 partials); lse_*: contiguous fp32 [...]."""
    D = o_acc.shape[-1]
    rows = o_acc.numel() // D
    if o_part.shape != o_acc.shape or lse_acc.numel() != rows or lse_part.numel() != rows:
        raise GAEError(1, "lse_merge_: shape mismatch")
    if not (o_acc.is_contiguous() and o_part.is_contiguous() and lse_acc.is_contiguous()
            and lse_part.is_contiguous()):
        raise GAEError(1, "lse_merge_: tensors must be contiguous")
    _check(lib().gae_lse_merge(o_acc.data_ptr(), lse_acc.data_ptr(), o_part.data_ptr(),
                               lse_part.data_ptr(), rows, D, D, D, _dtype_code(o_acc),
                               _dtype_code(o_part), _stream_ptr(stream)))
    return o_acc, lse_acc


def quantize_rows_int8(x, stream=None):
    """Per-row symmetric int8 quantisation of a contiguous [..., d] bf16/fp32 tensor."""
    torch = _torch()
    x = x.contiguous()
    d = x.shape[-1]
    rows = x.numel() // d
    q = torch.empty(x.shape, dtype=torch.int8, device=x.device)
    s = torch.empty(x.shape[:-1], dtype=torch.float32, device=x.device)
    _check(lib().gae_quantize_rows_int8(x.data_ptr(), _dtype_code(x), rows, d, q.data_ptr(),
                                        s.data_ptr(), _stream_ptr(stream)))
    return q, s


def attention_int8(q, k, q_scale, k_scale, v, *, causal=False, scale=None, out=None,
                   return_lse=False, stream=None, logits_out=None):
    """INT8 attention: q, k int8 [BH, N, D] + fp32 row scales [BH, N]; v bf16 [BH, N, D].
    logits_out (diagnostics, int32 [BH, N, N] on the device): the same kernel
    also writes the exact int32 logits it computed (gae_debug_attn_int8_logits)."""
    torch = _torch()
    BH, N, D = q.shape
    if out is None:
        out = torch.empty((BH, N, D), dtype=torch.bfloat16, device=q.device)
    lse = torch.empty((BH, N), dtype=torch.float32, device=q.device) if return_lse else None
    for t in (q, k, q_scale, k_scale, v, out):
        if not t.is_contiguous():
            raise GAEError(1, "attention_int8: tensors must be contiguous")
    a = AttnInt8Args()
    a.q, a.k, a.q_scale, a.k_scale = q.data_ptr(), k.data_ptr(), q_scale.data_ptr(), k_scale.data_ptr()
    a.v, a.o = v.data_ptr(), out.data_ptr()
    a.lse = lse.data_ptr() if lse is not None else None
    a.batch_heads, a.seq, a.head_dim = BH, N, D
    a.causal = 1 if causal else 0
    a.scale = (1.0 / math.sqrt(D)) if scale is None else float(scale)
    if logits_out is not None:
        if tuple(logits_out.shape) != (BH, N, N) or logits_out.dtype != torch.int32 or \
                not logits_out.is_contiguous():
            raise GAEError(1, "attention_int8: logits_out must be contiguous int32 [BH, N, N]")
        _check(lib().gae_debug_attn_int8_logits(C.byref(a), logits_out.data_ptr(), _stream_ptr(stream)))
    else:
        _check(lib().gae_attn_int8_fwd(C.byref(a), _stream_ptr(stream)))
    return (out, lse) if return_lse else out


def int8_logits(q, k, stream=None):
    """Exact int32 logits q @ k^T per (batch*head) through the tcgen05 int8 tiles."""
    torch = _torch()
    BH, Nq, D = q.shape
    Nkv = k.shape[1]
    out = torch.empty((BH, Nq, Nkv), dtype=torch.int32, device=q.device)
    _check(lib().gae_int8_logits(q.contiguous().data_ptr(), k.contiguous().data_ptr(), BH, Nq,
                                 Nkv, D, out.data_ptr(), _stream_ptr(stream)))
    return out


# ------------------------------------------------- host drop-ins of `ate`
def _host_f32(x, n):
    a = np.ascontiguousarray(np.asarray(x, dtype=np.float32).reshape(-1))
    if a.size < n:
        # The crate indexes q[i*head_dim..] and panics on a short slice.
        raise GAEError(1, f"input slice has {a.size} elements, need {n}")
    return a


def _host_call(fn, q, k, v, seq_len, head_dim, scale, causal):
    n = seq_len * head_dim
    qa, ka, va = (_host_f32(t, n) for t in (q, k, v))
    out = np.empty(n, np.float32)
    _check(fn(qa.ctypes.data, ka.ctypes.data, va.ctypes.data, seq_len, head_dim, scale,
              1 if causal else 0, out.ctypes.data))
    return out


def waller_operator(q, k, v, seq_len: int, head_dim: int, scale: float, causal: bool = True):
    """ate::waller_operator (rust_src/src/waller_operator.rs:8-15): causal fused
    attention of one head, [seq_len, head_dim] fp32 row-major, on the GPU."""
    return _host_call(lib().gae_waller_operator_f32_host, q, k, v, seq_len, head_dim, scale, causal)


def waller_operator_parallel(q, k, v, seq_len: int, head_dim: int, scale: float,
                             causal: bool = True):
    """ate::waller_operator_parallel (rust_src/src/waller_operator.rs:63-70)."""
    return _host_call(lib().gae_waller_operator_parallel_f32_host, q, k, v, seq_len, head_dim,
                      scale, causal)


def standard_attention(q, k, v, seq_len: int, head_dim: int, scale: float, causal: bool = True):
    """ate::standard_attention (rust_src/src/standard_attention.rs:13-20)."""
    return _host_call(lib().gae_standard_attention_f32_host, q, k, v, seq_len, head_dim, scale,
                      causal)


# ------------------------------------------ scalar helpers of the crate
class AteGpu:
    """ate::gpu::AteGpu (rust_src/src/gpu/wgpu_backend.rs:17-146): the crate's
    GPU backend API, served by this library's CUDA path instead of wgpu.  Its
    WGSL kernel (gpu/waller.wgsl) is the causal Waller recurrence over
    [seq_len, head_dim] f32 with the running max starting at -FLT_MAX;
    waller_operator here runs the fp32 kernel with the reference's operation
    order (the shader's head_dim <= 64 register array is not a limit here)."""

    @classmethod
    def new(cls):
        lib()  # the library loads (and fails loudly) at construction, as wgpu's adapter request would
        return cls()

    def waller_operator(self, q, k, v, seq_len: int, head_dim: int, scale: float):
        return waller_operator(q, k, v, seq_len, head_dim, scale, causal=True)


class OnlineSoftmax:
    """ate::OnlineSoftmax (rust_src/src/online_softmax.rs:5-41)."""

    def __init__(self):
        self.max = float("-inf")
        self.sum = 0.0

    def update(self, score: float):
        score = float(np.float32(score))
        if score > self.max:
            self.sum = float(np.float32(self.sum) * np.float32(math.exp(self.max - score)) + np.float32(1.0))
            self.max = score
        else:
            self.sum = float(np.float32(self.sum) + np.float32(math.exp(score - self.max)))

    def probability(self, score: float) -> float:
        return float(np.float32(math.exp(score - self.max)) / np.float32(self.sum))


class OnlineSoftmaxVec:
    """ate::OnlineSoftmaxVec (rust_src/src/online_softmax.rs:44-68)."""

    def __init__(self, n_heads: int):
        self.states = [OnlineSoftmax() for _ in range(n_heads)]

    def update(self, head: int, score: float):
        self.states[head].update(score)

    def reset(self):
        self.states = [OnlineSoftmax() for _ in self.states]


class WelfordState:
    """ate::WelfordState (rust_src/src/welford.rs:5-55), f32 arithmetic."""

    def __init__(self, mean=0.0, m2=0.0, count=0):
        self.mean, self.m2, self.count = np.float32(mean), np.float32(m2), int(count)

    def update(self, x: float):
        x = np.float32(x)
        self.count += 1
        delta = x - self.mean
        self.mean = self.mean + delta / np.float32(self.count)
        self.m2 = self.m2 + delta * (x - self.mean)

    def variance(self) -> float:
        return 0.0 if self.count < 2 else float(self.m2 / np.float32(self.count))

    def std(self, eps: float) -> float:
        return float(np.sqrt(np.float32(self.variance()) + np.float32(eps)))

    @staticmethod
    def merge(a: "WelfordState", b: "WelfordState") -> "WelfordState":
        count = a.count + b.count
        if count == 0:
            return WelfordState()
        delta = b.mean - a.mean
        mean = a.mean + delta * np.float32(b.count) / np.float32(count)
        m2 = a.m2 + b.m2 + delta * delta * np.float32(a.count) * np.float32(b.count) / np.float32(count)
        return WelfordState(mean, m2, count)


def gelu(x: float) -> float:
    """ate::gelu (rust_src/src/activations.rs:5-7), the tanh form."""
    x = np.float32(x)
    c = np.float32(math.sqrt(np.float32(2.0) / np.float32(math.pi)))
    return float(np.float32(0.5) * x * (np.float32(1.0) + np.tanh(c * (x + np.float32(0.044715) * x * x * x))))


def silu(x: float) -> float:
    """ate::silu (rust_src/src/activations.rs:11-13)."""
    x = np.float32(x)
    return float(x / (np.float32(1.0) + np.float32(math.exp(-x))))


def relu(x: float) -> float:
    """ate::relu (rust_src/src/activations.rs:17-19)."""
    return max(float(x), 0.0)


@dataclass
class GAEConfig:
    """ate::GAEConfig (rust_src/src/config.rs:5-48)."""
    hidden_dim: int
    num_heads: int
    head_dim: int
    mlp_dim: int
    ln_eps: float
    max_seq_len: int

    @classmethod
    def new(cls, hidden_dim, num_heads, mlp_dim, max_seq_len):
        if hidden_dim % num_heads != 0:
            raise GAEError(1, "hidden_dim must be divisible by num_heads")
        return cls(hidden_dim, num_heads, hidden_dim // num_heads, mlp_dim, 1e-5, max_seq_len)

    @classmethod
    def gpt2_small(cls):
        return cls.new(768, 12, 3072, 1024)

    @classmethod
    def gpt2_medium(cls):
        return cls.new(1024, 16, 4096, 1024)

    @classmethod
    def llama_7b(cls):
        return cls.new(4096, 32, 11008, 4096)


@dataclass
class TransformerConfig:
    """ate::TransformerConfig (rust_src/src/transformer.rs:9-33)."""
    hidden_dim: int
    num_heads: int
    head_dim: int
    mlp_dim: int
    eps: float

    @classmethod
    def from_gae(cls, cfg: GAEConfig):
        return cls(cfg.hidden_dim, cfg.num_heads, cfg.head_dim, cfg.mlp_dim, cfg.ln_eps)


# ------------------------------------------------------ fused layer (GPU)
EPI_BIAS, EPI_GELU, EPI_RESIDUAL = 0, 1, 2


def linear(x, w, bias=None, res=None, gelu=False, out=None, stream=None):
    """y = x @ w^T (+ bias) then tanh-GELU or + res; bf16 [M, K] x [N, K] on tcgen05.

    The tensor-core replacement of the crate's matvecs (rust_src/src/mlp.rs:7-36,
    transformer.rs:124-134): w is stored [out, in]."""
    torch = _torch()
    M, K = x.shape
    N = w.shape[0]
    if w.shape[1] != K:
        raise GAEError(1, "linear: w must be [N, K]")
    for t in (x, w) + ((res,) if res is not None else ()):
        if t.dtype != torch.bfloat16 or not t.is_contiguous():
            raise GAEError(1, "linear: x, w, res must be contiguous bf16")
    if bias is not None and (bias.dtype != torch.float32 or not bias.is_contiguous()):
        raise GAEError(1, "linear: bias must be contiguous fp32")
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    epi = EPI_GELU if gelu else (EPI_RESIDUAL if res is not None else EPI_BIAS)
    _check(lib().gae_linear_fwd(x.data_ptr(), w.data_ptr(),
                                bias.data_ptr() if bias is not None else None,
                                res.data_ptr() if res is not None else None, out.data_ptr(),
                                M, N, K, epi, _stream_ptr(stream)))
    return out


def layernorm_rows(x, gamma, beta, eps=1e-5, res=None, sum_out=None, out=None, stream=None):
    """Row LayerNorm of bf16 [rows, d] (layernorm.rs:20-47 semantics): optional
    fused residual add (the rounded sum is written to sum_out when given)."""
    torch = _torch()
    rows, d = x.shape
    if out is None:
        out = torch.empty_like(x)
    _check(lib().gae_layernorm_fwd(x.data_ptr(), res.data_ptr() if res is not None else None,
                                   sum_out.data_ptr() if sum_out is not None else None,
                                   out.data_ptr(), gamma.data_ptr(), beta.data_ptr(), rows, d,
                                   float(eps), _stream_ptr(stream)))
    return out


class LayerArgs(C.Structure):
    """Mirror of gae_layer_args (include/gae.h)."""
    _fields_ = [("x", C.c_void_p), ("out", C.c_void_p), ("batch", C.c_int64), ("seq", C.c_int64),
                ("d_model", C.c_int64), ("heads", C.c_int64), ("d_ff", C.c_int64),
                ("eps", C.c_float), ("workspace", C.c_void_p), ("workspace_bytes", C.c_size_t)]


class LayerWeights(C.Structure):
    """Mirror of gae_layer_weights (include/gae.h)."""
    _fields_ = [(n, C.c_void_p) for n in (
        "ln1_gamma", "ln1_beta", "w_qkv", "b_qkv", "w_proj", "b_proj", "ln2_gamma", "ln2_beta",
        "w_fc", "b_fc", "w_fc2", "b_fc2")]


class Gpt2Layer:
    """One pre-norm GPT-2 layer on the device (gae_layer_fwd):
    x1 = x + proj(attn(LN1(x))); out = x1 + fc2(gelu(fc1(LN2(x1)))).
    Weights bf16 [out, in], biases and LN parameters fp32, all on the GPU."""
    NAMES = ("ln1_gamma", "ln1_beta", "w_qkv", "b_qkv", "w_proj", "b_proj", "ln2_gamma",
             "ln2_beta", "w_fc", "b_fc", "w_fc2", "b_fc2")

    def __init__(self, d_model, heads, d_ff, weights: dict, eps=1e-5):
        self.d_model, self.heads, self.d_ff, self.eps = d_model, heads, d_ff, eps
        self.w = {n: weights[n].contiguous() for n in self.NAMES}
        self._cw = LayerWeights(*(self.w[n].data_ptr() for n in self.NAMES))

    @classmethod
    def random(cls, d_model, heads, d_ff, device="cuda", seed=0, eps=1e-5):
        """GPT-2-style init: weights N(0, 0.02), biases 0, LN gamma 1 / beta 0."""
        torch = _torch()
        g = torch.Generator().manual_seed(seed)
        mk = lambda *s: (torch.randn(*s, generator=g) * 0.02).to(torch.bfloat16).to(device)
        z = lambda n: torch.zeros(n, dtype=torch.float32, device=device)
        o = lambda n: torch.ones(n, dtype=torch.float32, device=device)
        D, F = d_model, d_ff
        return cls(D, heads, F, dict(ln1_gamma=o(D), ln1_beta=z(D), w_qkv=mk(3 * D, D),
                                     b_qkv=z(3 * D), w_proj=mk(D, D), b_proj=z(D),
                                     ln2_gamma=o(D), ln2_beta=z(D), w_fc=mk(F, D), b_fc=z(F),
                                     w_fc2=mk(D, F), b_fc2=z(D)), eps)

    # Raw-weight file stems (GPT-2 module names: attn.c_attn, attn.c_proj,
    # mlp.c_fc, mlp.c_proj, ln_1, ln_2) -> layer tensor.  The reference ships
    # `layer_weights/{b_fc,b_proj}_layer{0..11}.bin` (3072 and 768 f32 each; its
    # large matrices are not distributed), i.e. the MLP pair c_fc / c_proj.
    FILE_MAP = {"ln_1_g": "ln1_gamma", "ln_1_b": "ln1_beta", "w_attn": "w_qkv",
                "b_attn": "b_qkv", "w_attn_proj": "w_proj", "b_attn_proj": "b_proj",
                "ln_2_g": "ln2_gamma", "ln_2_b": "ln2_beta", "w_fc": "w_fc", "b_fc": "b_fc",
                "w_proj": "w_fc2", "b_proj": "b_fc2"}

    def load_weights(self, directory, layer_index, file_map=None):
        """Overwrites this layer's tensors with the raw little-endian f32 files
        `<stem>_layer<layer_index>.bin` present in `directory` (stems from
        `file_map`, default FILE_MAP).  Matrices are stored as GPT-2 keeps
        them, [in, out], and are transposed to this layer's [out, in].  Files
        that are absent leave the tensor as it was; a file whose size does not
        match raises GAEError(GAE_ERR_INVALID_ARG).  Returns the loaded names."""
        torch = _torch()
        loaded = []
        for stem, name in (file_map or self.FILE_MAP).items():
            path = os.path.join(directory, f"{stem}_layer{layer_index}.bin")
            if not os.path.exists(path):
                continue
            dst = self.w[name]
            raw = np.fromfile(path, dtype="<f4")
            if raw.size != dst.numel():
                raise GAEError(1, f"{path}: {raw.size} floats, {name} needs {dst.numel()}")
            t = torch.from_numpy(raw.astype(np.float32))
            if dst.dim() == 2:
                t = t.reshape(dst.shape[1], dst.shape[0]).t()
            dst.copy_(t.reshape(dst.shape).to(dst.dtype))
            loaded.append(name)
        return loaded

    @classmethod
    def load_stack(cls, directory, n_layers, d_model, heads, d_ff, device="cuda", seed=0,
                   eps=1e-5, file_map=None):
        """n_layers layers initialised as `random` (seed + layer index), then
        every weight file present in `directory` loaded over them.  Returns
        (layers, {layer index: loaded names})."""
        layers, report = [], {}
        for i in range(n_layers):
            layer = cls.random(d_model, heads, d_ff, device=device, seed=seed + i, eps=eps)
            report[i] = layer.load_weights(directory, i, file_map)
            layers.append(layer)
        return layers, report

    def _args(self, x, out, ws):
        B, S, D = x.shape
        return LayerArgs(x.data_ptr(), out.data_ptr(), B, S, D, self.heads, self.d_ff, self.eps,
                         ws.data_ptr(), ws.numel())

    def workspace(self, B, S, device="cuda"):
        torch = _torch()
        n = lib().gae_layer_workspace_bytes(B, S, self.d_model, self.d_ff)
        return torch.empty(n, dtype=torch.uint8, device=device)

    def forward(self, x, out=None, workspace=None, stream=None):
        """x: bf16 [B, S, d_model] contiguous; returns bf16 [B, S, d_model]."""
        torch = _torch()
        B, S, D = x.shape
        out = torch.empty_like(x) if out is None else out
        ws = self.workspace(B, S, x.device) if workspace is None else workspace
        a = self._args(x, out, ws)
        _check(lib().gae_layer_fwd(C.byref(a), C.byref(self._cw), _stream_ptr(stream)))
        return out


def layer_stack_forward(layers, x, out=None, workspace=None, stream=None):
    """Applies layers (a list of Gpt2Layer of one shape) in order through
    gae_layer_stack_fwd (one call, ping-pong buffers in the workspace)."""
    torch = _torch()
    B, S, D = x.shape
    out = torch.empty_like(x) if out is None else out
    ws = layers[0].workspace(B, S, x.device) if workspace is None else workspace
    arr = (LayerWeights * len(layers))(*(l._cw for l in layers))
    a = layers[0]._args(x, out, ws)
    _check(lib().gae_layer_stack_fwd(C.byref(a), arr, len(layers), _stream_ptr(stream)))
    return out


def _slice(x, n, what):
    a = np.ascontiguousarray(np.asarray(x, dtype=np.float32).reshape(-1))
    if a.size < n:
        # The crate indexes these slices directly and panics on a short one.
        raise GAEError(1, f"{what} has {a.size} elements, need {n}")
    return a


def _ptr(a):
    return a.ctypes.data


def layernorm_batched(input, gamma, beta, batch_size: int, hidden_dim: int, eps: float):
    """ate::layernorm_batched (rust_src/src/layernorm.rs:20-47) through
    gae_layernorm_batched_f32_host: fp32, the crate's Welford statistics in
    its order (bit-identical results).  Host f32 in, host f32 out."""
    n = batch_size * hidden_dim
    x = _slice(input, n, "input")
    g, b = _slice(gamma, hidden_dim, "gamma"), _slice(beta, hidden_dim, "beta")
    out = np.empty(n, np.float32)
    _check(lib().gae_layernorm_batched_f32_host(_ptr(x), _ptr(g), _ptr(b), batch_size, hidden_dim,
                                                eps, _ptr(out)))
    return out


def layernorm(input, gamma, beta, eps: float):
    """ate::layernorm (layernorm.rs:6-17): one row, the length of `input`."""
    x = np.ascontiguousarray(np.asarray(input, dtype=np.float32).reshape(-1))
    n = x.size
    g, b = _slice(gamma, n, "gamma"), _slice(beta, n, "beta")
    out = np.empty(n, np.float32)
    _check(lib().gae_layernorm_f32_host(_ptr(x), _ptr(g), _ptr(b), n, eps, _ptr(out)))
    return out


def mlp_block(input, w1, b1, w2, b2, hidden_dim: int, mlp_dim: int):
    """ate::mlp_block (rust_src/src/mlp.rs:7-36): gelu(x @ W1 + b1) @ W2 + b2
    in fp32 with the crate's sequential sums (gae_mlp_block_f32_host).
    `input` may hold several tokens (len = tokens * hidden_dim; the crate
    takes one); any widths."""
    x = np.ascontiguousarray(np.asarray(input, dtype=np.float32).reshape(-1))
    tokens = max(1, x.size // hidden_dim)
    x = _slice(x, tokens * hidden_dim, "input")
    a1, c1 = _slice(w1, hidden_dim * mlp_dim, "w1"), _slice(b1, mlp_dim, "b1")
    a2, c2 = _slice(w2, hidden_dim * mlp_dim, "w2"), _slice(b2, hidden_dim, "b2")
    out = np.empty(tokens * hidden_dim, np.float32)
    _check(lib().gae_mlp_block_f32_host(_ptr(x), _ptr(a1), _ptr(c1), _ptr(a2), _ptr(c2), hidden_dim,
                                        mlp_dim, tokens, _ptr(out)))
    return out


def fused_mlp_layernorm(input, residual, w1, b1, w2, b2, gamma, beta, hidden_dim: int,
                        mlp_dim: int, eps: float):
    """ate::fused_mlp_layernorm (mlp.rs:39-73): LayerNorm(mlp_block(x) +
    residual) in fp32 (gae_fused_mlp_layernorm_f32_host), per token."""
    x = np.ascontiguousarray(np.asarray(input, dtype=np.float32).reshape(-1))
    tokens = max(1, x.size // hidden_dim)
    n = tokens * hidden_dim
    x, r = _slice(x, n, "input"), _slice(residual, n, "residual")
    a1, c1 = _slice(w1, hidden_dim * mlp_dim, "w1"), _slice(b1, mlp_dim, "b1")
    a2, c2 = _slice(w2, hidden_dim * mlp_dim, "w2"), _slice(b2, hidden_dim, "b2")
    g, bt = _slice(gamma, hidden_dim, "gamma"), _slice(beta, hidden_dim, "beta")
    out = np.empty(n, np.float32)
    _check(lib().gae_fused_mlp_layernorm_f32_host(_ptr(x), _ptr(r), _ptr(a1), _ptr(c1), _ptr(a2),
                                                  _ptr(c2), _ptr(g), _ptr(bt), hidden_dim, mlp_dim,
                                                  eps, tokens, _ptr(out)))
    return out


class TransformerBlockF32(C.Structure):
    """Mirror of gae_transformer_block_f32 (host pointers + config)."""
    _fields_ = ([(n, C.c_void_p) for n in ("wq", "wk", "wv", "wo", "ln1_gamma", "ln1_beta", "w1",
                                            "b1", "w2", "b2", "ln2_gamma", "ln2_beta")] +
                [("hidden_dim", C.c_size_t), ("num_heads", C.c_size_t), ("head_dim", C.c_size_t),
                 ("mlp_dim", C.c_size_t), ("eps", C.c_float)])


class TransformerBlock:
    """ate::TransformerBlock (rust_src/src/transformer.rs:36-120) on the GPU.
    Weights keep the crate's layouts (wq/wk/wv/wo [h, h] as W[out, in]; w1
    [h, m]; w2 [m, h]); forward() reproduces the crate's demo forward exactly
    as written (transformer.rs:87-120: per-token LN1 -> Wv -> Wo + residual ->
    MLP + residual -> LN2, no cross-token attention) in fp32 with the crate's
    operation order, through gae_transformer_block_forward_f32_host."""

    _names = ("wq", "wk", "wv", "wo", "ln1_gamma", "ln1_beta", "w1", "b1", "w2", "b2",
              "ln2_gamma", "ln2_beta")

    def __init__(self, config: TransformerConfig, **w):
        self.config = config
        for k, v in w.items():
            setattr(self, k, np.ascontiguousarray(np.asarray(v, np.float32).reshape(-1)))

    @classmethod
    def new_random(cls, config: TransformerConfig):
        """transformer.rs:66-84: constant 0.02 weights, unit/zero LN parameters."""
        h, m = config.hidden_dim, config.mlp_dim
        f = lambda n, v: np.full(n, v, np.float32)
        return cls(config, wq=f(h * h, .02), wk=f(h * h, .02), wv=f(h * h, .02),
                   wo=f(h * h, .02), ln1_gamma=f(h, 1), ln1_beta=f(h, 0), w1=f(h * m, .02),
                   b1=f(m, 0), w2=f(m * h, .02), b2=f(h, 0), ln2_gamma=f(h, 1), ln2_beta=f(h, 0))

    def forward(self, input, seq_len: int):
        cfg = self.config
        h, m = cfg.hidden_dim, cfg.mlp_dim
        sizes = dict(wq=h * h, wk=h * h, wv=h * h, wo=h * h, ln1_gamma=h, ln1_beta=h, w1=h * m, b1=m,
                     w2=m * h, b2=h, ln2_gamma=h, ln2_beta=h)
        arrs = {n: _slice(getattr(self, n), sizes[n], n) for n in self._names}
        blk = TransformerBlockF32(*(_ptr(arrs[n]) for n in self._names), h, cfg.num_heads,
                                  cfg.head_dim, m, cfg.eps)
        x = _slice(input, seq_len * h, "input")
        out = np.empty(seq_len * h, np.float32)
        _check(lib().gae_transformer_block_forward_f32_host(C.byref(blk), _ptr(x), seq_len, _ptr(out)))
        return out


class TuningFork(C.Structure):
    """Mirror of gae_tuning_fork = the reference's TuningFork
    (cuda_src/waller_fused_layer.cu:23-32)."""
    _fields_ = [("attn_scale", C.c_float), ("attn_temperature", C.c_float),
                ("residual_alpha", C.c_float), ("residual_beta", C.c_float),
                ("norm_eps", C.c_float), ("activation_type", C.c_int), ("mlp_gate", C.c_float),
                ("output_scale", C.c_float)]

    @classmethod
    def reference_defaults(cls, head_dim):
        """The reference benchmark's settings (waller_fused_layer.cu:311-318)."""
        return cls(1.0 / (math.sqrt(head_dim) * 127.0 * 127.0), 1.0, 1.0, 1.0, 1e-6, 0, 1.0, 1.0)


def symphony_forward(x, k, v, w_up, w_down, norm1_w, norm2_w, tuning: TuningFork, out=None,
                     workspace=None, stream=None):
    """The reference's fused symphony layer (cuda_src/waller_fused_layer.cu:64-247)
    on device tensors: x fp32 [N, d], k/v int8 [N, d], w_up fp32 [d, 4d],
    w_down fp32 [4d, d], norms fp32 [d].  Returns fp32 [N, d]."""
    torch = _torch()
    N, d = x.shape
    out = torch.empty_like(x) if out is None else out
    if workspace is None:
        workspace = torch.empty(lib().gae_symphony_workspace_bytes(N, d), dtype=torch.uint8,
                                device=x.device)
    for t in (x, k, v, w_up, w_down, norm1_w, norm2_w, out):
        if not t.is_contiguous():
            raise GAEError(1, "symphony_forward: tensors must be contiguous")
    _check(lib().gae_symphony_fwd(x.data_ptr(), k.data_ptr(), v.data_ptr(), w_up.data_ptr(),
                                  w_down.data_ptr(), norm1_w.data_ptr(), norm2_w.data_ptr(), N, d,
                                  C.byref(tuning), out.data_ptr(), workspace.data_ptr(),
                                  workspace.numel(), _stream_ptr(stream)))
    return out

"""ctypes bindings for the CPU parity oracle (oracle/gae_oracle.c).

TEST INFRASTRUCTURE ONLY: tests/, ``__graft_entry__.smoke()`` and bench.py's
CPU-baseline leg use this module as the checker.  The product library
(libgae.so) never imports or links it.

Every function mirrors one restated reference function; the docstrings cite
the Rust source line it follows (paths inside the reference project).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "build", "libgae_oracle.so")


def reference_root() -> str:
    """Root of the reference checkout: $GAE_REFERENCE_ROOT, else a
    `reference/` directory beside this repository.  It exists only where the
    reference is checked out (never on a GPU box); callers test for it."""
    return os.environ.get("GAE_REFERENCE_ROOT") or os.path.join(
        os.path.dirname(os.path.dirname(_HERE)), "reference")
_lib = None

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(dtype=np.int8, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_sz = C.c_size_t


def build() -> str:
    """Compile the oracle with its Makefile (gcc, -ffp-contract=off)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    root = reference_root()
    if os.path.exists(os.path.join(root, "cuda_src", "waller_fused_layer.cu")):
        subprocess.run(["make", "-s", "-C", _HERE, "ref", f"REF={os.path.abspath(root)}"], check=True)
    return _LIB_PATH


REF_SYMPHONY_PATH = os.path.join(_HERE, "_ref", "libref_symphony.so")
REF_SYMPHONY128_PATH = os.path.join(_HERE, "_ref", "libref_symphony128.so")


REF_WALLER_PATH = os.path.join(_HERE, "_ref", "libref_waller.so")


def ref_waller():
    """ctypes handle on the reference's own fp32 Waller operator kernels
    (cuda_src/waller_operator.cu, built by oracle/ref_waller_operator.cu), or
    None where they were not built.  Device pointers."""
    if not os.path.exists(REF_WALLER_PATH):
        return None
    L = C.CDLL(REF_WALLER_PATH)
    vp = C.c_void_p
    L.ref_waller_operator_fwd.argtypes = [vp, vp, vp, vp, C.c_int, C.c_int, C.c_float, vp]
    L.ref_waller_operator_multihead_fwd.argtypes = [vp, vp, vp, vp, C.c_int, C.c_int, C.c_int, C.c_float, vp]
    return L


REF_WALLER_INT8_PATH = os.path.join(_HERE, "_ref", "libref_waller_int8.so")


def ref_waller_int8():
    """ctypes handle on the reference's own INT8 Waller kernel
    (cuda_src/waller_operator_int8.cu, built by oracle/ref_waller_int8.cu), or
    None where it was not built.  Device pointers."""
    if not os.path.exists(REF_WALLER_INT8_PATH):
        return None
    L = C.CDLL(REF_WALLER_INT8_PATH)
    vp = C.c_void_p
    L.ref_waller_int8_fwd.argtypes = [vp, vp, vp, vp, C.c_int, C.c_int, C.c_float, C.c_float, vp]
    return L


def ref_symphony128():
    """ctypes handle on the reference's head_dim-128 fused layer kernel
    (waller_fused_realistic.cu, built by oracle/ref_symphony_realistic.cu),
    or None where it was not built.  Same arguments as ref_symphony_fwd."""
    if not os.path.exists(REF_SYMPHONY128_PATH):
        return None
    L = C.CDLL(REF_SYMPHONY128_PATH)
    vp = C.c_void_p
    L.ref_symphony128_fwd.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, C.c_int, _f32p, C.c_int, vp]
    if hasattr(L, "ref_symphony256_fwd"):  # head_dim 256 (waller_fused_256)
        L.ref_symphony256_fwd.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, C.c_int, _f32p, C.c_int, vp]
    return L


REF_KERNEL_BENCH_PATH = os.path.join(_HERE, "_ref", "libref_kernel_bench.so")


def ref_kernel_bench():
    """ctypes handle on the reference's published attention chain
    (cuda_src/waller_kernel_bench.cu: cuBLAS score/PV tiles + SIMT softmax)
    built from its source (oracle/ref_kernel_bench.cu), or None where it was
    not built.  ref_kernel_bench_tflops(seq_len, head_dim, tile, iters) runs
    the reference's own run_benchmark on one fp16 sequence and returns its
    TFLOPS figure (4 N^2 d per iteration)."""
    if not os.path.exists(REF_KERNEL_BENCH_PATH):
        return None
    L = C.CDLL(REF_KERNEL_BENCH_PATH)
    L.ref_kernel_bench_tflops.restype = C.c_float
    L.ref_kernel_bench_tflops.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int]
    return L


def ref_symphony():
    """ctypes handle on the reference's own symphony kernel built from its
    source (oracle/ref_symphony.cu), or None where it was not built.  Takes
    device pointers: ref_symphony_fwd(k, v, w_up, w_down, n1, n2, input,
    output, seq_len, tf[7] host array, act, stream)."""
    if not os.path.exists(REF_SYMPHONY_PATH):
        return None
    L = C.CDLL(REF_SYMPHONY_PATH)
    vp = C.c_void_p
    L.ref_symphony_fwd.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, C.c_int, _f32p, C.c_int, vp]
    return L


class _Softmax(C.Structure):
    _fields_ = [("max", C.c_float), ("sum", C.c_float)]


class _Welford(C.Structure):
    _fields_ = [("mean", C.c_float), ("m2", C.c_float), ("count", C.c_uint32)]


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH):
        build()
    L = C.CDLL(_LIB_PATH)
    L.ora_online_softmax_init.argtypes = [C.POINTER(_Softmax)]
    L.ora_online_softmax_update.argtypes = [C.POINTER(_Softmax), C.c_float]
    L.ora_online_softmax_probability.argtypes = [C.POINTER(_Softmax), C.c_float]
    L.ora_online_softmax_probability.restype = C.c_float
    L.ora_welford_init.argtypes = [C.POINTER(_Welford)]
    L.ora_welford_update.argtypes = [C.POINTER(_Welford), C.c_float]
    L.ora_welford_variance.argtypes = [C.POINTER(_Welford)]
    L.ora_welford_variance.restype = C.c_float
    L.ora_welford_std.argtypes = [C.POINTER(_Welford), C.c_float]
    L.ora_welford_std.restype = C.c_float
    L.ora_welford_merge.argtypes = [C.POINTER(_Welford)] * 3
    for f in ("ora_gelu", "ora_silu", "ora_relu", "ora_bf16_round"):
        getattr(L, f).argtypes = [C.c_float]
        getattr(L, f).restype = C.c_float
    L.ora_layernorm.argtypes = [_f32p, _f32p, _f32p, _sz, C.c_float, _f32p]
    L.ora_layernorm_batched.argtypes = [_f32p, _f32p, _f32p, _sz, _sz, C.c_float, _f32p]
    L.ora_mlp_block.argtypes = [_f32p] * 5 + [_sz, _sz, _f32p]
    L.ora_fused_mlp_layernorm.argtypes = [_f32p] * 8 + [_sz, _sz, C.c_float, _f32p]
    L.ora_transformer_block_forward.argtypes = (
        [_f32p, _sz, _sz, _sz, C.c_float] + [_f32p] * 10 + [_f32p])
    att = [_f32p, _f32p, _f32p, _sz, _sz, C.c_float, C.c_int, _f32p]
    L.ora_waller_operator.argtypes = att
    L.ora_waller_operator_parallel.argtypes = att
    L.ora_standard_attention.argtypes = att
    L.ora_attention_batched.argtypes = [
        _f32p, _f32p, _f32p, _sz, _sz, _sz, _sz, _sz, C.c_float, C.c_int,
        C.c_longlong, C.c_longlong, C.c_void_p, _sz, _f32p, C.c_void_p]
    L.ora_lse_merge.argtypes = [_f32p, _f32p, _f32p, _f32p, _sz, _sz]
    L.ora_quantize_rows_int8.argtypes = [_f32p, _sz, _sz, _i8p, _f32p]
    L.ora_int8_logits.argtypes = [_i8p, _i8p, _sz, _sz, _sz, _sz, _i32p]
    L.ora_attention_int8.argtypes = [
        _i8p, _i8p, _f32p, _f32p, _f32p, _sz, _sz, _sz, C.c_float, C.c_int,
        C.c_void_p, _sz, _f32p]
    L.ora_gpt2_layer.argtypes = (
        [_f32p, _sz, _sz, _sz, _sz, _sz, C.c_float] + [_f32p] * 12 + [C.c_int, _f32p])
    L.ora_symphony_layer.argtypes = [_f32p, _i8p, _i8p, _f32p, _f32p, _f32p, _f32p, _sz, _sz,
                                     _f32p, C.c_int, _f32p]
    L.ora_num_threads.restype = C.c_int
    L.ora_set_num_threads.argtypes = [C.c_int]
    _lib = L
    return L


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


# --- OnlineSoftmax (rust_src/src/online_softmax.rs:5-41) --------------------
class OnlineSoftmax:
    def __init__(self):
        self._s = _Softmax()
        lib().ora_online_softmax_init(C.byref(self._s))

    @property
    def max(self):
        return self._s.max

    @property
    def sum(self):
        return self._s.sum

    def update(self, score):
        lib().ora_online_softmax_update(C.byref(self._s), score)

    def probability(self, score):
        return lib().ora_online_softmax_probability(C.byref(self._s), score)


# --- WelfordState (rust_src/src/welford.rs:20-55) ---------------------------
class WelfordState:
    def __init__(self):
        self._w = _Welford()
        lib().ora_welford_init(C.byref(self._w))

    @property
    def mean(self):
        return self._w.mean

    @property
    def count(self):
        return self._w.count

    def update(self, x):
        lib().ora_welford_update(C.byref(self._w), x)

    def variance(self):
        return lib().ora_welford_variance(C.byref(self._w))

    def std(self, eps):
        return lib().ora_welford_std(C.byref(self._w), eps)

    @staticmethod
    def merge(a, b):
        out = WelfordState()
        lib().ora_welford_merge(C.byref(a._w), C.byref(b._w), C.byref(out._w))
        return out


def gelu(x):
    return lib().ora_gelu(x)


def silu(x):
    return lib().ora_silu(x)


def relu(x):
    return lib().ora_relu(x)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even to bf16, returned widened to fp32."""
    u = _f32(x).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32).reshape(np.shape(x))


def layernorm(x, gamma, beta, eps):
    x = _f32(x); out = np.empty_like(x)
    lib().ora_layernorm(x, _f32(gamma), _f32(beta), x.size, eps, out)
    return out


def layernorm_batched(x, gamma, beta, batch, hidden, eps):
    x = _f32(x); out = np.empty_like(x)
    lib().ora_layernorm_batched(x, _f32(gamma), _f32(beta), batch, hidden, eps, out)
    return out


def mlp_block(x, w1, b1, w2, b2, hidden, mlp):
    out = np.empty(hidden, np.float32)
    lib().ora_mlp_block(_f32(x), _f32(w1), _f32(b1), _f32(w2), _f32(b2), hidden, mlp, out)
    return out


def fused_mlp_layernorm(x, res, w1, b1, w2, b2, g, b, hidden, mlp, eps):
    out = np.empty(hidden, np.float32)
    lib().ora_fused_mlp_layernorm(_f32(x), _f32(res), _f32(w1), _f32(b1), _f32(w2), _f32(b2),
                                  _f32(g), _f32(b), hidden, mlp, eps, out)
    return out


def transformer_block_forward(x, seq_len, h, m, eps, wv, wo, ln1_g, ln1_b, w1, b1, w2, b2,
                              ln2_g, ln2_b):
    out = np.empty(seq_len * h, np.float32)
    lib().ora_transformer_block_forward(_f32(x), seq_len, h, m, eps, _f32(wv), _f32(wo),
                                        _f32(ln1_g), _f32(ln1_b), _f32(w1), _f32(b1),
                                        _f32(w2), _f32(b2), _f32(ln2_g), _f32(ln2_b), out)
    return out


def waller_operator(q, k, v, seq_len, head_dim, scale, causal=True, parallel=False):
    """rust_src/src/waller_operator.rs:8-59 (parallel: :62-109)."""
    out = np.empty(seq_len * head_dim, np.float32)
    f = lib().ora_waller_operator_parallel if parallel else lib().ora_waller_operator
    f(_f32(q).ravel(), _f32(k).ravel(), _f32(v).ravel(), seq_len, head_dim, scale,
      int(causal), out)
    return out


def standard_attention(q, k, v, seq_len, head_dim, scale, causal=True):
    """rust_src/src/standard_attention.rs:13-65."""
    out = np.empty(seq_len * head_dim, np.float32)
    lib().ora_standard_attention(_f32(q).ravel(), _f32(k).ravel(), _f32(v).ravel(), seq_len,
                                 head_dim, scale, int(causal), out)
    return out


def attention_batched(q, k, v, scale, causal, q_offset=0, kv_offset=0, rows=None,
                      want_lse=False):
    """Batched Waller recurrence. q [B,H,Nq,d], k/v [B,H,Nkv,d] fp32."""
    q = _f32(q); k = _f32(k); v = _f32(v)
    B, H, nq, d = q.shape
    nkv = k.shape[2]
    out = np.zeros_like(q)
    lse = np.full((B, H, nq), np.nan, np.float32) if want_lse else None
    rows_arr = None if rows is None else np.ascontiguousarray(rows, dtype=np.int64)
    lib().ora_attention_batched(
        q, k, v, B, H, nq, nkv, d, scale, int(causal), q_offset, kv_offset,
        None if rows_arr is None else rows_arr.ctypes.data_as(C.c_void_p),
        0 if rows_arr is None else rows_arr.size, out,
        None if lse is None else lse.ctypes.data_as(C.c_void_p))
    return (out, lse) if want_lse else out


def lse_merge(o1, l1, o2, l2):
    o1 = _f32(o1).copy(); l1 = _f32(l1).copy()
    d = o1.shape[-1]
    rows = o1.size // d
    lib().ora_lse_merge(o1, l1, _f32(o2), _f32(l2), rows, d)
    return o1, l1


def quantize_rows_int8(x):
    x = _f32(x)
    d = x.shape[-1]
    rows = x.size // d
    q = np.empty(x.shape, np.int8)
    s = np.empty(x.shape[:-1], np.float32)
    lib().ora_quantize_rows_int8(x, rows, d, q, s)
    return q, s


def int8_logits(q, k):
    """q [BH,Nq,d], k [BH,Nkv,d] int8 -> int32 [BH,Nq,Nkv]."""
    q = np.ascontiguousarray(q, np.int8); k = np.ascontiguousarray(k, np.int8)
    BH, nq, d = q.shape
    nkv = k.shape[1]
    out = np.empty((BH, nq, nkv), np.int32)
    lib().ora_int8_logits(q, k, BH, nq, nkv, d, out)
    return out


def attention_int8(q, k, sq, sk, v, scale, causal=False, rows=None):
    q = np.ascontiguousarray(q, np.int8); k = np.ascontiguousarray(k, np.int8)
    BH, n, d = q.shape
    out = np.zeros((BH, n, d), np.float32)
    rows_arr = None if rows is None else np.ascontiguousarray(rows, dtype=np.int64)
    lib().ora_attention_int8(
        q, k, _f32(sq), _f32(sk), _f32(v), BH, n, d, scale, int(causal),
        None if rows_arr is None else rows_arr.ctypes.data_as(C.c_void_p),
        0 if rows_arr is None else rows_arr.size, out)
    return out


def gpt2_layer(x, B, S, D, nh, F, eps, w, round_bf16=True):
    """Pre-norm GPT-2 layer; w = dict of fp32 weights (see gae_oracle.c)."""
    out = np.empty((B * S, D), np.float32)
    lib().ora_gpt2_layer(_f32(x), B, S, D, nh, F, eps, _f32(w["ln1_g"]), _f32(w["ln1_b"]),
                         _f32(w["wqkv"]), _f32(w["bqkv"]), _f32(w["wproj"]), _f32(w["bproj"]),
                         _f32(w["ln2_g"]), _f32(w["ln2_b"]), _f32(w["wfc"]), _f32(w["bfc"]),
                         _f32(w["wfc2"]), _f32(w["bfc2"]), int(round_bf16), out)
    return out


def num_threads() -> int:
    return lib().ora_num_threads()


def use_all_cores() -> int:
    """Runs later oracle parallel regions on every core this process may use
    (launchers such as torchrun export OMP_NUM_THREADS=1); returns the count."""
    n = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    lib().ora_set_num_threads(n)
    return num_threads()


def symphony_layer(x, k, v, w_up, w_down, n1, n2, tuning, act=0):
    """cuda_src/waller_fused_layer.cu:64-247.  tuning = (attn_scale, temperature,
    alpha, beta, eps, mlp_gate, output_scale)."""
    x = _f32(x)
    n, d = x.shape
    out = np.empty_like(x)
    lib().ora_symphony_layer(x, np.ascontiguousarray(k, np.int8), np.ascontiguousarray(v, np.int8),
                             _f32(w_up), _f32(w_down), _f32(n1), _f32(n2), n, d,
                             _f32(np.asarray(tuning, np.float32)), int(act), out)
    return out


def attention_bwd(q, k, v, dout, scale, causal):
    """Attention gradients (an extension: the reference is inference-only),
    double precision from the definition.  q, dout [BH, Nq, D]; k, v
    [BH, Nkv, D].  Returns (dq, dk, dv) float32."""
    q, k, v, dout = (_f32(a) for a in (q, k, v, dout))
    BH, nq, d = q.shape
    nkv = k.shape[1]
    dq, dk, dv = np.empty_like(q), np.empty_like(k), np.empty_like(v)
    L = lib()
    L.ora_attention_bwd.argtypes = [_f32p, _f32p, _f32p, _f32p, _sz, _sz, _sz, _sz, C.c_float, C.c_int,
                                    _f32p, _f32p, _f32p]
    L.ora_attention_bwd(q, k, v, dout, BH, nq, nkv, d, float(scale), int(bool(causal)), dq, dk, dv)
    return dq, dk, dv

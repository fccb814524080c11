"""numpy/ctypes front end of the CPU oracle (oracle/strata_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg as the checker, never by the product path.
Parity of the decoder ops (RMSNorm, RoPE, SwiGLU, attention, quantisation)
is unpinned by the reference, which has none of them; the reference-kernel
restatements are pinned by the reference's own known-answer tests
(tests/golden/reference_kat.json).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libstrata_oracle.so")


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = C.CDLL(LIB_PATH)
        i64, f32, f64, i32, u64 = C.c_int64, C.c_float, C.c_double, C.c_int32, C.c_uint64
        P = C.c_void_p
        sigs = {
            "ora_f32_to_bf16": (C.c_uint16, [f32]),
            "ora_bf16_to_f32": (f32, [C.c_uint16]),
            "ora_erf": (f32, [f32]),
            "ora_gelu": (f32, [f32]),
            "ora_map_gelu": (None, [P, i64, P]),
            "ora_map_exp": (None, [P, i64, P]),
            "ora_map_log": (None, [P, i64, P]),
            "ora_elementwise": (C.c_int, [C.c_int, P, P, C.c_int, P, P, C.c_int, P, P, C.c_int]),
            "ora_broadcast_to": (C.c_int, [P, P, C.c_int, P, P, C.c_int]),
            "ora_matmul": (None, [P, P, i64, i64, i64, P]),
            "ora_linear": (None, [P, P, P, i64, i64, i64, P]),
            "ora_softmax": (None, [P, i64, i64, P]),
            "ora_layer_norm": (None, [P, P, P, i64, i64, f32, P]),
            "ora_transpose2": (None, [P, i64, i64, P]),
            "ora_slice_cols": (i64, [P, i64, i64, i64, i64, i64, P]),
            "ora_quant_w8pc": (None, [P, i64, i64, P, P]),
            "ora_quant_w4g32": (None, [P, i64, i64, P, P]),
            "ora_quant_mx": (None, [P, i64, i64, C.c_int, P, P]),
            "ora_dequant_mx": (None, [P, P, i64, i64, C.c_int, P]),
            "ora_linear_mx_mt": (None, [P, P, P, C.c_int, i64, i64, i64, P, C.c_int]),
            "ora_e4m3_to_f32": (C.c_float, [C.c_uint8]),
            "ora_e2m1_to_f32": (C.c_float, [C.c_uint8]),
            "ora_f32_to_e4m3": (C.c_uint8, [C.c_float]),
            "ora_f32_to_e2m1": (C.c_uint8, [C.c_float]),
            "ora_dequant_w8pc": (None, [P, P, i64, i64, P]),
            "ora_dequant_w4g32": (None, [P, P, i64, i64, P]),
            "ora_rms_norm": (None, [P, P, i64, i64, f32, P]),
            "ora_rope": (None, [P, P, i64, i64, i64, f64, P]),
            "ora_silu": (f32, [f32]),
            "ora_swiglu": (None, [P, P, i64, P]),
            "ora_attention": (None, [P, P, P, P, P, i64, i64, i64, i64, i64, P]),
            "ora_attention_mt": (None, [P, P, P, P, P, i64, i64, i64, i64, i64, P, C.c_int]),
            "ora_linear_w4g32": (None, [P, P, P, i64, i64, i64, P]),
            "ora_linear_w8pc": (None, [P, P, P, i64, i64, i64, P]),
            "ora_linear_w4g32_mt": (None, [P, P, P, i64, i64, i64, P, C.c_int]),
            "ora_linear_w8pc_mt": (None, [P, P, P, i64, i64, i64, P, C.c_int]),
            "ora_embed": (C.c_int, [P, i64, P, i64, i64, P]),
            "ora_argmax": (None, [P, i64, i64, P]),
            "ora_normal_f32": (None, [u64, i64, f64, f64, P]),
            "ora_uniform_i32": (None, [u64, i64, i32, i32, P]),
            "ora_max_threads": (C.c_int, []),
            "ora_round_bf16": (None, [P, i64, P]),
            "ora_widen_bf16": (None, [P, i64, P]),
        }
        for name, (res, args) in sigs.items():
            fn = getattr(_lib, name)
            fn.restype = res
            fn.argtypes = args
    return _lib


def _p(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


# ---- bf16 ------------------------------------------------------------------
def to_bf16(x) -> np.ndarray:
    x = _f32(x)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().ora_round_bf16(_p(x), x.size, _p(out))
    return out


def from_bf16(x) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.uint16)
    out = np.empty(x.shape, dtype=np.float32)
    lib().ora_widen_bf16(_p(x), x.size, _p(out))
    return out


def round_bf16(x) -> np.ndarray:
    return from_bf16(to_bf16(x))


# ---- inputs ----------------------------------------------------------------
def normal(seed: int, shape, std: float = 1.0, mean: float = 0.0) -> np.ndarray:
    n = int(np.prod(shape)) if len(shape) else 1
    out = np.empty(n, dtype=np.float32)
    lib().ora_normal_f32(seed, n, mean, std, _p(out))
    return out.reshape(shape)


def uniform_i32(seed: int, n: int, lo: int, hi: int) -> np.ndarray:
    out = np.empty(n, dtype=np.int32)
    lib().ora_uniform_i32(seed, n, lo, hi, _p(out))
    return out


# ---- reference kernels -----------------------------------------------------
def gelu(x):
    x = _f32(x)
    out = np.empty_like(x)
    lib().ora_map_gelu(_p(x), x.size, _p(out))
    return out


def exp(x):
    x = _f32(x)
    out = np.empty_like(x)
    lib().ora_map_exp(_p(x), x.size, _p(out))
    return out


def log(x):
    x = _f32(x)
    out = np.empty_like(x)
    lib().ora_map_log(_p(x), x.size, _p(out))
    return out


def elementwise(op: str, a, b, out_shape):
    a, b = _f32(a), _f32(b)
    out = np.empty(out_shape, dtype=np.float32)
    ad = np.array(a.shape, dtype=np.int64)
    bd = np.array(b.shape, dtype=np.int64)
    od = np.array(out_shape, dtype=np.int64)
    rc = lib().ora_elementwise(0 if op == "add" else 1, _p(a), _p(ad), a.ndim, _p(b), _p(bd),
                               b.ndim, _p(out), _p(od), len(out_shape))
    if rc:
        raise ValueError("operands do not broadcast")
    return out


def broadcast_to(a, out_shape):
    a = _f32(a)
    out = np.empty(out_shape, dtype=np.float32)
    ad = np.array(a.shape, dtype=np.int64)
    od = np.array(out_shape, dtype=np.int64)
    if lib().ora_broadcast_to(_p(a), _p(ad), a.ndim, _p(out), _p(od), len(out_shape)):
        raise ValueError("does not broadcast")
    return out


def matmul(a, b):
    a, b = _f32(a), _f32(b)
    m, k = a.shape
    k2, n = b.shape
    if k != k2:
        raise ValueError("inner dimensions")
    out = np.empty((m, n), dtype=np.float32)
    lib().ora_matmul(_p(a), _p(b), m, k, n, _p(out))
    return out


def linear(x, w, bias=None):
    x, w = _f32(x), _f32(w)
    m, k = x.shape
    n = w.shape[0]
    out = np.empty((m, n), dtype=np.float32)
    b_keep = _f32(bias) if bias is not None else None
    lib().ora_linear(_p(x), _p(w), _p(b_keep) if b_keep is not None else None, m, k, n, _p(out))
    return out


def softmax(x):
    x = _f32(x)
    out = np.empty_like(x)
    cols = x.shape[-1]
    lib().ora_softmax(_p(x), x.size // cols, cols, _p(out))
    return out


def layer_norm(x, gamma, beta, eps=1e-5):
    x, g, b = _f32(x), _f32(gamma), _f32(beta)
    out = np.empty_like(x)
    cols = x.shape[-1]
    lib().ora_layer_norm(_p(x), _p(g), _p(b), x.size // cols, cols, eps, _p(out))
    return out


def transpose2(x):
    x = _f32(x)
    out = np.empty((x.shape[1], x.shape[0]), dtype=np.float32)
    lib().ora_transpose2(_p(x), x.shape[0], x.shape[1], _p(out))
    return out


def slice_cols(x, start, end, stride):
    x = _f32(x)
    out = np.empty(x.shape[0] * max(x.shape[1], 1), dtype=np.float32)
    n = lib().ora_slice_cols(_p(x), x.shape[0], x.shape[1], start, end, stride, _p(out))
    return out[: x.shape[0] * n].reshape(x.shape[0], n)


# ---- quantisation ----------------------------------------------------------
def quant_w4g32(w):
    w = _f32(w)
    n, k = w.shape
    packed = np.empty((n, k // 2), dtype=np.uint8)
    s = np.empty((n, k // 32), dtype=np.uint16)
    lib().ora_quant_w4g32(_p(w), n, k, _p(packed), _p(s))
    return packed, s


def quant_w8pc(w):
    w = _f32(w)
    n, k = w.shape
    q = np.empty((n, k), dtype=np.int8)
    s = np.empty((n,), dtype=np.float32)
    lib().ora_quant_w8pc(_p(w), n, k, _p(q), _p(s))
    return q, s


def dequant_w4g32(packed, s):
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    s = np.ascontiguousarray(s, dtype=np.uint16)
    n, k = packed.shape[0], packed.shape[1] * 2
    out = np.empty((n, k), dtype=np.float32)
    lib().ora_dequant_w4g32(_p(packed), _p(s), n, k, _p(out))
    return out


MX_FORMATS = {"mxfp8": 0, "mxfp4": 1}


def quant_mx(w, fmt: str):
    """MX quantisation (block 32 along k): E4M3 codes [n, k] (mxfp8) or E2M1
    codes packed two per byte [n, k/2] (mxfp4), and E8M0 scales [n, k/32]."""
    w = _f32(w)
    n, k = w.shape
    f = MX_FORMATS[fmt]
    codes = np.zeros((n, k if f == 0 else k // 2), dtype=np.uint8)
    s = np.empty((n, k // 32), dtype=np.uint8)
    lib().ora_quant_mx(_p(w), n, k, f, _p(codes), _p(s))
    return codes, s


def dequant_mx(codes, s, fmt: str):
    codes = np.ascontiguousarray(codes, dtype=np.uint8)
    s = np.ascontiguousarray(s, dtype=np.uint8)
    f = MX_FORMATS[fmt]
    n = codes.shape[0]
    k = codes.shape[1] * (1 if f == 0 else 2)
    out = np.empty((n, k), dtype=np.float32)
    lib().ora_dequant_mx(_p(codes), _p(s), n, k, f, _p(out))
    return out


def linear_mx(x, codes, s, fmt: str, threads: int = 1):
    x = _f32(x)
    codes = np.ascontiguousarray(codes, dtype=np.uint8)
    s = np.ascontiguousarray(s, dtype=np.uint8)
    m, k = x.shape
    n = codes.shape[0]
    out = np.empty((m, n), dtype=np.float32)
    lib().ora_linear_mx_mt(_p(x), _p(codes), _p(s), MX_FORMATS[fmt], m, k, n, _p(out), max(1, threads))
    return out


def dequant_w8pc(q, s):
    q = np.ascontiguousarray(q, dtype=np.int8)
    s = _f32(s)
    n, k = q.shape
    out = np.empty((n, k), dtype=np.float32)
    lib().ora_dequant_w8pc(_p(q), _p(s), n, k, _p(out))
    return out


# ---- decoder ops -----------------------------------------------------------
def rms_norm(x, g, eps=1e-5):
    x, g = _f32(x), _f32(g)
    out = np.empty_like(x)
    cols = x.shape[-1]
    lib().ora_rms_norm(_p(x), _p(g), x.size // cols, cols, eps, _p(out))
    return out


def rope(x, pos, head_dim, theta=10000.0):
    x = _f32(x)
    pos = np.ascontiguousarray(pos, dtype=np.int32)
    cols = x.shape[-1]
    rows = x.size // cols
    out = np.empty_like(x)
    lib().ora_rope(_p(x), _p(pos), rows, cols // head_dim, head_dim, theta, _p(out))
    return out


def swiglu(g, u):
    g, u = _f32(g), _f32(u)
    out = np.empty_like(g)
    lib().ora_swiglu(_p(g), _p(u), g.size, _p(out))
    return out


def attention(q, k_cache, v_cache, seq, pos, heads, kv_heads, head_dim, threads: int = 1):
    q, kc, vc = _f32(q), _f32(k_cache), _f32(v_cache)
    seq = np.ascontiguousarray(seq, dtype=np.int32)
    pos = np.ascontiguousarray(pos, dtype=np.int32)
    rows = q.size // (heads * head_dim)
    out = np.empty_like(q)
    max_len = kc.shape[2]
    if threads > 1:
        lib().ora_attention_mt(_p(q), _p(kc), _p(vc), _p(seq), _p(pos), rows, heads, kv_heads,
                               head_dim, max_len, _p(out), threads)
    else:
        lib().ora_attention(_p(q), _p(kc), _p(vc), _p(seq), _p(pos), rows, heads, kv_heads,
                            head_dim, max_len, _p(out))
    return out


def linear_w4g32(x, packed, s, threads: int = 1):
    x = _f32(x)
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    s = np.ascontiguousarray(s, dtype=np.uint16)
    m, k = x.shape
    n = packed.shape[0]
    out = np.empty((m, n), dtype=np.float32)
    if threads > 1:
        lib().ora_linear_w4g32_mt(_p(x), _p(packed), _p(s), m, k, n, _p(out), threads)
    else:
        lib().ora_linear_w4g32(_p(x), _p(packed), _p(s), m, k, n, _p(out))
    return out


def linear_w8pc(x, q, s, threads: int = 1):
    x = _f32(x)
    q = np.ascontiguousarray(q, dtype=np.int8)
    s = _f32(s)
    m, k = x.shape
    n = q.shape[0]
    out = np.empty((m, n), dtype=np.float32)
    if threads > 1:
        lib().ora_linear_w8pc_mt(_p(x), _p(q), _p(s), m, k, n, _p(out), threads)
    else:
        lib().ora_linear_w8pc(_p(x), _p(q), _p(s), m, k, n, _p(out))
    return out


def embed(ids, table):
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    table = _f32(table)
    out = np.zeros((ids.size, table.shape[1]), dtype=np.float32)
    rc = lib().ora_embed(_p(ids), ids.size, _p(table), table.shape[0], table.shape[1], _p(out))
    return out, rc


def argmax(x):
    x = _f32(x)
    cols = x.shape[-1]
    out = np.empty(x.size // cols, dtype=np.int32)
    lib().ora_argmax(_p(x), x.size // cols, cols, _p(out))
    return out


def max_threads() -> int:
    return lib().ora_max_threads()

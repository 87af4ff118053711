"""numpy front end of the CPU oracle -- TEST INFRASTRUCTURE ONLY.

`Oracle` wraps liboracle.so (our restatement of the reference goldens, oracle.cpp);
`Reference` wraps _ref/libref_golden.so (the reference's own golden sources compiled by
oracle/Makefile).  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
module; the product library never does.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "liboracle.so"
REF_SO = HERE / "_ref" / "libref_golden.so"

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_i64 = C.c_int64
_sz = C.c_size_t


def build(ref: str | None = None) -> None:
    """Runs oracle/Makefile (liboracle.so, and _ref/libref_golden.so when the reference tree exists)."""
    cmd = ["make", "-s", "-C", str(HERE)]
    if ref:
        cmd.append(f"REF={ref}")
    subprocess.run(cmd, check=True)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _opt_f32(a):
    return None if a is None else _f32(a).ctypes.data_as(C.c_void_p)


class Oracle:
    def __init__(self, path: Path = ORACLE_SO):
        if not Path(path).exists():
            build()
        self.lib = lib = C.CDLL(str(path))
        lib.oracle_uniform_f32.argtypes = [_f32p, _sz, C.c_uint64, C.c_float, C.c_float]
        lib.oracle_normal_f32.argtypes = [_f32p, _sz, C.c_uint64, C.c_float, C.c_float]
        lib.oracle_rope_cos_sin.argtypes = [_sz, _sz, _f32p, _f32p, C.c_float]
        lib.oracle_f32_to_bf16.argtypes = [_f32p, _u16p, _sz]
        lib.oracle_bf16_to_f32.argtypes = [_u16p, _f32p, _sz]
        lib.oracle_f32_to_f16.argtypes = [_f32p, _u16p, _sz]
        lib.oracle_f16_to_f32.argtypes = [_u16p, _f32p, _sz]
        lib.oracle_elementwise_add.argtypes = [_f32p, _f32p, _f32p, _sz]
        lib.oracle_axpy_scalar_affine.argtypes = [_f32p, _f32p, _sz, C.c_float, C.c_float]
        lib.oracle_broadcast_binary.argtypes = [_f32p, _f32p, _f32p, _f32p, _i64, _i64, _i64, _i64, _i64]
        lib.oracle_activation_gelu_silu.argtypes = [_f32p, _f32p, _sz, C.c_int]
        lib.oracle_reduce_sum_lastdim.argtypes = [_f32p, _f32p, _i64, _i64, _i64]
        lib.oracle_transpose.argtypes = [C.c_void_p, C.c_void_p, C.c_int, _i64, _i64, _i64, _i64, C.c_int]
        lib.oracle_layer_norm.argtypes = [_f32p, _f32p, _f32p, _f32p, _i64, _i64, C.c_float]
        lib.oracle_rms_norm_rope.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, _i64, _i64, _i64, C.c_float, _i64,
                                             _i64, C.c_int]
        lib.oracle_matmul_bias.argtypes = [_f32p, _f32p, C.c_void_p, _f32p, _i64, _i64, _i64]
        fa_args = [_f32p, _f32p, _f32p, _f32p, C.c_void_p, _i64, _i64, _i64, _i64, _i64, _i64, C.c_float, C.c_int]
        lib.oracle_flash_attention_fwd.argtypes = fa_args
        lib.oracle_flash_attention_fwd_mt.argtypes = fa_args + [C.c_int]
        lib.oracle_flash_attention_bwd.argtypes = [_f32p] * 7 + [_i64] * 6 + [C.c_float, C.c_int]

    # ---- generators / codecs ----
    def uniform(self, n, seed, lo=-1.0, hi=1.0):
        out = np.empty(int(n), np.float32)
        self.lib.oracle_uniform_f32(out, out.size, seed, lo, hi)
        return out

    def normal(self, n, seed, mean=0.0, std=1.0):
        out = np.empty(int(n), np.float32)
        self.lib.oracle_normal_f32(out, out.size, seed, mean, std)
        return out

    def rope_cos_sin(self, seq_len, half, base=10000.0):
        c = np.empty(seq_len * half, np.float32)
        s = np.empty(seq_len * half, np.float32)
        self.lib.oracle_rope_cos_sin(seq_len, half, c, s, base)
        return c.reshape(seq_len, half), s.reshape(seq_len, half)

    def to_bf16(self, a):
        a = _f32(a)
        out = np.empty(a.shape, np.uint16)
        self.lib.oracle_f32_to_bf16(a.reshape(-1), out.reshape(-1), a.size)
        return out

    def from_bf16(self, a):
        a = np.ascontiguousarray(a, np.uint16)
        out = np.empty(a.shape, np.float32)
        self.lib.oracle_bf16_to_f32(a.reshape(-1), out.reshape(-1), a.size)
        return out

    def to_f16(self, a):
        a = _f32(a)
        out = np.empty(a.shape, np.uint16)
        self.lib.oracle_f32_to_f16(a.reshape(-1), out.reshape(-1), a.size)
        return out

    def from_f16(self, a):
        a = np.ascontiguousarray(a, np.uint16)
        out = np.empty(a.shape, np.float32)
        self.lib.oracle_f16_to_f32(a.reshape(-1), out.reshape(-1), a.size)
        return out

    # ---- goldens ----
    def elementwise_add(self, x, y):
        x, y = _f32(x), _f32(y)
        z = np.empty_like(x)
        self.lib.oracle_elementwise_add(x.reshape(-1), y.reshape(-1), z.reshape(-1), x.size)
        return z

    def axpy_scalar_affine(self, x, alpha, beta):
        x = _f32(x)
        y = np.empty_like(x)
        self.lib.oracle_axpy_scalar_affine(x.reshape(-1), y.reshape(-1), x.size, alpha, beta)
        return y

    def broadcast_binary(self, x, y, bias, y_batch):
        x = _f32(x)
        B, Cc, H, W = x.shape
        z = np.empty_like(x)
        self.lib.oracle_broadcast_binary(x, _f32(y).reshape(-1), _f32(bias).reshape(-1), z, B, Cc, H, W, y_batch)
        return z

    def activation_gelu_silu(self, x, act):
        x = _f32(x)
        y = np.empty_like(x)
        self.lib.oracle_activation_gelu_silu(x.reshape(-1), y.reshape(-1), x.size, 0 if act == "gelu" else 1)
        return y

    def reduce_sum_lastdim(self, x):
        x = _f32(x)
        K = x.shape[-1]
        out = np.empty(x.shape[:-1], np.float32)
        self.lib.oracle_reduce_sum_lastdim(x.reshape(-1), out.reshape(-1), 1, x.size // K, K)
        return out

    def transpose(self, x, mode):
        x = np.ascontiguousarray(x)
        if mode == 0:
            M, N = x.shape
            dims, shape = (M, N, 0, 0), (N, M)
        elif mode == 1:
            n, c, h, w = x.shape
            dims, shape = (n, c, h, w), (n, h, w, c)
        else:
            n, h, w, c = x.shape
            dims, shape = (n, c, h, w), (n, c, h, w)
        out = np.empty(shape, x.dtype)
        self.lib.oracle_transpose(x.ctypes.data_as(C.c_void_p), out.ctypes.data_as(C.c_void_p), mode, *dims,
                                  x.dtype.itemsize)
        return out

    def layer_norm(self, x, gamma, beta, eps):
        x = _f32(x)
        y = np.empty_like(x)
        last = x.shape[-1]
        self.lib.oracle_layer_norm(x.reshape(-1), _f32(gamma), _f32(beta), y.reshape(-1), x.size // last, last, eps)
        return y

    def rms_norm_rope(self, x, weight, cos, sin, rot, eps, heads=1, style=0):
        """x [B, S, H] (heads=1) or [B, S, heads, H]."""
        x = _f32(x)
        out = np.empty_like(x)
        H = x.shape[-1]
        S = x.shape[1]
        self.lib.oracle_rms_norm_rope(x.reshape(-1), _f32(weight), _f32(cos).reshape(-1), _f32(sin).reshape(-1),
                                      out.reshape(-1), x.size // H, H, rot, eps, heads, S, style)
        return out

    def matmul_bias(self, A, B, bias=None):
        A, B = _f32(A), _f32(B)
        M, K = A.shape
        N = B.shape[1]
        out = np.empty((M, N), np.float32)
        b = None if bias is None else _f32(bias)
        self.lib.oracle_matmul_bias(A, B, None if b is None else b.ctypes.data_as(C.c_void_p), out, M, K, N)
        return out

    def flash_attention_fwd(self, q, k, v, scale, causal, threads: int = 1):
        """q [B,H,S_q,D], k [B,H,S_k,D], v [B,H,S_k,D_v] -> (O, lse)."""
        q, k, v = _f32(q), _f32(k), _f32(v)
        B, H, S_q, D = q.shape
        S_k, D_v = k.shape[2], v.shape[3]
        o = np.empty((B, H, S_q, D_v), np.float32)
        lse = np.empty((B, H, S_q), np.float32)
        args = (q.reshape(-1), k.reshape(-1), v.reshape(-1), o.reshape(-1), lse.ctypes.data_as(C.c_void_p), B, H, S_q,
                S_k, D, D_v, scale, 1 if causal else 0)
        if threads > 1:
            self.lib.oracle_flash_attention_fwd_mt(*args, threads)
        else:
            self.lib.oracle_flash_attention_fwd(*args)
        return o, lse

    def flash_attention_bwd(self, q, k, v, do, scale, causal):
        """q [B,H,S_q,D], k [B,H,S_k,D], v [B,H,S_k,D_v], dO [B,H,S_q,D_v] -> (dQ, dK, dV), fp64 math."""
        q, k, v, do = _f32(q), _f32(k), _f32(v), _f32(do)
        B, H, S_q, D = q.shape
        S_k, D_v = k.shape[2], v.shape[3]
        dq, dk, dv = np.empty_like(q), np.empty_like(k), np.empty_like(v)
        self.lib.oracle_flash_attention_bwd(q.reshape(-1), k.reshape(-1), v.reshape(-1), do.reshape(-1),
                                            dq.reshape(-1), dk.reshape(-1), dv.reshape(-1), B, H, S_q, S_k, D, D_v,
                                            scale, 1 if causal else 0)
        return dq, dk, dv


class Reference:
    """The reference harness's own goldens (compiled from its sources), when available."""

    def __init__(self, path: Path = REF_SO):
        if not Path(path).exists():
            raise FileNotFoundError(f"{path} not built (needs the reference tree; see oracle/Makefile)")
        self.lib = lib = C.CDLL(str(path))
        lib.ref_generate_random_float.argtypes = [_f32p, _sz, C.c_uint64, C.c_float, C.c_float]
        lib.ref_generate_rope_cos_sin.argtypes = [_sz, _sz, _f32p, _f32p, C.c_float]
        lib.ref_elementwise_add.argtypes = [_f32p, _f32p, _f32p, _sz]
        lib.ref_axpy_scalar_affine.argtypes = [_f32p, _f32p, _sz, C.c_float, C.c_float]
        lib.ref_broadcast_binary.argtypes = [_f32p, _f32p, _f32p, _f32p, _i64, _i64, _i64, _i64, _i64]
        lib.ref_activation_gelu_silu.argtypes = [_f32p, _f32p, _sz, C.c_int]
        lib.ref_reduce_sum_lastdim.argtypes = [_f32p, _f32p, _i64, _i64, _i64]
        lib.ref_transpose.argtypes = [C.c_void_p, C.c_void_p, C.c_int, _i64, _i64, _i64, _i64, C.c_int]
        lib.ref_layer_norm.argtypes = [_f32p, _f32p, _f32p, _f32p, _i64, _i64, C.c_float]
        lib.ref_rms_norm_rope_fused.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, _i64, _i64, _i64, _i64, C.c_float]
        lib.ref_matmul_bias.argtypes = [_f32p, _f32p, C.c_void_p, _f32p, _i64, _i64, _i64]
        fa = [_f32p, _f32p, _f32p, _f32p, _i64, _i64, _i64, _i64, _i64, _i64, C.c_float, C.c_int]
        lib.ref_flash_attention_fwd.argtypes = fa
        lib.ref_flash_attention_fwd_mt.argtypes = fa + [C.c_int]

    def uniform(self, n, seed, lo=-1.0, hi=1.0):
        out = np.empty(int(n), np.float32)
        self.lib.ref_generate_random_float(out, out.size, seed, lo, hi)
        return out

    def rope_cos_sin(self, seq_len, half, base=10000.0):
        c = np.empty(seq_len * half, np.float32)
        s = np.empty(seq_len * half, np.float32)
        self.lib.ref_generate_rope_cos_sin(seq_len, half, c, s, base)
        return c.reshape(seq_len, half), s.reshape(seq_len, half)

    def elementwise_add(self, x, y):
        x, y = _f32(x), _f32(y)
        z = np.empty_like(x)
        self.lib.ref_elementwise_add(x.reshape(-1), y.reshape(-1), z.reshape(-1), x.size)
        return z

    def axpy_scalar_affine(self, x, alpha, beta):
        x = _f32(x)
        y = np.empty_like(x)
        self.lib.ref_axpy_scalar_affine(x.reshape(-1), y.reshape(-1), x.size, alpha, beta)
        return y

    def broadcast_binary(self, x, y, bias, y_batch):
        x = _f32(x)
        B, Cc, H, W = x.shape
        z = np.empty_like(x)
        self.lib.ref_broadcast_binary(x, _f32(y).reshape(-1), _f32(bias).reshape(-1), z, B, Cc, H, W, y_batch)
        return z

    def activation_gelu_silu(self, x, act):
        x = _f32(x)
        y = np.empty_like(x)
        self.lib.ref_activation_gelu_silu(x.reshape(-1), y.reshape(-1), x.size, 0 if act == "gelu" else 1)
        return y

    def reduce_sum_lastdim(self, x):
        x = _f32(x)
        K = x.shape[-1]
        out = np.empty(x.shape[:-1], np.float32)
        self.lib.ref_reduce_sum_lastdim(x.reshape(-1), out.reshape(-1), 1, x.size // K, K)
        return out

    def transpose(self, x, mode):
        x = np.ascontiguousarray(x)
        is_int = 1 if x.dtype == np.int32 else 0
        if mode == 0:
            M, N = x.shape
            dims, shape = (M, N, 0, 0), (N, M)
        elif mode == 1:
            n, c, h, w = x.shape
            dims, shape = (n, c, h, w), (n, h, w, c)
        else:
            n, h, w, c = x.shape
            dims, shape = (n, c, h, w), (n, c, h, w)
        out = np.empty(shape, x.dtype)
        self.lib.ref_transpose(x.ctypes.data_as(C.c_void_p), out.ctypes.data_as(C.c_void_p), mode, *dims, is_int)
        return out

    def layer_norm(self, x, gamma, beta, eps):
        x = _f32(x)
        y = np.empty_like(x)
        last = x.shape[-1]
        self.lib.ref_layer_norm(x.reshape(-1), _f32(gamma), _f32(beta), y.reshape(-1), x.size // last, last, eps)
        return y

    def rms_norm_rope_fused(self, x, weight, cos, sin, rot, eps):
        """The golden's own layout: x [B, S, H], interleaved RoPE."""
        x = _f32(x)
        B, S, H = x.shape
        out = np.empty_like(x)
        self.lib.ref_rms_norm_rope_fused(x.reshape(-1), _f32(weight), _f32(cos).reshape(-1), _f32(sin).reshape(-1),
                                         out.reshape(-1), B, S, H, rot, eps)
        return out

    def matmul_bias(self, A, B, bias=None):
        A, B = _f32(A), _f32(B)
        M, K = A.shape
        N = B.shape[1]
        out = np.empty((M, N), np.float32)
        b = None if bias is None else _f32(bias)
        self.lib.ref_matmul_bias(A, B, None if b is None else b.ctypes.data_as(C.c_void_p), out, M, K, N)
        return out

    def flash_attention_fwd(self, q, k, v, scale, causal, threads: int = 1):
        q, k, v = _f32(q), _f32(k), _f32(v)
        B, H, S_q, D = q.shape
        S_k, D_v = k.shape[2], v.shape[3]
        o = np.empty((B, H, S_q, D_v), np.float32)
        args = (q.reshape(-1), k.reshape(-1), v.reshape(-1), o.reshape(-1), B, H, S_q, S_k, D, D_v, scale,
                1 if causal else 0)
        if threads > 1:
            self.lib.ref_flash_attention_fwd_mt(*args, threads)
        else:
            self.lib.ref_flash_attention_fwd(*args)
        return o


def reference_available() -> bool:
    return REF_SO.exists()

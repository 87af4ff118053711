"""Python binding of the B200 operator ladder's C ABI (include/hc_runtime.h, include/hc_ops.h).

Loads lib/libhc_b200.so with ctypes and exposes
  * `lib`: the raw C entry points (argument/return types declared), for callers that hold plain
    pointers, exactly as a C or C++ host would call them;
  * tiling structs with the reference's field names (host/<op>_tiling.h of each op);
  * one function per ladder operator taking torch CUDA tensors, mirroring the reference runners
    (`run_<op>` in ops/<op>/runner of z-zijie/ascend-npu-harness): same argument meaning, outputs
    allocated when not given, and any non-zero status raised as HcError.

There is no fallback: if the library is missing or a launch fails, an exception is raised.
torch is only used for device memory and the current stream.
"""
from __future__ import annotations

import ctypes as C
import math
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "lib" / "libhc_b200.so"
TORCH_OPS_PATH = HERE / "lib" / "libhc_torch.so"

HC_OK, HC_ERR_INVALID, HC_ERR_CUDA, HC_ERR_UNSUPPORTED, HC_ERR_TIMEOUT, HC_ERR_NO_DEVICE, HC_ERR_INJECTED = range(7)
DT_F32, DT_F16, DT_BF16, DT_I32, DT_I8, DT_U8 = range(6)


class HcError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"hc status {status}: {msg}")
        self.status = status


# ---------------------------------------------------------------------------------------------
# tiling PODs (same layout as the reference's host/<op>_tiling.h)
# ---------------------------------------------------------------------------------------------
class ElementwiseAddTiling(C.Structure):
    _fields_ = [("totalLength", C.c_uint32), ("tileNum", C.c_uint32)]


class AxpyScalarAffineTiling(C.Structure):
    _fields_ = [("totalLength", C.c_uint32), ("tileNum", C.c_uint32)]


class BroadcastBinaryTiling(C.Structure):
    _fields_ = [("B", C.c_uint32), ("C", C.c_uint32), ("H", C.c_uint32), ("W", C.c_uint32),
                ("y_batch", C.c_uint32), ("tileNum", C.c_uint32)]


class ActivationGeluSiluTiling(C.Structure):
    _fields_ = [("totalLength", C.c_uint32), ("tileNum", C.c_uint32), ("actType", C.c_uint32)]


class ReduceSumLastdimTiling(C.Structure):
    _fields_ = [("totalRows", C.c_uint32), ("K", C.c_uint32), ("tileNum", C.c_uint32)]


class Transpose2d4dTiling(C.Structure):
    _fields_ = [("mode", C.c_uint32), ("M", C.c_uint32), ("N_dim", C.c_uint32), ("H", C.c_uint32),
                ("W", C.c_uint32), ("tileNum", C.c_uint32)]


class LayerNormTiling(C.Structure):
    _fields_ = [("rows", C.c_uint32), ("lastDim", C.c_uint32), ("tileNum", C.c_uint32), ("eps", C.c_float)]


class RmsNormRopeFusedTiling(C.Structure):
    _fields_ = [("B", C.c_uint32), ("S", C.c_uint32), ("H", C.c_uint32), ("rotaryDim", C.c_uint32),
                ("tileNum", C.c_uint32), ("eps", C.c_float)]


class MatmulBiasTiling(C.Structure):
    _fields_ = [("M", C.c_uint32), ("K", C.c_uint32), ("N", C.c_uint32), ("tileM", C.c_uint32),
                ("tileK", C.c_uint32), ("tileN", C.c_uint32)]


class FlashAttentionFwdFusedTiling(C.Structure):
    _fields_ = [("B", C.c_uint32), ("H", C.c_uint32), ("S_q", C.c_uint32), ("S_k", C.c_uint32),
                ("D", C.c_uint32), ("D_v", C.c_uint32), ("scale", C.c_float), ("maskType", C.c_uint32)]


_vp = C.c_void_p
_i = C.c_int
_u32 = C.c_uint32
_f = C.c_float
_sz = C.c_size_t
_P = C.POINTER

# name -> (restype, argtypes)
SIGNATURES = {
    "hc_init": (_i, []),
    "hc_device_count": (_i, [_P(_i)]),
    "hc_set_device": (_i, [_i]),
    "hc_get_device": (_i, [_P(_i)]),
    "hc_driver_version": (_i, [_P(_i)]),
    "hc_device_sm_count": (_i, [_P(_i)]),
    "hc_device_name": (_i, [C.c_char_p, _sz]),
    "hc_malloc": (_i, [_P(_vp), _sz]),
    "hc_free": (_i, [_vp]),
    "hc_malloc_host": (_i, [_P(_vp), _sz]),
    "hc_free_host": (_i, [_vp]),
    "hc_memcpy_h2d": (_i, [_vp, _vp, _sz, _vp]),
    "hc_memcpy_d2h": (_i, [_vp, _vp, _sz, _vp]),
    "hc_memcpy_d2d": (_i, [_vp, _vp, _sz, _vp]),
    "hc_memset": (_i, [_vp, _i, _sz, _vp]),
    "hc_stream_create": (_i, [_P(_vp)]),
    "hc_stream_destroy": (_i, [_vp]),
    "hc_stream_sync": (_i, [_vp]),
    "hc_device_sync": (_i, []),
    "hc_event_create": (_i, [_P(_vp)]),
    "hc_event_destroy": (_i, [_vp]),
    "hc_event_record": (_i, [_vp, _vp]),
    "hc_event_sync": (_i, [_vp]),
    "hc_event_elapsed_ms": (_i, [_P(_f), _vp, _vp]),
    "hc_check_device_error": (_i, []),
    "hc_last_error_string": (C.c_char_p, []),
    "hc_last_error": (_i, []),
    "hc_set_fault": (_i, [C.c_char_p]),
    "hc_selftest_bounded_wait": (_i, [_u32]),
    "hc_elementwise_add_launch": (_i, [_vp, _vp, _vp, _P(ElementwiseAddTiling), _i, _vp]),
    "hc_axpy_scalar_affine_launch": (_i, [_vp, _vp, _P(AxpyScalarAffineTiling), _f, _f, _i, _vp]),
    "hc_broadcast_binary_launch": (_i, [_vp, _vp, _vp, _vp, _P(BroadcastBinaryTiling), _i, _vp]),
    "hc_activation_gelu_silu_launch": (_i, [_vp, _vp, _P(ActivationGeluSiluTiling), _i, _vp]),
    "hc_reduce_sum_lastdim_launch": (_i, [_vp, _vp, _P(ReduceSumLastdimTiling), _i, _vp]),
    "hc_transpose_2d_4d_launch": (_i, [_vp, _vp, _P(Transpose2d4dTiling), _i, _vp]),
    "hc_layer_norm_launch": (_i, [_vp, _vp, _vp, _vp, _P(LayerNormTiling), _i, _vp]),
    "hc_rms_norm_rope_fused_launch": (_i, [_vp, _vp, _vp, _vp, _vp, _P(RmsNormRopeFusedTiling), _u32, _u32, _i,
                                           _vp]),
    "hc_matmul_bias_launch": (_i, [_vp, _vp, _vp, _vp, _P(MatmulBiasTiling), _i, _vp]),
    "hc_flash_attention_fwd_fused_launch": (_i, [_vp, _vp, _vp, _vp, _vp, _P(FlashAttentionFwdFusedTiling), _i,
                                                 _vp]),
    "hc_flash_attention_fwd_fused_gqa_launch": (_i, [_vp, _vp, _vp, _vp, _vp, _P(FlashAttentionFwdFusedTiling), _u32, _i,
                                                 _vp]),
    "hc_flash_attention_fwd_fused_host_workspace_size": (_i, [_P(FlashAttentionFwdFusedTiling), _i, _P(_sz)]),
    "hc_flash_attention_fwd_fused_host": (_i, [_vp, _vp, _vp, _vp, _vp, _P(FlashAttentionFwdFusedTiling), _i, _vp,
                                               _sz, _vp]),
    "hc_flash_attention_fwd_fused_host_noalloc": (_i, [_vp, _vp, _vp, _vp, _vp, _P(FlashAttentionFwdFusedTiling),
                                                       _i, _vp]),
    "hc_flash_attention_fwd_fused_host_noalloc_limit": (_sz, []),
    "hc_flash_attention_bwd_launch": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                           _P(FlashAttentionFwdFusedTiling), _i, _vp]),
    "hc_flash_attention_bwd_last_path": (_i, []),
    "hc_flash_attention_last_path": (_i, []),
    "hc_matmul_bias_last_path": (_i, []),
}

_lib = None


def load(path: Path | str | None = None) -> C.CDLL:
    """Loads the library (once) and declares every entry point's signature."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise FileNotFoundError(f"{p} is missing: run `python {HERE / 'build.py'}` (or __graft_entry__.build())")
    lib = C.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def check(status: int) -> None:
    if status != HC_OK:
        raise HcError(status, load().hc_last_error_string().decode(errors="replace"))


# ---------------------------------------------------------------------------------------------
# torch-tensor level API
# ---------------------------------------------------------------------------------------------
def _torch():
    import torch
    return torch


def dtype_code(t) -> int:
    torch = _torch()
    m = {torch.float32: DT_F32, torch.float16: DT_F16, torch.bfloat16: DT_BF16, torch.int32: DT_I32,
         torch.int8: DT_I8, torch.uint8: DT_U8}
    if t.dtype not in m:
        raise HcError(HC_ERR_UNSUPPORTED, f"dtype {t.dtype}")
    return m[t.dtype]


def _ptr(t):
    if t is None:
        return None
    if not t.is_cuda:
        raise HcError(HC_ERR_INVALID, "expected a CUDA tensor")
    if not t.is_contiguous():
        raise HcError(HC_ERR_INVALID, "expected a contiguous tensor")
    return C.c_void_p(t.data_ptr())


def _stream(stream):
    if stream is not None:
        return C.c_void_p(stream)
    torch = _torch()
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def elementwise_add(x, y, z=None, stream=None):
    """z = x + y (ops/elementwise_add/runner/elementwise_add_runner.hpp: run(x, y, z, shape))."""
    if z is None:
        z = _torch().empty_like(x)
    t = ElementwiseAddTiling(x.numel(), 0)
    check(load().hc_elementwise_add_launch(_ptr(x), _ptr(y), _ptr(z), C.byref(t), dtype_code(x), _stream(stream)))
    return z


def axpy_scalar_affine(x, alpha: float, beta: float, y=None, stream=None):
    if y is None:
        y = _torch().empty_like(x)
    t = AxpyScalarAffineTiling(x.numel(), 0)
    check(load().hc_axpy_scalar_affine_launch(_ptr(x), _ptr(y), C.byref(t), alpha, beta, dtype_code(x),
                                              _stream(stream)))
    return y


def broadcast_binary(x, y, bias, y_batch: int, z=None, stream=None):
    """z[b,c,h,w] = x * y[yb,c] + bias[c] with x NCHW."""
    if z is None:
        z = _torch().empty_like(x)
    B, Cc, H, W = x.shape
    t = BroadcastBinaryTiling(B, Cc, H, W, y_batch, 0)
    check(load().hc_broadcast_binary_launch(_ptr(x), _ptr(y), _ptr(bias), _ptr(z), C.byref(t), dtype_code(x),
                                            _stream(stream)))
    return z


def activation_gelu_silu(x, act: str, y=None, stream=None):
    if act not in ("gelu", "silu"):
        raise HcError(HC_ERR_INVALID, f"unknown activation {act!r}")
    if y is None:
        y = _torch().empty_like(x)
    t = ActivationGeluSiluTiling(x.numel(), 0, 0 if act == "gelu" else 1)
    check(load().hc_activation_gelu_silu_launch(_ptr(x), _ptr(y), C.byref(t), dtype_code(x), _stream(stream)))
    return y


def reduce_sum_lastdim(x, out=None, stream=None):
    """out[..., m] = sum_k x[..., m, k] (fp32 output)."""
    torch = _torch()
    K = x.shape[-1]
    rows = x.numel() // K if K else 0
    if out is None:
        out = torch.empty(x.shape[:-1], dtype=torch.float32, device=x.device)
    t = ReduceSumLastdimTiling(rows, K, 0)
    check(load().hc_reduce_sum_lastdim_launch(_ptr(x), _ptr(out), C.byref(t), dtype_code(x), _stream(stream)))
    return out


def transpose_2d_4d(x, mode: int, out=None, stream=None):
    """mode 0: [M,N]->[N,M]; 1: NCHW->NHWC; 2: NHWC->NCHW (x given in its input layout)."""
    torch = _torch()
    if mode == 0:
        M, N = x.shape
        t = Transpose2d4dTiling(0, M, N, 0, 0, 0)
        shape = (N, M)
    elif mode == 1:
        n, c, h, w = x.shape
        t = Transpose2d4dTiling(1, n, c, h, w, 0)
        shape = (n, h, w, c)
    elif mode == 2:
        n, h, w, c = x.shape
        t = Transpose2d4dTiling(2, n, c, h, w, 0)
        shape = (n, c, h, w)
    else:
        raise HcError(HC_ERR_INVALID, f"mode {mode}")
    if out is None:
        out = torch.empty(shape, dtype=x.dtype, device=x.device)
    check(load().hc_transpose_2d_4d_launch(_ptr(x), _ptr(out), C.byref(t), dtype_code(x), _stream(stream)))
    return out


def layer_norm(x, gamma, beta, eps: float, y=None, stream=None):
    if y is None:
        y = _torch().empty_like(x)
    last = x.shape[-1]
    t = LayerNormTiling(x.numel() // last, last, 0, eps)
    check(load().hc_layer_norm_launch(_ptr(x), _ptr(gamma), _ptr(beta), _ptr(y), C.byref(t), dtype_code(x),
                                      _stream(stream)))
    return y


def rms_norm_rope_fused(x, weight, cos, sin, rotary_dim: int, eps: float, heads: int = 1, rope_style: int = 0,
                        out=None, stream=None):
    """x [B, S, H] (heads=1) or [B, S, heads, H]; cos/sin [S, rotary_dim/2] fp32."""
    if out is None:
        out = _torch().empty_like(x)
    B, S = x.shape[0], x.shape[1]
    H = x.shape[-1]
    t = RmsNormRopeFusedTiling(B, S, H, rotary_dim, 0, eps)
    check(load().hc_rms_norm_rope_fused_launch(_ptr(x), _ptr(weight), _ptr(cos), _ptr(sin), _ptr(out), C.byref(t),
                                               heads, rope_style, dtype_code(x), _stream(stream)))
    return out


def matmul_bias(A, B, bias=None, out=None, stream=None):
    torch = _torch()
    M, K = A.shape
    N = B.shape[1]
    if out is None:
        out = torch.empty((M, N), dtype=A.dtype, device=A.device)
    t = MatmulBiasTiling(M, K, N, 0, 0, 0)
    check(load().hc_matmul_bias_launch(_ptr(A), _ptr(B), _ptr(bias), _ptr(out), C.byref(t), dtype_code(A),
                                       _stream(stream)))
    return out


def flash_attention_fwd(q, k, v, causal: bool, scale: float | None = None, with_lse: bool = True, out=None,
                        lse=None, stream=None):
    """O = softmax(Q K^T * scale [causal]) V for [B, H, S, D] tensors; returns (O, lse or None).
    K and V may have fewer heads than Q (a divisor of H): grouped-query attention."""
    torch = _torch()
    B, H, S_q, D = q.shape
    S_k, D_v = k.shape[2], v.shape[3]
    kv_heads = k.shape[1]  # < H: grouped-query attention (query head h reads K/V head h // (H // kv_heads))
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty((B, H, S_q, D_v), dtype=q.dtype, device=q.device)
    if with_lse and lse is None:
        lse = torch.empty((B, H, S_q), dtype=torch.float32, device=q.device)
    t = FlashAttentionFwdFusedTiling(B, H, S_q, S_k, D, D_v, scale, 1 if causal else 0)
    if kv_heads == H:
        check(load().hc_flash_attention_fwd_fused_launch(_ptr(q), _ptr(k), _ptr(v), _ptr(out),
                                                         _ptr(lse) if with_lse else None, C.byref(t), dtype_code(q),
                                                         _stream(stream)))
    else:
        check(load().hc_flash_attention_fwd_fused_gqa_launch(_ptr(q), _ptr(k), _ptr(v), _ptr(out),
                                                             _ptr(lse) if with_lse else None, C.byref(t), kv_heads,
                                                             dtype_code(q), _stream(stream)))
    return out, (lse if with_lse else None)


def flash_attention_bwd(q, k, v, o, lse, dout, causal: bool, scale: float | None = None, out=None, stream=None):
    """Gradients of O = softmax(Q K^T * scale [causal]) V for [B, H, S, D] tensors, from the forward's
    o and lse and the output gradient dout; returns (dq, dk, dv, delta) with delta = rowsum(dout * o)
    fp32 [B, H, S_q].  K and V have H heads (no grouped-query form).  `out` may give the four
    output tensors (allocated otherwise)."""
    torch = _torch()
    B, H, S_q, D = q.shape
    S_k, D_v = k.shape[2], v.shape[3]
    if k.shape[1] != H or v.shape[1] != H:
        raise HcError(HC_ERR_UNSUPPORTED, "flash_attention_bwd: K/V must have the query head count")
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if out is None:
        out = (torch.empty_like(q), torch.empty_like(k), torch.empty_like(v),
               torch.empty((B, H, S_q), dtype=torch.float32, device=q.device))
    dq, dk, dv, delta = out
    t = FlashAttentionFwdFusedTiling(B, H, S_q, S_k, D, D_v, scale, 1 if causal else 0)
    check(load().hc_flash_attention_bwd_launch(_ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(dout), _ptr(lse), _ptr(dq),
                                               _ptr(dk), _ptr(dv), _ptr(delta), C.byref(t), dtype_code(q),
                                               _stream(stream)))
    return dq, dk, dv, delta


_torch_ops_loaded = False


def load_torch_ops():
    """Registers the `hc` torch custom ops (lib/libhc_torch.so, csrc/torch_ops.cpp) and returns torch.ops.hc.
    The ops call the same C ABI as this module, on the current CUDA stream; they raise on CPU tensors.
    hc::flash_attention_fwd_fused gets an autograd formula: hc::flash_attention_bwd (q, k, v get
    gradients; the lse output is not differentiable)."""
    global _torch_ops_loaded
    torch = _torch()
    if not _torch_ops_loaded:
        if not TORCH_OPS_PATH.exists():
            raise HcError(HC_ERR_INVALID, f"{TORCH_OPS_PATH} is missing; run ascend-npu-harness_b200/build.py")
        torch.ops.load_library(str(TORCH_OPS_PATH))
        torch.library.register_autograd("hc::flash_attention_fwd_fused", _fa_backward, setup_context=_fa_setup)
        _torch_ops_loaded = True
    return torch.ops.hc


def _fa_setup(ctx, inputs, output):
    q, k, v, scale, mask_type = inputs
    o, lse = output
    ctx.save_for_backward(q, k, v, o, lse)
    ctx.scale, ctx.mask_type = scale, mask_type
    ctx.mark_non_differentiable(lse)


def _fa_backward(ctx, grad_o, grad_lse):
    """Gradients of hc::flash_attention_fwd_fused through hc::flash_attention_bwd.  Grouped-query K/V
    (fewer heads) are expanded to the query heads for the kernel and their gradients summed back
    over each group (query head h reads K/V head h // (H / kv_heads), as in the forward)."""
    torch = _torch()
    q, k, v, o, lse = ctx.saved_tensors
    H, kv = q.shape[1], k.shape[1]
    group = H // kv
    ke, ve = (k, v) if group == 1 else (k.repeat_interleave(group, 1), v.repeat_interleave(group, 1))
    dq, dk, dv, _ = torch.ops.hc.flash_attention_bwd(q, ke.contiguous(), ve.contiguous(), o, lse,
                                                      grad_o.contiguous(), ctx.scale, ctx.mask_type)
    if group > 1:
        dk = dk.view(k.shape[0], kv, group, *k.shape[2:]).sum(2)
        dv = dv.view(v.shape[0], kv, group, *v.shape[2:]).sum(2)
    return dq, dk, dv, None, None


def check_device_error() -> None:
    check(load().hc_check_device_error())

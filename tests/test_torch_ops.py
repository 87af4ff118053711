"""The `hc` torch custom-op library (csrc/torch_ops.cpp): registration and shape inference on CPU,
results on the GPU identical to the ctypes binding (both call the same C ABI), and autograd through
hc::flash_attention_fwd_fused (the backward kernels) against an fp32 torch restatement."""
from __future__ import annotations

import math
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "ascend-npu-harness_b200"))

import hc  # noqa: E402

OPS = ("elementwise_add", "axpy_scalar_affine", "broadcast_binary", "activation_gelu_silu", "reduce_sum_lastdim",
       "transpose_2d_4d", "layer_norm", "rms_norm_rope_fused", "matmul_bias", "flash_attention_fwd_fused",
       "flash_attention_bwd")


@pytest.fixture(scope="module")
def ops():
    import torch  # noqa: F401

    if not hc.TORCH_OPS_PATH.exists():
        sys.path.insert(0, str(ROOT / "ascend-npu-harness_b200"))
        import build

        build.build()
        build.build_torch()
    return hc.load_torch_ops()


def test_all_ops_registered(ops):
    import torch

    for name in OPS:
        op = getattr(ops, name)
        assert op.default._schema.name == f"hc::{name}"
    s = str(torch.ops.hc.flash_attention_fwd_fused.default._schema)
    assert "(Tensor, Tensor)" in s and "int mask_type" in s


def test_meta_shapes(ops):
    import torch

    m = dict(device="meta")
    x = torch.empty(4, 6, 8, 16, dtype=torch.bfloat16, **m)
    assert ops.elementwise_add(x, x).shape == x.shape
    assert ops.axpy_scalar_affine(x, 2.0, 1.0).shape == x.shape
    assert ops.broadcast_binary(x, torch.empty(6, dtype=torch.bfloat16, **m), torch.empty(6, dtype=torch.bfloat16, **m),
                                1).shape == x.shape
    assert ops.activation_gelu_silu(x, 0).dtype == torch.bfloat16
    r = ops.reduce_sum_lastdim(x)
    assert r.shape == (4, 6, 8) and r.dtype == torch.float32
    assert ops.transpose_2d_4d(x, 1).shape == (4, 8, 16, 6)
    assert ops.transpose_2d_4d(x, 2).shape == (4, 16, 6, 8)
    assert ops.transpose_2d_4d(torch.empty(3, 5, **m), 0).shape == (5, 3)
    f = torch.empty(16, dtype=torch.float32, **m)
    assert ops.layer_norm(x, f, f, 1e-5).shape == x.shape
    assert ops.rms_norm_rope_fused(x, f, f, f, 16, 1e-6, 8, 1).shape == x.shape
    a = torch.empty(32, 64, dtype=torch.bfloat16, **m)
    b = torch.empty(64, 48, dtype=torch.bfloat16, **m)
    assert ops.matmul_bias(a, b, None).shape == (32, 48)
    q = torch.empty(2, 3, 100, 128, dtype=torch.bfloat16, **m)
    kv = torch.empty(2, 3, 70, 128, dtype=torch.bfloat16, **m)
    o, lse = ops.flash_attention_fwd_fused(q, kv, kv, 0.088, 1)
    assert o.shape == (2, 3, 100, 128) and lse.shape == (2, 3, 100) and lse.dtype == torch.float32
    q6 = torch.empty(2, 6, 100, 128, dtype=torch.bfloat16, **m)  # grouped-query: 3 K/V heads for 6 query heads
    assert ops.flash_attention_fwd_fused(q6, kv, kv, 0.088, 1)[0].shape == (2, 6, 100, 128)
    with pytest.raises(RuntimeError, match="must divide"):
        ops.flash_attention_fwd_fused(torch.empty(2, 4, 100, 128, dtype=torch.bfloat16, **m), kv, kv, 0.088, 1)
    dq, dk, dv, delta = ops.flash_attention_bwd(q, kv, kv, o, lse, o, 0.088, 1)
    assert dq.shape == q.shape and dk.shape == kv.shape and dv.shape == kv.shape
    assert delta.shape == (2, 3, 100) and delta.dtype == torch.float32


def test_cpu_tensors_have_no_kernel(ops):
    """No CPU fallback: a CPU tensor is a dispatch error, not a silently computed result."""
    import torch

    x = torch.ones(8)
    with pytest.raises(NotImplementedError):
        ops.elementwise_add(x, x)


@pytest.mark.gpu
def test_ops_match_ctypes_binding(ops):
    import torch

    g = torch.Generator(device="cuda").manual_seed(7)
    rnd = lambda *s, dt=torch.bfloat16: torch.randn(*s, generator=g, device="cuda").to(dt)  # noqa: E731
    x = rnd(4, 16, 32, 32)
    y = rnd(4, 16, 32, 32)
    eq = lambda a, b: torch.equal(a.view(torch.int16) if a.dtype == torch.bfloat16 else a,  # noqa: E731
                                  b.view(torch.int16) if b.dtype == torch.bfloat16 else b)
    assert eq(ops.elementwise_add(x, y), hc.elementwise_add(x, y))
    assert eq(ops.axpy_scalar_affine(x, 0.5, -1.0), hc.axpy_scalar_affine(x, 0.5, -1.0))
    yv, bias = rnd(16), rnd(16)
    assert eq(ops.broadcast_binary(x, yv, bias, 1), hc.broadcast_binary(x, yv, bias, 1))
    assert eq(ops.activation_gelu_silu(x, 0), hc.activation_gelu_silu(x, "gelu"))
    assert eq(ops.activation_gelu_silu(x, 1), hc.activation_gelu_silu(x, "silu"))
    assert eq(ops.reduce_sum_lastdim(x), hc.reduce_sum_lastdim(x))
    for mode in (1, 2):
        assert eq(ops.transpose_2d_4d(x, mode), hc.transpose_2d_4d(x, mode))
    x2 = x.reshape(64, 1024)
    assert eq(ops.transpose_2d_4d(x2, 0), hc.transpose_2d_4d(x2, 0))
    gamma = torch.rand(1024, generator=g, device="cuda") + 0.5
    beta = torch.rand(1024, generator=g, device="cuda") - 0.5
    assert eq(ops.layer_norm(x2, gamma, beta, 1e-5), hc.layer_norm(x2, gamma, beta, 1e-5))
    xr = rnd(2, 64, 4, 128)
    w = torch.rand(128, generator=g, device="cuda") + 0.5
    pos = torch.arange(64, device="cuda", dtype=torch.float32)[:, None]
    theta = pos / (10000.0 ** (torch.arange(64, device="cuda", dtype=torch.float32) * 2 / 128))
    cos, sin = torch.cos(theta).contiguous(), torch.sin(theta).contiguous()
    assert eq(ops.rms_norm_rope_fused(xr, w, cos, sin, 128, 1e-6, 4, 1),
              hc.rms_norm_rope_fused(xr, w, cos, sin, 128, 1e-6, heads=4, rope_style=1))
    a, b, bb = rnd(256, 512), rnd(512, 384), rnd(384)
    assert eq(ops.matmul_bias(a, b, bb), hc.matmul_bias(a, b, bb))
    assert eq(ops.matmul_bias(a, b), hc.matmul_bias(a, b))
    q, k, v = rnd(1, 4, 300, 128), rnd(1, 4, 300, 128), rnd(1, 4, 300, 128)
    o, lse = ops.flash_attention_fwd_fused(q, k, v, 1 / math.sqrt(128), 1)
    o2, lse2 = hc.flash_attention_fwd(q, k, v, True)
    assert eq(o, o2) and torch.equal(lse, lse2)
    kg, vg = rnd(1, 2, 300, 128), rnd(1, 2, 300, 128)  # grouped-query: 2 K/V heads for 4 query heads
    o, lse = ops.flash_attention_fwd_fused(q, kg, vg, 1 / math.sqrt(128), 1)
    o2, lse2 = hc.flash_attention_fwd(q, kg, vg, True)
    assert eq(o, o2) and torch.equal(lse, lse2)
    dout = rnd(1, 4, 300, 128)
    o, lse = hc.flash_attention_fwd(q, k, v, True)
    g1 = ops.flash_attention_bwd(q, k, v, o, lse, dout, 1 / math.sqrt(128), 1)
    g2 = hc.flash_attention_bwd(q, k, v, o, lse, dout, True)
    assert all(eq(a, b) for a, b in zip(g1[:3], g2[:3])) and torch.equal(g1[3], g2[3])
    torch.cuda.synchronize()
    hc.check_device_error()


def _reference_grads(q, k, v, dout, scale, causal):
    """fp32 gradients of softmax(q k^T * scale [causal]) v by torch autograd (no TF32); K/V heads
    repeated for grouped-query inputs."""
    import torch

    group = q.shape[1] // k.shape[1]
    qf, kf, vf = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    s = (qf @ kf.repeat_interleave(group, 1).transpose(-1, -2)) * scale
    if causal:
        s = s.masked_fill(torch.ones(s.shape[-2:], dtype=torch.bool, device=s.device).triu(1), float("-inf"))
    (torch.softmax(s, -1) @ vf.repeat_interleave(group, 1)).backward(dout.float())
    return qf.grad, kf.grad, vf.grad


@pytest.mark.gpu
@pytest.mark.parametrize("causal", [True, False], ids=["causal", "none"])
@pytest.mark.parametrize("kv_heads", [4, 2], ids=["mha", "gqa"])
def test_flash_attention_autograd(ops, causal, kv_heads):
    """loss.backward() through hc::flash_attention_fwd_fused runs the tcgen05 backward kernels; the
    gradients match fp32 autograd of the same attention (normwise 1e-2, the bf16 backward bound)."""
    import torch

    g = torch.Generator(device="cuda").manual_seed(3)
    rnd = lambda *s: torch.randn(*s, generator=g, device="cuda").to(torch.bfloat16)  # noqa: E731
    q = rnd(2, 4, 384, 128).requires_grad_(True)
    k, v = (rnd(2, kv_heads, 384, 128).requires_grad_(True) for _ in range(2))
    dout = rnd(2, 4, 384, 128)
    scale = 1 / math.sqrt(128)
    o, _ = ops.flash_attention_fwd_fused(q, k, v, scale, 1 if causal else 0)
    o.backward(dout)
    assert hc.load().hc_flash_attention_bwd_last_path() == 1
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        ref = _reference_grads(q, k, v, dout, scale, causal)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    for name, got, exp in zip(("dq", "dk", "dv"), (q.grad, k.grad, v.grad), ref):
        assert got.shape == exp.shape and got.dtype == torch.bfloat16
        err = float((got.float() - exp).norm() / exp.norm())
        assert err <= 1e-2, f"{name}: normwise {err:.3g}"
    hc.check_device_error()


@pytest.mark.gpu
def test_ops_run_on_current_stream_and_report_errors(ops):
    import torch

    s = torch.cuda.Stream()
    x = torch.randn(1 << 20, device="cuda").to(torch.float16)
    with torch.cuda.stream(s):
        z = ops.elementwise_add(x, x)
    s.synchronize()
    assert torch.equal(z, x + x)
    with pytest.raises(RuntimeError, match="hc::activation_gelu_silu"):
        ops.activation_gelu_silu(x, 5)  # actType 5 is rejected by the C ABI with its message
    assert np.isfinite(z.float().cpu().numpy()).all()

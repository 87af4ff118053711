"""GPU parity of the flash-attention backward (hc_flash_attention_bwd_launch) against the oracle.

The reference ladder has no backward, so there is no golden from it: the oracle
(oracle_flash_attention_bwd, fp64, pinned against torch float64 autograd in test_oracle_pins.py)
is the exact gradient of the same forward.  The device backward consumes the device forward's O
and lse, as a training step does.
  * tensor-core path (bf16/fp16, D = D_v = 128, and 64 on a subset): single and multiple 128-row blocks, ragged
    S_q and S_k, S_q != S_k both ways with causal masking (key blocks that no query sees get zero
    gradients), B*H > 1;
  * SIMT path: fp32, and 16-bit with D = 96 or D != D_v;
  * delta against rowsum(dO * O) of the same device tensors;
  * the benchmarked shape B=16 H=32 S=8192 D=128 (causal and non-causal, and D=64 causal): sampled heads against a
    torch fp32 restatement of the gradients on the device, every head through the identities
    sum_k dV[k] = sum_r dO[r] and sum_k dK[k] = 0 (rows of P sum to 1);
  * argument errors (null pointer, mask type, grouped-query K/V) before any device work.
Tolerances are normwise (||got - exact|| / ||exact||) per gradient, with the max-abs error
bounded relative to the largest exact magnitude."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from gpu_util import dev, host, quantize

pytestmark = pytest.mark.gpu

# normwise relative error per gradient, and max-abs error / max |exact|
BWD_TOL = {"bf16": (1e-2, 3e-2), "f16": (3e-3, 1e-2), "f32": (5e-5, 2e-4)}


def _normwise(exact, got):
    e = np.asarray(exact, np.float64)
    g = np.asarray(got, np.float64)
    n = np.linalg.norm(e)
    return float(np.linalg.norm(g - e) / n) if n > 0 else float(np.linalg.norm(g)), float(
        np.abs(g - e).max() / max(np.abs(e).max(), 1e-30))


def _check(name, exact, got, kind):
    assert np.isfinite(got).all(), f"{name}: non-finite values"
    if np.abs(exact).max() < 1e-6:  # an identically zero gradient (one visible key: dS = 0)
        assert np.abs(got).max() <= 1e-5, f"{name}: expected zeros, got max |g| {np.abs(got).max():.3g}"
        return 0.0
    nw, ma = _normwise(exact, got)
    tn, tm = BWD_TOL[kind]
    assert nw <= tn and ma <= tm, f"{name} ({kind}): normwise {nw:.3g} (<= {tn}), max-abs/max {ma:.3g} (<= {tm})"
    return nw


def _run(hc_lib, oracle, B, H, S_q, S_k, D, Dv, causal, kind, seed=7):
    import torch

    q = oracle.normal(B * H * S_q * D, seed).reshape(B, H, S_q, D)
    k = oracle.normal(B * H * S_k * D, seed + 1).reshape(B, H, S_k, D)
    v = oracle.normal(B * H * S_k * Dv, seed + 2).reshape(B, H, S_k, Dv)
    do = oracle.normal(B * H * S_q * Dv, seed + 3).reshape(B, H, S_q, Dv)
    qd, kd, vd, dod = (dev(a, kind, oracle) for a in (q, k, v, do))
    scale = 1.0 / np.sqrt(D)
    o, lse = hc_lib.flash_attention_fwd(qd, kd, vd, causal, scale=scale)
    dq, dk, dv, delta = hc_lib.flash_attention_bwd(qd, kd, vd, o, lse, dod, causal, scale=scale)
    torch.cuda.synchronize()
    hc_lib.check_device_error()
    path = hc_lib.load().hc_flash_attention_bwd_last_path()
    qq, kq, vq, doq = (quantize(a, kind, oracle) for a in (q, k, v, do))
    ref = oracle.flash_attention_bwd(qq, kq, vq, doq, scale, causal)
    got = tuple(host(t, oracle) for t in (dq, dk, dv))
    # delta = rowsum(dO * O) over the device's own O
    o_h = host(o, oracle).astype(np.float64)
    d_ref = (doq.astype(np.float64) * o_h).sum(-1)
    d_got = delta.cpu().numpy()
    assert np.abs(d_got - d_ref).max() <= 1e-4 * max(1.0, np.abs(d_ref).max()), "delta"
    return ref, got, path


TC_CASES = [
    (1, 1, 128, 128, True), (1, 1, 128, 128, False), (1, 2, 256, 256, True), (2, 2, 384, 384, False),
    (1, 2, 200, 328, True), (1, 2, 200, 328, False), (1, 1, 384, 130, True), (1, 1, 130, 384, True),
    (1, 1, 130, 384, False), (1, 3, 1, 1, True), (1, 1, 77, 513, False), (3, 1, 640, 640, True),
]


@pytest.mark.parametrize("kind", ["bf16", "f16"])
@pytest.mark.parametrize("case", TC_CASES, ids=lambda c: "B{}_H{}_Sq{}_Sk{}_{}".format(*c[:4], "causal" if c[4] else "none"))
def test_tensor_core_path(cuda, hc_lib, oracle, case, kind):
    B, H, S_q, S_k, causal = case
    ref, got, path = _run(hc_lib, oracle, B, H, S_q, S_k, 128, 128, causal, kind)
    assert path == 1, "D = D_v = 128 in 16-bit must take the tcgen05 backward"
    for name, e, g in zip(("dq", "dk", "dv"), ref, got):
        _check(f"{name} {case}", e, g, kind)


TC64_CASES = [(1, 2, 128, 128, True), (1, 2, 200, 328, True), (2, 1, 384, 130, False), (1, 1, 130, 384, True),
              (1, 3, 640, 640, True)]


@pytest.mark.parametrize("kind", ["bf16", "f16"])
@pytest.mark.parametrize("case", TC64_CASES, ids=lambda c: "B{}_H{}_Sq{}_Sk{}_{}".format(*c[:4], "causal" if c[4] else "none"))
def test_tensor_core_path_d64(cuda, hc_lib, oracle, case, kind):
    B, H, S_q, S_k, causal = case
    ref, got, path = _run(hc_lib, oracle, B, H, S_q, S_k, 64, 64, causal, kind)
    assert path == 1, "D = D_v = 64 in 16-bit must take the tcgen05 backward"
    for name, e, g in zip(("dq", "dk", "dv"), ref, got):
        _check(f"{name} {case}", e, g, kind)


def test_unseen_key_blocks_are_zero(cuda, hc_lib, oracle):
    """Causal with S_k > S_q: keys past the last query are seen by no row; their dK, dV are 0."""
    ref, got, path = _run(hc_lib, oracle, 1, 2, 130, 700, 128, 128, True, "bf16")
    assert path == 1
    dk, dv = got[1], got[2]
    assert not dk[:, :, 130:].any() and not dv[:, :, 130:].any()
    for name, e, g in zip(("dq", "dk", "dv"), ref, got):
        _check(name, e, g, "bf16")


SIMT_CASES = [
    ("f32", 1, 2, 100, 70, 64, 64, True), ("f32", 2, 1, 33, 129, 128, 128, False), ("f32", 1, 1, 50, 60, 32, 48, True),
    ("bf16", 1, 2, 100, 70, 96, 96, True), ("bf16", 1, 1, 90, 90, 128, 64, False), ("f16", 1, 1, 65, 40, 80, 80, True),
    ("f32", 1, 1, 17, 23, 256, 256, False),
]


@pytest.mark.parametrize("case", SIMT_CASES, ids=lambda c: "{}_B{}_H{}_Sq{}_Sk{}_D{}_Dv{}_{}".format(*c[:7], "causal" if c[7] else "none"))
def test_simt_path(cuda, hc_lib, oracle, case):
    kind, B, H, S_q, S_k, D, Dv, causal = case
    ref, got, path = _run(hc_lib, oracle, B, H, S_q, S_k, D, Dv, causal, kind)
    assert path == 2
    for name, e, g in zip(("dq", "dk", "dv"), ref, got):
        _check(f"{name} {case}", e, g, kind)


def _torch_grads(q, k, v, do, scale, causal):
    """fp32 restatement on the device of the gradients of one head (no TF32)."""
    import torch

    q, k, v, do = (t.float() for t in (q, k, v, do))
    s = (q @ k.T) * scale
    if causal:
        s = s.masked_fill(torch.ones_like(s, dtype=torch.bool).triu(1), float("-inf"))
    p = torch.softmax(s, dim=-1)
    dp = do @ v.T
    ds = p * (dp - (p * dp).sum(-1, keepdim=True))
    return (ds @ k) * scale, (ds.T @ q) * scale, p.T @ do


@pytest.mark.parametrize("causal,D", [(True, 128), (False, 128), (True, 64)], ids=["causal", "none", "causal_d64"])
def test_benchmarked_shape(cuda, hc_lib, causal, D):
    """B=16 H=32 S=8192 D=128 bf16 (and D=64): sampled heads against fp32 gradients, all heads by identities."""
    import torch

    B, H, S = 16, 32, 8192
    scale = 1.0 / np.sqrt(D)
    g = torch.Generator(device="cuda").manual_seed(11)
    q, k, v, do = (torch.randn((B, H, S, D), generator=g, device="cuda", dtype=torch.bfloat16) for _ in range(4))
    o, lse = hc_lib.flash_attention_fwd(q, k, v, causal, scale=scale)
    dq, dk, dv, delta = hc_lib.flash_attention_bwd(q, k, v, o, lse, do, causal, scale=scale)
    torch.cuda.synchronize()
    hc_lib.check_device_error()
    assert hc_lib.load().hc_flash_attention_bwd_last_path() == 1
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        for b, h in ((0, 0), (7, 19), (15, 31)):
            ref = _torch_grads(q[b, h], k[b, h], v[b, h], do[b, h], scale, causal)
            for name, e, got in zip(("dq", "dk", "dv"), ref, (dq[b, h], dk[b, h], dv[b, h])):
                _check(f"{name} head ({b},{h})", e.cpu().numpy(), got.float().cpu().numpy(), "bf16")
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    # every head: sum_k dV = sum_r dO and sum_k dK = 0
    sdv = dv.float().sum(2)
    sdo = do.float().sum(2)
    err_v = ((sdv - sdo).norm(dim=-1) / sdo.norm(dim=-1)).max().item()
    assert err_v <= 1e-2, f"sum_k dV vs sum_r dO: {err_v:.3g}"
    sdk = dk.float().sum(2).norm(dim=-1)
    err_k = (sdk / dk.float().norm(dim=(2, 3))).max().item()
    assert err_k <= 2e-2, f"sum_k dK: {err_k:.3g} of ||dK||"
    assert torch.isfinite(delta).all()


def test_argument_errors(cuda, hc_lib):
    import torch

    lib = hc_lib.load()
    x = torch.zeros((1, 2, 128, 128), device="cuda", dtype=torch.bfloat16)
    lse = torch.zeros((1, 2, 128), device="cuda", dtype=torch.float32)
    t = hc_lib.FlashAttentionFwdFusedTiling(1, 2, 128, 128, 128, 128, 0.1, 1)
    p = ctypes.c_void_p(x.data_ptr())
    lp = ctypes.c_void_p(lse.data_ptr())
    args = [p, p, p, p, p, lp, p, p, p, lp]
    assert lib.hc_flash_attention_bwd_launch(*args[:6], None, *args[7:], ctypes.byref(t), hc_lib.DT_BF16,
                                             None) == hc_lib.HC_ERR_INVALID
    t.maskType = 3
    assert lib.hc_flash_attention_bwd_launch(*args, ctypes.byref(t), hc_lib.DT_BF16, None) == hc_lib.HC_ERR_INVALID
    t.maskType = 1
    t.D = 300
    assert lib.hc_flash_attention_bwd_launch(*args, ctypes.byref(t), hc_lib.DT_BF16, None) == hc_lib.HC_ERR_UNSUPPORTED
    assert lib.hc_flash_attention_bwd_launch(*args, None, hc_lib.DT_BF16, None) == hc_lib.HC_ERR_INVALID
    kv = torch.zeros((1, 1, 128, 128), device="cuda", dtype=torch.bfloat16)
    with pytest.raises(hc_lib.HcError):
        hc_lib.flash_attention_bwd(x, kv, kv, x, lse, x, True)
    torch.cuda.synchronize()
    hc_lib.check_device_error()

"""GPU parity of flash_attention_fwd_fused (the headline operator) against the pinned oracle.

Golden: ops/flash_attention_fwd_fused/golden/flash_attention_fwd_fused_golden.cpp (online softmax,
fp64), restated in oracle/oracle.cpp with an added lse output.
  * the reference suite's 14 shape cases + its three hand-built tests, fp32 (SIMT kernel) at the
    reference tolerance 5e-4 and bf16 (tcgen05 kernel where D = D_v = 128) at max-abs 2e-2;
  * the check slice B=1 H=2 S=1024 D=128, N(0,1) inputs seeds 0/1/2, causal and non-causal,
    O max-abs 2e-2 and lse max-abs 2e-3;
  * ragged shapes for the tensor-core path (sequence tails, S_q != S_k, causal blocks that are not
    multiples of the 256-row work unit), fp16;
  * the full benchmarked configuration B=16 H=32 S=8192 D=128 (causal and non-causal) against the
    independent fp32-math SIMT kernel on sampled heads, plus size-independent properties;
  * the host-buffer runner against the device entry point (bit-identical);
  * the bounded-wait machinery reporting an expired wait as HC_ERR_TIMEOUT;
  * grouped-query attention (K/V with fewer heads) on both kernels;
  * head dimension 64, and D != D_v (64/128 either way), on the tensor-core kernel.
"""
from __future__ import annotations

import numpy as np
import pytest

import cases as C
from accuracy import assert_close
from gpu_util import bits, dev, host, quantize

pytestmark = pytest.mark.gpu

import specs

O_TOL_BF16 = specs.tolerance("flash_attention_fwd_fused", "bfloat16")["abs"]     # max-abs 2e-2 vs the golden (bf16 O)
LSE_TOL = specs.tolerance("flash_attention_fwd_fused", "bfloat16")["lse_abs"]    # 2e-3


def run_gpu(hc_lib, oracle, q, k, v, causal, kind, scale=None):
    import torch

    qd, kd, vd = dev(q, kind, oracle), dev(k, kind, oracle), dev(v, kind, oracle)
    o, lse = hc_lib.flash_attention_fwd(qd, kd, vd, bool(causal), scale=scale)
    torch.cuda.synchronize()
    hc_lib.check_device_error()
    return host(o, oracle), lse.cpu().numpy()


@pytest.mark.parametrize("case", C.FA_CASES, ids=lambda c: "B{}_H{}_Sq{}_Sk{}_D{}_Dv{}_{}".format(*c[:6], "causal" if c[6] else "none"))
def test_reference_cases_f32(cuda, hc_lib, oracle, case):
    B, H, Sq, Sk, D, Dv, causal = case
    q, k, v = C.fa_inputs(oracle, B, H, Sq, Sk, D, Dv)
    sc = C.default_scale(D)
    o, lse = run_gpu(hc_lib, oracle, q, k, v, causal, "f32", sc)
    ref, ref_lse = oracle.flash_attention_fwd(q, k, v, sc, causal)
    assert_close(ref, o, 5e-4, 5e-4, f"f32 {case}")  # test_flash_attention_fwd_fused.cpp:93-94
    assert_close(ref_lse, lse, 1e-4, 1e-4, f"lse {case}")


@pytest.mark.parametrize("case", C.FA_CASES, ids=lambda c: "B{}_H{}_Sq{}_Sk{}_D{}_Dv{}_{}".format(*c[:6], "causal" if c[6] else "none"))
def test_reference_cases_bf16(cuda, hc_lib, oracle, case):
    B, H, Sq, Sk, D, Dv, causal = case
    q, k, v = C.fa_inputs(oracle, B, H, Sq, Sk, D, Dv)
    sc = C.default_scale(D)
    o, lse = run_gpu(hc_lib, oracle, q, k, v, causal, "bf16", sc)
    if D == Dv and D in (64, 128):
        assert hc_lib.load().hc_flash_attention_last_path() == 1, "D = D_v = 64 or 128 must take the tcgen05 path"
    qq, kq, vq = (quantize(a, "bf16", oracle) for a in (q, k, v))
    ref, ref_lse = oracle.flash_attention_fwd(qq, kq, vq, sc, causal)
    r = assert_close(ref, o, O_TOL_BF16, 0.0, f"bf16 {case}")
    assert r.max_abs <= O_TOL_BF16
    assert_close(ref_lse, lse, LSE_TOL, 0.0, f"lse {case}")


@pytest.mark.parametrize("kind", ["f32", "bf16"])
def test_reference_special_cases(cuda, hc_lib, oracle, kind):
    """test_flash_attention_fwd_fused.cpp:183-288 on the device (D=128 variants hit tcgen05 for bf16)."""
    from golden.make_golden import special_fa_inputs

    for name, (q, k, v, sc, causal) in special_fa_inputs().items():
        for D in (q.shape[-1], 128):
            if D != q.shape[-1]:  # widen to D=128 with zero padding (scores unchanged: zeros add nothing)
                pad = ((0, 0), (0, 0), (0, 0), (0, D - q.shape[-1]))
                q2, k2, v2 = np.pad(q, pad), np.pad(k, pad), np.pad(v, pad)
            else:
                q2, k2, v2 = q, k, v
            o, _ = run_gpu(hc_lib, oracle, q2, k2, v2, causal, kind, float(sc))
            ref, _ = oracle.flash_attention_fwd(quantize(q2, kind, oracle), quantize(k2, kind, oracle),
                                                quantize(v2, kind, oracle), float(sc), causal)
            tol = 5e-4 if kind == "f32" else O_TOL_BF16
            assert_close(ref, o, tol, 0.0 if kind != "f32" else 5e-4, f"{name} D={D} {kind}")
            if name == "causal_constraint":
                col = o[0, 0, :, 0]
                assert np.all(col >= -tol) and np.all(col <= np.arange(8) + 0.01 + tol)
            else:
                np.testing.assert_allclose(o[0, 0, :, 0], 1.0, atol=max(tol, 1e-4))
    # ScaleInvariance: Q.(2K).(s/2) == Q.K.s
    q = oracle.uniform(2 * 8 * 32, 99).reshape(1, 2, 8, 32)
    k = oracle.uniform(2 * 8 * 32, 100).reshape(1, 2, 8, 32)
    v = oracle.uniform(2 * 8 * 32, 101).reshape(1, 2, 8, 32)
    base = float(np.float32(1.0) / np.sqrt(np.float32(32)))
    o1, _ = run_gpu(hc_lib, oracle, q, k, v, 0, kind, base)
    o2, _ = run_gpu(hc_lib, oracle, q, 2 * k, v, 0, kind, base / 2)
    np.testing.assert_allclose(o1, o2, atol=1e-4 if kind == "f32" else O_TOL_BF16)


@pytest.mark.parametrize("causal", [0, 1], ids=["none", "causal"])
def test_baseline_subslice(cuda, hc_lib, oracle, causal):
    """Check slice: B=1 H=2 S=1024 D=128, Q/K/V ~ N(0,1) seeds 0/1/2, scale 1/sqrt(128)."""
    B, H, S, D = 1, 2, 1024, 128
    q = oracle.normal(B * H * S * D, 0).reshape(B, H, S, D)
    k = oracle.normal(B * H * S * D, 1).reshape(B, H, S, D)
    v = oracle.normal(B * H * S * D, 2).reshape(B, H, S, D)
    sc = C.default_scale(D)
    o, lse = run_gpu(hc_lib, oracle, q, k, v, causal, "bf16", sc)
    assert hc_lib.load().hc_flash_attention_last_path() == 1
    ref, ref_lse = oracle.flash_attention_fwd(*(quantize(a, "bf16", oracle) for a in (q, k, v)), sc, causal, threads=8)
    r = assert_close(ref, o, O_TOL_BF16, 0.0, "subslice O")
    print(f"subslice causal={causal}: max_abs={r.max_abs:.3e} max_rel={r.max_rel:.3e}")
    assert_close(ref_lse, lse, LSE_TOL, 0.0, "subslice lse")


@pytest.mark.parametrize("shape", [
    (1, 3, 1000, 1000, 1), (2, 2, 300, 700, 0), (1, 1, 257, 257, 1), (1, 2, 384, 384, 1), (1, 1, 1, 1, 0),
    (1, 1, 129, 1, 0), (1, 2, 300, 200, 1), (3, 5, 640, 640, 0), (1, 1, 513, 1024, 1), (1, 1, 64, 2048, 0),
], ids=lambda s: "B{}_H{}_Sq{}_Sk{}_{}".format(*s[:4], "causal" if s[4] else "none"))
@pytest.mark.parametrize("kind", ["bf16", "f16"])
def test_tensor_core_ragged_shapes(cuda, hc_lib, oracle, shape, kind):
    B, H, Sq, Sk, causal = shape
    D = 128
    q = oracle.normal(B * H * Sq * D, 10).reshape(B, H, Sq, D)
    k = oracle.normal(B * H * Sk * D, 11).reshape(B, H, Sk, D)
    v = oracle.normal(B * H * Sk * D, 12).reshape(B, H, Sk, D)
    sc = C.default_scale(D)
    o, lse = run_gpu(hc_lib, oracle, q, k, v, causal, kind, sc)
    assert hc_lib.load().hc_flash_attention_last_path() == 1
    ref, ref_lse = oracle.flash_attention_fwd(*(quantize(a, kind, oracle) for a in (q, k, v)), sc, causal, threads=8)
    assert_close(ref, o, O_TOL_BF16 if kind == "bf16" else 5e-3, 0.0, f"{kind} {shape}")
    assert_close(ref_lse, lse, LSE_TOL, 0.0, f"lse {shape}")


@pytest.mark.parametrize("shape", [(2, 8, 2, 300, 300, 1), (1, 4, 1, 512, 700, 0), (1, 6, 3, 257, 257, 1),
                                   (2, 4, 2, 128, 64, 0)],
                         ids=lambda s: "B{}_H{}_Hkv{}_Sq{}_Sk{}_{}".format(*s[:5], "causal" if s[5] else "none"))
@pytest.mark.parametrize("kind", ["bf16", "f16"])
def test_grouped_query_attention(cuda, hc_lib, oracle, shape, kind):
    """K/V with H_kv < H heads (hc_flash_attention_fwd_fused_gqa_launch): against the oracle on K/V
    heads repeated H / H_kv times, and bit-identical to the tensor-core kernel run on that repeated copy."""
    import torch

    B, H, Hkv, Sq, Sk, causal = shape
    D, g = 128, H // Hkv
    q = oracle.normal(B * H * Sq * D, 20).reshape(B, H, Sq, D)
    k = oracle.normal(B * Hkv * Sk * D, 21).reshape(B, Hkv, Sk, D)
    v = oracle.normal(B * Hkv * Sk * D, 22).reshape(B, Hkv, Sk, D)
    sc = C.default_scale(D)
    o, lse = run_gpu(hc_lib, oracle, q, k, v, causal, kind, sc)
    assert hc_lib.load().hc_flash_attention_last_path() == 1
    kx, vx = np.repeat(k, g, axis=1), np.repeat(v, g, axis=1)
    ref, ref_lse = oracle.flash_attention_fwd(*(quantize(a, kind, oracle) for a in (q, kx, vx)), sc, causal, threads=8)
    assert_close(ref, o, O_TOL_BF16 if kind == "bf16" else 5e-3, 0.0, f"gqa {kind} {shape}")
    assert_close(ref_lse, lse, LSE_TOL, 0.0, f"gqa lse {shape}")
    o_mha, lse_mha = run_gpu(hc_lib, oracle, q, kx, vx, causal, kind, sc)
    assert np.array_equal(o, o_mha) and np.array_equal(lse, lse_mha)
    torch.cuda.synchronize()


@pytest.mark.parametrize("kind", ["f32", "bf16"])
def test_grouped_query_attention_simt(cuda, hc_lib, oracle, kind):
    """D = 32 GQA takes the SIMT kernel, which maps heads the same way."""
    B, H, Hkv, S, D = 1, 4, 2, 96, 32
    q = oracle.uniform(B * H * S * D, 30).reshape(B, H, S, D)
    k = oracle.uniform(B * Hkv * S * D, 31).reshape(B, Hkv, S, D)
    v = oracle.uniform(B * Hkv * S * D, 32).reshape(B, Hkv, S, D)
    sc = C.default_scale(D)
    o, lse = run_gpu(hc_lib, oracle, q, k, v, 1, kind, sc)
    assert hc_lib.load().hc_flash_attention_last_path() == 2
    kx, vx = np.repeat(k, 2, axis=1), np.repeat(v, 2, axis=1)
    ref, ref_lse = oracle.flash_attention_fwd(*(quantize(a, kind, oracle) for a in (q, kx, vx)), sc, 1)
    tol = 5e-4 if kind == "f32" else O_TOL_BF16
    assert_close(ref, o, tol, 0.0, f"gqa simt {kind}")
    assert_close(ref_lse, lse, 1e-3, 0.0, f"gqa simt lse {kind}")


@pytest.mark.parametrize("shape", [
    (1, 3, 1000, 1000, 1), (2, 2, 300, 700, 0), (1, 1, 257, 257, 1), (1, 1, 1, 1, 0), (1, 2, 300, 200, 1),
    (3, 5, 640, 640, 0), (1, 1, 513, 1024, 1),
], ids=lambda s: "B{}_H{}_Sq{}_Sk{}_{}".format(*s[:4], "causal" if s[4] else "none"))
@pytest.mark.parametrize("kind", ["bf16", "f16"])
def test_tensor_core_head_dim_64(cuda, hc_lib, oracle, shape, kind):
    """D = D_v = 64 on the tcgen05 kernel (one swizzle panel per tile, N = 64 P.V, 8-stage K/V ring)."""
    B, H, Sq, Sk, causal = shape
    D = 64
    q = oracle.normal(B * H * Sq * D, 40).reshape(B, H, Sq, D)
    k = oracle.normal(B * H * Sk * D, 41).reshape(B, H, Sk, D)
    v = oracle.normal(B * H * Sk * D, 42).reshape(B, H, Sk, D)
    sc = C.default_scale(D)
    o, lse = run_gpu(hc_lib, oracle, q, k, v, causal, kind, sc)
    assert hc_lib.load().hc_flash_attention_last_path() == 1
    ref, ref_lse = oracle.flash_attention_fwd(*(quantize(a, kind, oracle) for a in (q, k, v)), sc, causal, threads=8)
    assert_close(ref, o, O_TOL_BF16 if kind == "bf16" else 5e-3, 0.0, f"D64 {kind} {shape}")
    assert_close(ref_lse, lse, LSE_TOL, 0.0, f"D64 lse {shape}")


@pytest.mark.parametrize("dims", [(128, 64), (64, 128)], ids=lambda d: "D{}_Dv{}".format(*d))
@pytest.mark.parametrize("shape", [(1, 2, 300, 300, 1, 2), (2, 2, 257, 400, 0, 2), (1, 4, 513, 513, 1, 1),
                                   (1, 1, 1, 1, 0, 1)],
                         ids=lambda s: "B{}_H{}_Sq{}_Sk{}_{}_Hkv{}".format(*s[:4], "causal" if s[4] else "none", s[5]))
@pytest.mark.parametrize("kind", ["bf16", "f16"])
def test_tensor_core_value_dim_differs(cuda, hc_lib, oracle, dims, shape, kind):
    """D != D_v on the tcgen05 kernel: Q/K tiles of D columns, V and O of D_v, K/V ring slots of the larger."""
    D, Dv = dims
    B, H, Sq, Sk, causal, Hkv = shape
    q = oracle.normal(B * H * Sq * D, 50).reshape(B, H, Sq, D)
    k = oracle.normal(B * Hkv * Sk * D, 51).reshape(B, Hkv, Sk, D)
    v = oracle.normal(B * Hkv * Sk * Dv, 52).reshape(B, Hkv, Sk, Dv)
    sc = C.default_scale(D)
    o, lse = run_gpu(hc_lib, oracle, q, k, v, causal, kind, sc)
    assert hc_lib.load().hc_flash_attention_last_path() == 1
    g = H // Hkv
    kx, vx = np.repeat(k, g, axis=1), np.repeat(v, g, axis=1)
    ref, ref_lse = oracle.flash_attention_fwd(*(quantize(a, kind, oracle) for a in (q, kx, vx)), sc, causal, threads=8)
    assert o.shape == (B, H, Sq, Dv)
    assert_close(ref, o, O_TOL_BF16 if kind == "bf16" else 5e-3, 0.0, f"D{D} Dv{Dv} {kind} {shape}")
    assert_close(ref_lse, lse, LSE_TOL, 0.0, f"D{D} Dv{Dv} lse {shape}")


def test_tensor_core_head_dim_64_gqa_against_simt(cuda, hc_lib, oracle):
    """D = 64 grouped-query causal on the tcgen05 kernel against the fp32-math SIMT kernel (fp32 inputs)."""
    import torch

    B, H, Hkv, S, D = 2, 8, 2, 1536, 64
    g = torch.Generator(device="cuda").manual_seed(3)
    q = torch.randn(B, H, S, D, generator=g, device="cuda").to(torch.bfloat16)
    k = torch.randn(B, Hkv, S, D, generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn(B, Hkv, S, D, generator=g, device="cuda").to(torch.bfloat16)
    o, lse = hc_lib.flash_attention_fwd(q, k, v, True)
    assert hc_lib.load().hc_flash_attention_last_path() == 1
    o32, lse32 = hc_lib.flash_attention_fwd(q.float(), k.float(), v.float(), True)
    assert hc_lib.load().hc_flash_attention_last_path() == 2
    torch.cuda.synchronize()
    hc_lib.check_device_error()
    assert (o.float() - o32).abs().max().item() <= O_TOL_BF16
    assert (lse - lse32).abs().max().item() <= LSE_TOL


def test_large_logits_lazy_rescale(cuda, hc_lib, oracle):
    """Scores that grow along the sequence force the running max to move many times (exercises the
    O rescale in TMEM); a large scale makes softmax nearly one-hot."""
    B, H, S, D = 1, 2, 768, 128
    q = oracle.normal(B * H * S * D, 20).reshape(B, H, S, D)
    k = (oracle.normal(B * H * S * D, 21).reshape(B, H, S, D) * np.linspace(0.1, 4.0, S, dtype=np.float32)[None, None, :, None])
    v = oracle.normal(B * H * S * D, 22).reshape(B, H, S, D)
    for causal in (0, 1):
        o, lse = run_gpu(hc_lib, oracle, q, k, v, causal, "bf16", 0.5)
        ref, ref_lse = oracle.flash_attention_fwd(*(quantize(a, "bf16", oracle) for a in (q, k, v)), 0.5, causal, threads=8)
        assert_close(ref, o, 3e-2, 0.0, f"large logits causal={causal}")
        assert_close(ref_lse, lse, 1e-2, 1e-4, "large logits lse")


def _fa_reference_fp64(q, k, v, causal, scale):
    """softmax(q k^T * scale) v and the natural-log lse of one head ([S, D]) in float64 on the device."""
    import torch

    s = (q.double() @ k.double().transpose(0, 1)) * scale
    if causal:
        s = s.masked_fill(torch.ones_like(s, dtype=torch.bool).triu(1), float("-inf"))
    return torch.softmax(s, dim=-1) @ v.double(), torch.logsumexp(s, dim=-1)


@pytest.mark.parametrize("causal", [1, 0], ids=["causal", "none"])
def test_full_config_against_simt(cuda, hc_lib, oracle, causal):
    """Benchmarked configuration: Q, K, V bf16 [16, 32, 8192, 128] ~ N(0,1) (device generator seeds 0/1/2),
    causal and non-causal.  32 heads spread over all of batch x heads are recomputed in float64 on the
    device (a plain softmax(QK^T)V); three of them also by the fp32-math SIMT kernel (an independent
    code path pinned to the oracle by test_reference_cases_f32); every row is checked for the
    convex-combination property min_j V <= O <= max_j V and a finite lse."""
    import torch

    cfg = specs.bench_config("flash_attention_fwd_fused")
    B, H, S, D = cfg["B"], cfg["H"], cfg["S_q"], cfg["D"]
    gens = [torch.Generator(device="cuda").manual_seed(s) for s in (0, 1, 2)]
    q, k, v = (torch.randn((B, H, S, D), generator=g, device="cuda", dtype=torch.float32).to(torch.bfloat16) for g in gens)
    o, lse = hc_lib.flash_attention_fwd(q, k, v, bool(causal))
    torch.cuda.synchronize()
    hc_lib.check_device_error()
    assert hc_lib.load().hc_flash_attention_last_path() == 1
    assert torch.isfinite(lse).all()
    vmin = v.float().amin(dim=2, keepdim=True)
    vmax = v.float().amax(dim=2, keepdim=True)
    of = o.float()
    assert bool(((of >= vmin - 1e-2) & (of <= vmax + 1e-2)).all()), "O outside the convex hull of V"
    del vmin, vmax, of
    spread = sorted({(i * B * H // 32 + (i * 7) % (B * H // 32)) for i in range(32)} | {0, B * H - 1})
    scale = C.default_scale(D)
    for bh in spread:
        b, h = divmod(bh, H)
        o_ref, l_ref = _fa_reference_fp64(q[b, h], k[b, h], v[b, h], bool(causal), scale)
        err = (o[b, h].double() - o_ref).abs().max().item()
        lerr = (lse[b, h].double() - l_ref).abs().max().item()
        assert err <= O_TOL_BF16, (b, h, err)
        assert lerr <= LSE_TOL, (b, h, lerr)
    heads = [(0, 0), (B - 1, H - 1), (B // 2, 7)]
    for (b, h) in heads:
        qs, ks, vs = (t[b:b + 1, h:h + 1].contiguous().float() for t in (q, k, v))
        o_ref, lse_ref = hc_lib.flash_attention_fwd(qs, ks, vs, bool(causal))
        assert hc_lib.load().hc_flash_attention_last_path() == 2
        err = (o[b:b + 1, h:h + 1].float() - o_ref).abs().max().item()
        lerr = (lse[b:b + 1, h:h + 1] - lse_ref).abs().max().item()
        assert err <= O_TOL_BF16, (b, h, err)
        assert lerr <= LSE_TOL, (b, h, lerr)
    if causal:  # query 0 sees only key 0: O[.., 0, :] == V[.., 0, :] up to one bf16 rounding
        assert torch.allclose(o[:, :, 0].float(), v[:, :, 0].float(), atol=1e-2, rtol=0)


def test_host_runner_matches_device(cuda, hc_lib, oracle):
    """hc_flash_attention_fwd_fused_host (host buffers, chunked, copies overlapped) produces the
    same bits as the device entry point."""
    import ctypes

    import torch

    B, H, S, D = 2, 40, 1024, 128
    gens = [torch.Generator(device="cuda").manual_seed(s) for s in (5, 6, 7)]
    q, k, v = (torch.randn((B, H, S, D), generator=g, device="cuda").to(torch.bfloat16) for g in gens)
    o_dev, lse_dev = hc_lib.flash_attention_fwd(q, k, v, True)
    hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
    ho = torch.empty_like(hq).pin_memory()
    hl = torch.empty((B, H, S), dtype=torch.float32).pin_memory()
    t = hc_lib.FlashAttentionFwdFusedTiling(B, H, S, S, D, D, C.default_scale(D), 1)
    lib = hc_lib.load()
    ws = ctypes.c_size_t()
    hc_lib.check(lib.hc_flash_attention_fwd_fused_host_workspace_size(ctypes.byref(t), hc_lib.DT_BF16, ctypes.byref(ws)))
    work = torch.empty(ws.value, dtype=torch.uint8, device="cuda")
    hc_lib.check(lib.hc_flash_attention_fwd_fused_host(hq.data_ptr(), hk.data_ptr(), hv.data_ptr(), ho.data_ptr(),
                                                       hl.data_ptr(),
                                                       ctypes.byref(t), hc_lib.DT_BF16, work.data_ptr(), ws.value,
                                                       torch.cuda.current_stream().cuda_stream))
    assert torch.equal(ho.view(torch.int16), o_dev.cpu().view(torch.int16))
    assert torch.equal(hl, lse_dev.cpu())


def test_host_runner_error_returns_after_queued_chunks(cuda, hc_lib):
    """An error in the middle of the chunked host runner (an injected copy failure at chunk 2 of 3)
    is returned only once the chunks already queued are finished: chunk 1's output is complete in
    host memory the moment the call returns, so the caller may free the workspace at once."""
    import ctypes

    import torch

    B, H, S, D = 1, 48, 8192, 128  # 6 MiB of q/k/v per head: 16 heads per ~96 MB chunk, three chunks
    gens = [torch.Generator(device="cuda").manual_seed(s) for s in (8, 9, 10)]
    q, k, v = (torch.randn((B, H, S, D), generator=g, device="cuda").to(torch.bfloat16) for g in gens)
    o_dev, _ = hc_lib.flash_attention_fwd(q, k, v, True)
    hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
    ho = torch.full((B, H, S, D), float("nan"), dtype=torch.bfloat16).pin_memory()
    t = hc_lib.FlashAttentionFwdFusedTiling(B, H, S, S, D, D, C.default_scale(D), 1)
    lib = hc_lib.load()
    ws = ctypes.c_size_t()
    hc_lib.check(lib.hc_flash_attention_fwd_fused_host_workspace_size(ctypes.byref(t), hc_lib.DT_BF16, ctypes.byref(ws)))
    work = torch.empty(ws.value, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    hc_lib.check(lib.hc_set_fault(b"memcpy:2"))
    try:
        st = lib.hc_flash_attention_fwd_fused_host(hq.data_ptr(), hk.data_ptr(), hv.data_ptr(), ho.data_ptr(), None,
                                                   ctypes.byref(t), hc_lib.DT_BF16, work.data_ptr(), ws.value,
                                                   torch.cuda.current_stream().cuda_stream)
        done = ho[:, :16].clone()  # read before any synchronisation of ours
    finally:
        lib.hc_set_fault(None)
    assert st == hc_lib.HC_ERR_INJECTED
    assert torch.equal(done.view(torch.int16), o_dev[:, :16].cpu().view(torch.int16))
    del work


def test_bounded_wait_reports_timeout(cuda, hc_lib):
    """A wait that can never complete gives up after its budget and is reported, not hung on."""
    lib = hc_lib.load()
    assert lib.hc_check_device_error() == hc_lib.HC_OK
    assert lib.hc_selftest_bounded_wait(20000) == hc_lib.HC_ERR_TIMEOUT
    assert b"bounded wait expired" in lib.hc_last_error_string()
    assert lib.hc_check_device_error() == hc_lib.HC_OK  # the word was cleared
    # the context is still usable
    import torch

    x = torch.ones(1024, device="cuda", dtype=torch.float16)
    assert torch.equal(hc_lib.elementwise_add(x, x), x * 2)

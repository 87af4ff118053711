"""C-ABI boundary checks that need no GPU: the library loads, exports every entry point declared
in include/*.h, keeps the reference's tiling-struct layouts, and rejects bad arguments (and
injected faults) on the host with a status code instead of running anything."""
from __future__ import annotations

import ctypes as C
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared_functions() -> set[str]:
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names.update(re.findall(r"\b(hc_[a-z0-9_]+)\s*\(", text))
    return names


def test_every_declared_symbol_is_exported(hc_lib):
    out = subprocess.run(["nm", "-D", "--defined-only", str(hc_lib.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = declared_functions() - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"
    assert declared_functions() <= set(hc_lib.SIGNATURES), "binding lacks a declared entry point"


def test_library_loads_and_reports_no_device_gracefully(hc_lib):
    lib = hc_lib.load()
    n = C.c_int(-1)
    st = lib.hc_device_count(C.byref(n))
    assert st in (hc_lib.HC_OK, hc_lib.HC_ERR_NO_DEVICE)
    if st == hc_lib.HC_ERR_NO_DEVICE:
        assert n.value == 0 and lib.hc_last_error_string()


def test_tiling_struct_layouts(hc_lib):
    """Same sizes as the reference PODs (host/<op>_tiling.h: u32/f32 fields, no padding)."""
    sizes = {hc_lib.ElementwiseAddTiling: 8, hc_lib.AxpyScalarAffineTiling: 8, hc_lib.BroadcastBinaryTiling: 24,
             hc_lib.ActivationGeluSiluTiling: 12, hc_lib.ReduceSumLastdimTiling: 12, hc_lib.Transpose2d4dTiling: 24,
             hc_lib.LayerNormTiling: 16, hc_lib.RmsNormRopeFusedTiling: 24, hc_lib.MatmulBiasTiling: 24,
             hc_lib.FlashAttentionFwdFusedTiling: 32}
    for cls, size in sizes.items():
        assert C.sizeof(cls) == size, cls.__name__


def test_host_side_validation_needs_no_gpu(hc_lib):
    lib = hc_lib.load()
    fake = C.c_void_p(0x1000)  # never dereferenced: every call below fails validation first
    t = hc_lib.FlashAttentionFwdFusedTiling(1, 1, 16, 0, 128, 128, 0.1, 0)
    assert lib.hc_flash_attention_fwd_fused_launch(fake, fake, fake, fake, None, C.byref(t), 2, None) == hc_lib.HC_ERR_INVALID
    assert b"S_k" in lib.hc_last_error_string()
    t = hc_lib.FlashAttentionFwdFusedTiling(1, 1, 16, 16, 512, 128, 0.1, 0)
    assert lib.hc_flash_attention_fwd_fused_launch(fake, fake, fake, fake, None, C.byref(t), 2, None) == hc_lib.HC_ERR_UNSUPPORTED
    t = hc_lib.FlashAttentionFwdFusedTiling(1, 1, 16, 16, 128, 128, 0.1, 2)
    assert lib.hc_flash_attention_fwd_fused_launch(fake, fake, fake, fake, None, C.byref(t), 2, None) == hc_lib.HC_ERR_INVALID
    t = hc_lib.FlashAttentionFwdFusedTiling(1, 1, 16, 16, 128, 128, 0.1, 0)
    assert lib.hc_flash_attention_fwd_fused_launch(None, fake, fake, fake, None, C.byref(t), 2, None) == hc_lib.HC_ERR_INVALID
    assert lib.hc_flash_attention_fwd_fused_launch(fake, fake, fake, fake, None, None, 2, None) == hc_lib.HC_ERR_INVALID
    bt = hc_lib.BroadcastBinaryTiling(2, 3, 4, 5, 3, 0)  # y_batch must be 1 or B
    assert lib.hc_broadcast_binary_launch(fake, fake, fake, fake, C.byref(bt), 0, None) == hc_lib.HC_ERR_INVALID
    rt = hc_lib.ReduceSumLastdimTiling(4, 0, 0)
    assert lib.hc_reduce_sum_lastdim_launch(fake, fake, C.byref(rt), 0, None) == hc_lib.HC_ERR_INVALID
    at = hc_lib.ActivationGeluSiluTiling(16, 0, 7)
    assert lib.hc_activation_gelu_silu_launch(fake, fake, C.byref(at), 0, None) == hc_lib.HC_ERR_INVALID
    tt = hc_lib.Transpose2d4dTiling(9, 2, 2, 1, 1, 0)
    assert lib.hc_transpose_2d_4d_launch(fake, fake, C.byref(tt), 0, None) == hc_lib.HC_ERR_INVALID
    rr = hc_lib.RmsNormRopeFusedTiling(1, 4, 64, 65, 0, 1e-6)  # odd rotary dim
    assert lib.hc_rms_norm_rope_fused_launch(fake, fake, fake, fake, fake, C.byref(rr), 1, 0, 2, None) == hc_lib.HC_ERR_INVALID
    mt = hc_lib.MatmulBiasTiling(4, 0, 4, 0, 0, 0)
    assert lib.hc_matmul_bias_launch(fake, fake, None, fake, C.byref(mt), 2, None) == hc_lib.HC_ERR_INVALID
    et = hc_lib.ElementwiseAddTiling(16, 0)
    assert lib.hc_elementwise_add_launch(fake, fake, fake, C.byref(et), 9, None) == hc_lib.HC_ERR_UNSUPPORTED
    gt = hc_lib.FlashAttentionFwdFusedTiling(1, 8, 16, 16, 128, 128, 0.1, 0)
    for kv_heads in (0, 3, 16):  # must divide H = 8
        assert lib.hc_flash_attention_fwd_fused_gqa_launch(fake, fake, fake, fake, None, C.byref(gt), kv_heads, 2,
                                                           None) == hc_lib.HC_ERR_INVALID
        assert b"kv_heads" in lib.hc_last_error_string()


def test_backward_validation_needs_no_gpu(hc_lib):
    """hc_flash_attention_bwd_launch checks the tiling, pointers and element type on the host before any
    device work, with the forward's rules, and an injected launch fault surfaces as HC_ERR_INJECTED."""
    lib = hc_lib.load()
    fake = C.c_void_p(0x1000)  # never dereferenced: every call below fails before device work
    args = [fake] * 5 + [fake] + [fake] * 3 + [fake]

    def call(t, dtype=2, a=args):
        return lib.hc_flash_attention_bwd_launch(*a, C.byref(t) if t is not None else None, dtype, None)

    assert call(None) == hc_lib.HC_ERR_INVALID
    assert call(hc_lib.FlashAttentionFwdFusedTiling(1, 1, 16, 0, 128, 128, 0.1, 0)) == hc_lib.HC_ERR_INVALID  # S_k = 0
    assert call(hc_lib.FlashAttentionFwdFusedTiling(1, 1, 16, 16, 512, 128, 0.1, 0)) == hc_lib.HC_ERR_UNSUPPORTED
    assert call(hc_lib.FlashAttentionFwdFusedTiling(1, 1, 16, 16, 128, 128, 0.1, 2)) == hc_lib.HC_ERR_INVALID  # mask
    assert call(hc_lib.FlashAttentionFwdFusedTiling(1, 1, 16, 16, 128, 128, float("nan"), 0)) == hc_lib.HC_ERR_INVALID
    good = hc_lib.FlashAttentionFwdFusedTiling(1, 1, 16, 16, 128, 128, 0.1, 0)
    assert call(good, dtype=9) == hc_lib.HC_ERR_UNSUPPORTED
    for i in range(10):  # every pointer argument is required
        a = list(args)
        a[i] = None
        assert call(good, a=a) == hc_lib.HC_ERR_INVALID, i
    assert call(hc_lib.FlashAttentionFwdFusedTiling(0, 1, 16, 16, 128, 128, 0.1, 0)) == hc_lib.HC_OK  # empty problem
    assert lib.hc_set_fault(b"launch:1") == hc_lib.HC_OK
    try:
        assert call(good) == hc_lib.HC_ERR_INJECTED
    finally:
        lib.hc_set_fault(None)


def test_fault_injection_is_reported_not_hidden(hc_lib):
    """HC_FAULT makes the n-th launch fail on the host; the status propagates (no fallback)."""
    lib = hc_lib.load()
    fake = C.c_void_p(0x1000)
    et = hc_lib.ElementwiseAddTiling(16, 0)
    assert lib.hc_set_fault(b"launch:1") == hc_lib.HC_OK
    try:
        assert lib.hc_elementwise_add_launch(fake, fake, fake, C.byref(et), 1, None) == hc_lib.HC_ERR_INJECTED
        assert b"injected" in lib.hc_last_error_string()
    finally:
        lib.hc_set_fault(None)
    assert lib.hc_set_fault(b"malloc:1") == hc_lib.HC_OK
    try:
        p = C.c_void_p()
        assert lib.hc_malloc(C.byref(p), 64) == hc_lib.HC_ERR_INJECTED and not p.value
    finally:
        lib.hc_set_fault(None)


def test_python_binding_raises_on_error(hc_lib):
    with pytest.raises(hc_lib.HcError) as ei:
        hc_lib.check(hc_lib.HC_ERR_INVALID)
    assert ei.value.status == hc_lib.HC_ERR_INVALID


def test_noalloc_runner_limits_are_checked_on_the_host(hc_lib):
    """The allocation-free runner rejects a head larger than its fixed scratch before any device work."""
    lib = hc_lib.load()
    assert lib.hc_flash_attention_fwd_fused_host_noalloc_limit() == 64 << 20
    fake = C.c_void_p(0x1000)
    big = hc_lib.FlashAttentionFwdFusedTiling(1, 1, 1 << 20, 1 << 20, 128, 128, 0.088, 1)  # one head: 1 GiB
    assert lib.hc_flash_attention_fwd_fused_host_noalloc(fake, fake, fake, fake, None, C.byref(big), 2, None) \
        == hc_lib.HC_ERR_UNSUPPORTED
    assert "scratch" in hc_lib.load().hc_last_error_string().decode()
    assert lib.hc_flash_attention_fwd_fused_host_noalloc(None, fake, fake, fake, None, C.byref(big), 2, None) \
        == hc_lib.HC_ERR_INVALID
    assert lib.hc_flash_attention_fwd_fused_host_noalloc(fake, fake, fake, fake, None, C.byref(big), 3, None) \
        == hc_lib.HC_ERR_UNSUPPORTED
    # tilings the kernel would reject are refused before the first copy is queued (no device here)
    for bad, status in (((1, 1, 64, 64, 300, 300, 0.05, 0), hc_lib.HC_ERR_UNSUPPORTED),   # D > 256
                        ((1, 1, 64, 64, 128, 128, 0.05, 2), hc_lib.HC_ERR_INVALID),       # maskType
                        ((1, 1, 64, 0, 128, 128, 0.05, 1), hc_lib.HC_ERR_INVALID),        # S_k = 0
                        ((1, 1, 64, 64, 128, 128, float("inf"), 1), hc_lib.HC_ERR_INVALID)):  # scale
        t = hc_lib.FlashAttentionFwdFusedTiling(*bad)
        for fn in ("hc_flash_attention_fwd_fused_host_noalloc",):
            assert getattr(lib, fn)(fake, fake, fake, fake, None, C.byref(t), 2, None) == status, (bad, fn)
        assert lib.hc_flash_attention_fwd_fused_host(fake, fake, fake, fake, None, C.byref(t), 2, fake, 1 << 30,
                                                     None) == status, bad

"""GPU test of the allocation-free host-buffer flash-attention runner
(hc_flash_attention_fwd_fused_host_noalloc: staging in a fixed scratch array inside the library),
for callers that cannot allocate device memory on this path.

Two calls in a row, on different shapes and inputs (the second reuses the scratch the first
wrote), must give results bit-identical to the workspace runner hc_flash_attention_fwd_fused_host
on the same inputs; the last case needs several chunks of the 64 MiB scratch.  A small case is
also checked against the CPU oracle, and the device's free memory is the same before and after a
call (torch's caching allocator idle meanwhile).  The file sorts last so it also runs after every
other GPU test."""
from __future__ import annotations

import ctypes as C
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _inputs(torch, B, H, Sq, Sk, D, seed):
    g = torch.Generator().manual_seed(seed)
    mk = lambda S: torch.randn((B, H, S, D), generator=g).to(torch.bfloat16).pin_memory()  # noqa: E731
    return mk(Sq), mk(Sk), mk(Sk)


def _run_both(hc_lib, torch, B, H, Sq, Sk, D, causal, seed):
    lib = hc_lib.load()
    q, k, v = _inputs(torch, B, H, Sq, Sk, D, seed)
    t = hc_lib.FlashAttentionFwdFusedTiling(B, H, Sq, Sk, D, D, 1.0 / math.sqrt(D), causal)
    stream = torch.cuda.current_stream().cuda_stream
    # workspace runner (reference entry point)
    o_ref = torch.empty((B, H, Sq, D), dtype=torch.bfloat16).pin_memory()
    l_ref = torch.empty((B, H, Sq), dtype=torch.float32).pin_memory()
    ws = C.c_size_t()
    hc_lib.check(lib.hc_flash_attention_fwd_fused_host_workspace_size(C.byref(t), hc_lib.DT_BF16, C.byref(ws)))
    work = torch.empty(ws.value, dtype=torch.uint8, device="cuda")
    hc_lib.check(lib.hc_flash_attention_fwd_fused_host(q.data_ptr(), k.data_ptr(), v.data_ptr(), o_ref.data_ptr(),
                                                       l_ref.data_ptr(), C.byref(t), hc_lib.DT_BF16, work.data_ptr(),
                                                       ws.value, stream))
    del work
    # allocation-free runner
    o = torch.full((B, H, Sq, D), float("nan"), dtype=torch.bfloat16).pin_memory()
    lse = torch.full((B, H, Sq), float("nan"), dtype=torch.float32).pin_memory()
    hc_lib.check(lib.hc_flash_attention_fwd_fused_host_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                                               lse.data_ptr(), C.byref(t), hc_lib.DT_BF16, stream))
    assert lib.hc_flash_attention_last_path() == 1
    return o_ref, l_ref, o, lse


def test_noalloc_matches_workspace_runner_on_two_calls_in_a_row(cuda, hc_lib):
    import torch

    cases = [(2, 5, 700, 700, 128, 1, 11),       # ragged causal, one chunk
             (1, 16, 8192, 8192, 128, 0, 12)]    # 8 MiB of staging per head: three chunks of the scratch
    for B, H, Sq, Sk, D, causal, seed in cases:
        o_ref, l_ref, o, lse = _run_both(hc_lib, torch, B, H, Sq, Sk, D, causal, seed)
        assert torch.equal(o.view(torch.int16), o_ref.view(torch.int16)), (B, H, Sq, causal)
        assert np.array_equal(lse.numpy(), l_ref.numpy()), (B, H, Sq, causal)


def test_noalloc_matches_oracle_and_allocates_nothing(cuda, hc_lib, oracle):
    import torch

    from accuracy import assert_close
    from gpu_util import quantize

    lib = hc_lib.load()
    B, H, S, D = 1, 2, 300, 128
    q, k, v = (oracle.normal(B * H * S * D, s).reshape(B, H, S, D) for s in (61, 62, 63))
    pin = lambda a: torch.from_numpy(oracle.to_bf16(a).view(np.int16).copy()).view(torch.bfloat16).pin_memory()  # noqa: E731
    hq, hk, hv = pin(q), pin(k), pin(v)
    o = torch.empty((B, H, S, D), dtype=torch.bfloat16).pin_memory()
    lse = torch.empty((B, H, S), dtype=torch.float32).pin_memory()
    t = hc_lib.FlashAttentionFwdFusedTiling(B, H, S, S, D, D, 1.0 / math.sqrt(D), 1)
    stream = torch.cuda.current_stream().cuda_stream
    call = lambda: lib.hc_flash_attention_fwd_fused_host_noalloc(hq.data_ptr(), hk.data_ptr(), hv.data_ptr(),  # noqa: E731
                                                                 o.data_ptr(), lse.data_ptr(), C.byref(t),
                                                                 hc_lib.DT_BF16, stream)
    hc_lib.check(call())  # the device's first call: address lookup and kernel attributes
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info()
    hc_lib.check(call())
    free_after, _ = torch.cuda.mem_get_info()
    assert free_after == free_before, (free_before, free_after)
    got = oracle.from_bf16(o.view(torch.int16).numpy().view(np.uint16))
    ref, ref_lse = oracle.flash_attention_fwd(*(quantize(a, "bf16", oracle) for a in (q, k, v)), 1.0 / np.sqrt(D), 1)
    assert_close(ref, got, 2e-2, 0.0, "no-alloc runner vs oracle")
    assert_close(ref_lse, lse.numpy(), 2e-3, 0.0, "no-alloc lse vs oracle")

"""One host thread per GPU in one process (the runner threading model of the reference's device
layer, src/ascend_runtime.cpp:170-172, made per thread): two threads each select their device with
hc_set_device and run the tensor-core flash attention, the tcgen05 GEMM, the direct-load
LayerNorm, the row-stream RMSNorm+RoPE and the TMA transpose; every result is compared with the
oracle, and the attention backward (its two tcgen05 kernels) against the oracle's gradients.  Device 1
first runs after device 0 has launched every kernel (its shared-memory opt-ins must be made on device 1
too), then both devices run at the same time, twice.  Needs 2 GPUs."""
from __future__ import annotations

import threading

import numpy as np
import pytest

from accuracy import assert_close
from gpu_util import bits, host, quantize

pytestmark = pytest.mark.gpu


def _inputs(oracle):
    x = {}
    B, H, S, D = 1, 3, 640, 128
    x["fa"] = tuple(oracle.normal(B * H * S * D, s).reshape(B, H, S, D) for s in (31, 32, 33))
    M, K, N = 384, 512, 640
    x["mm"] = ((oracle.normal(M * K, 34) / 16).reshape(M, K), (oracle.normal(K * N, 35) / 16).reshape(K, N),
               oracle.normal(N, 36, 0.0, 0.1))
    x["ln"] = (oracle.normal(96 * 4096, 37).reshape(96, 4096), oracle.uniform(4096, 38, 0.5, 1.5),
               oracle.uniform(4096, 39, -0.1, 0.1))
    cos, sin = oracle.rope_cos_sin(48, 64)
    x["rms"] = (oracle.normal(2 * 48 * 4 * 128, 40).reshape(2, 48, 4, 128), oracle.uniform(128, 41, 0.5, 1.5), cos, sin)
    x["tr"] = oracle.normal(256 * 320, 42).reshape(256, 320)
    x["do"] = oracle.normal(B * H * S * D, 43).reshape(B, H, S, D)
    return x


def _upload(a, oracle, kind="bf16"):
    import torch

    a = np.ascontiguousarray(a, np.float32)
    if kind == "f32":
        return torch.from_numpy(a.copy()).cuda()
    return torch.from_numpy(oracle.to_bf16(a).view(np.int16).copy()).cuda().view(torch.bfloat16)


def _run_device(device: int, hc_lib, oracle, x, out: dict, errors: list):
    """Body of one host thread: select the device, run the five kernels, bring the results back."""
    import torch

    try:
        lib = hc_lib.load()
        hc_lib.check(lib.hc_set_device(device))
        with torch.cuda.device(device):
            res = {}
            q, k, v = (_upload(a, oracle) for a in x["fa"])
            o, lse = hc_lib.flash_attention_fwd(q, k, v, True)
            res["fa_path"] = lib.hc_flash_attention_last_path()
            grads = hc_lib.flash_attention_bwd(q, k, v, o, lse, _upload(x["do"], oracle), True)[:3]
            res["bwd_path"] = lib.hc_flash_attention_bwd_last_path()
            A, B, bias = (_upload(a, oracle) for a in x["mm"])
            c = hc_lib.matmul_bias(A, B, bias)
            res["mm_path"] = lib.hc_matmul_bias_last_path()
            xl, g, b = x["ln"]
            y = hc_lib.layer_norm(_upload(xl, oracle), _upload(g, oracle, "f32"), _upload(b, oracle, "f32"), 1e-5)
            xr, w, cos, sin = x["rms"]
            r = hc_lib.rms_norm_rope_fused(_upload(xr, oracle), _upload(w, oracle, "f32"), _upload(cos, oracle, "f32"),
                                           _upload(sin, oracle, "f32"), 128, 1e-6, heads=4, rope_style=1)
            t = hc_lib.transpose_2d_4d(_upload(x["tr"], oracle), 0)
            torch.cuda.synchronize(device)
            hc_lib.check(lib.hc_check_device_error())
            cur = torch.cuda.current_device()
            res.update(device=cur, fa=host(o, oracle), lse=lse.cpu().numpy(), mm=host(c, oracle), ln=host(y, oracle),
                       rms=host(r, oracle), tr=bits(t), grads=[host(g_, oracle) for g_ in grads])
            out[device] = res
    except Exception as e:  # noqa: BLE001 -- reported by the main thread
        errors.append((device, repr(e)))


def _check(res, oracle, x):
    assert res["fa_path"] == 1 and res["mm_path"] == 3, "tensor-core paths not taken (M=384 takes the CTA-pair GEMM)"
    assert res["bwd_path"] == 1, "tcgen05 backward not taken"
    qq, kq, vq = (quantize(a, "bf16", oracle) for a in x["fa"])
    ref, ref_lse = oracle.flash_attention_fwd(qq, kq, vq, 1.0 / np.sqrt(128.0), 1)
    assert_close(ref, res["fa"], 2e-2, 0.0, "flash attention")
    assert_close(ref_lse, res["lse"], 2e-3, 0.0, "lse")
    gref = oracle.flash_attention_bwd(qq, kq, vq, quantize(x["do"], "bf16", oracle), 1.0 / np.sqrt(128.0), 1)
    for name, e, g_ in zip(("dq", "dk", "dv"), gref, res["grads"]):
        nw = float(np.linalg.norm(g_.astype(np.float64) - e) / np.linalg.norm(e))
        assert nw <= 1e-2, (name, nw)
    A, B, bias = (quantize(a, "bf16", oracle) for a in x["mm"])
    mref = oracle.matmul_bias(A, B, bias)
    assert float(np.abs(mref - res["mm"]).max() / np.abs(mref).max()) <= 1e-2
    xl, g, b = x["ln"]
    assert_close(oracle.layer_norm(quantize(xl, "bf16", oracle), g, b, 1e-5), res["ln"], 1e-2, 2.0 ** -8, "layer_norm")
    xr, w, cos, sin = x["rms"]
    rref = oracle.rms_norm_rope(quantize(xr, "bf16", oracle), w, cos, sin, 128, 1e-6, heads=4, style=1)
    assert_close(rref, res["rms"], 2e-2, 2.0 ** -8, "rms_norm_rope")
    assert np.array_equal(res["tr"], oracle.to_bf16(np.ascontiguousarray(x["tr"].T)))


def test_one_thread_per_gpu(cuda, hc_lib, oracle):
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs (one host thread per device)")
    x = _inputs(oracle)
    rounds = [[0], [1], [0, 1], [0, 1]]  # device 1 first alone after device 0, then both at once
    for devices in rounds:
        out, errors = {}, []
        threads = [threading.Thread(target=_run_device, args=(dv, hc_lib, oracle, x, out, errors)) for dv in devices]
        for th in threads:
            th.start()
        for th in threads:
            th.join(timeout=600)
        assert not any(th.is_alive() for th in threads), "a device thread did not finish"
        assert not errors, errors
        for dv in devices:
            assert out[dv]["device"] == dv
            _check(out[dv], oracle, x)

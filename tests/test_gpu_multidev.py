"""Several GPUs driven from one process (run with -m gpu; skipped with fewer
than two devices). Kestrel's NativeSession owns every device of a machine in
one process (crates/kestrel-backends/src/lib.rs:125-187), so the library must
work with one context per GPU side by side: kernel attributes are per device,
and the no-allocation router keeps one scratch address per device.

Each context runs a layer against the oracle; the second device's calls come
after the first device's, so a per-device setting made only once per process
would show up as a launch failure on the second device."""
import ctypes

import numpy as np
import pytest

import oracle

from gpu_util import make_layer, oracle_layer, tol_ok, upload

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _need_two():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")


def test_two_contexts_one_process():
    _need_two()
    from kestrel_b200.cuda import Context
    L = make_layer(E=16, k=4, d=2048, ff=768, seed=21)
    ctxs = [Context(0), Context(1)]
    try:
        for c in ctxs:
            upload(c, 0, L)
        for rnd in range(2):
            for dev, c in enumerate(ctxs):
                for n in (1, 3, 16, 40):  # int8 path, tcgen05 path, both
                    h = np.random.default_rng(1000 * rnd + 10 * dev + n).standard_normal((n, L["d"])).astype(
                        np.float32)
                    out, ids, _ = c.moe_ffn(0, h)
                    r_out, r_ids, _ = oracle_layer(oracle, L, h)
                    assert np.array_equal(ids, r_ids), (dev, n)
                    ok, err, scale = tol_ok(out, r_out)
                    assert ok, f"device {dev} n={n}: max err {err} vs scale {scale}"
    finally:
        for c in ctxs:
            c.close()


def test_route_noalloc_on_two_devices():
    _need_two()
    from kestrel_b200 import cuda as kc
    lib = kc.lib()
    E, d, k, n = 128, 2048, 8, 16
    results = []
    for dev in (0, 1, 0):
        with torch.cuda.device(dev):
            g = torch.Generator(device=f"cuda:{dev}").manual_seed(5)
            router = torch.randn((E, d), generator=g, device=f"cuda:{dev}") * 0.02
            h = torch.randn((n, d), generator=g, device=f"cuda:{dev}")
            ids = torch.full((n, k), -7, dtype=torch.int32, device=f"cuda:{dev}")
            w = torch.empty((n, k), device=f"cuda:{dev}")
            stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
            rc = lib.kc_route_noalloc(ctypes.c_void_p(router.data_ptr()), E, d, ctypes.c_void_p(h.data_ptr()), n, k,
                                      1, 0.0, ctypes.c_void_p(ids.data_ptr()), ctypes.c_void_p(w.data_ptr()),
                                      stream)
            assert rc == 0, lib.kc_last_error(None)
            torch.cuda.synchronize(dev)
            logits = oracle.matmul(0, router.cpu().numpy().view(np.uint8), E, d, h.cpu().numpy())  # F32 router
            r_ids, _ = oracle.route(logits, k)
            assert np.array_equal(ids.cpu().numpy(), r_ids), dev
            results.append(ids.cpu().numpy())
    assert np.array_equal(results[0], results[1]) and np.array_equal(results[0], results[2])

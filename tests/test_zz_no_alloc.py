"""kc_route_noalloc: routing for callers that cannot let the library allocate
device memory (a strict memory ledger, a latency-critical thread that cannot
take cudaMalloc's device-wide synchronisation, an embedding with its own
pool). It must give exactly what the allocating entry
points give -- kc_router_logits_dev followed by kc_route_dev -- through the C
ABI, on consecutive calls (its scratch array is shared and reused), and
refuse requests larger than its fixed scratch.

This file is named to be collected last, so a failure here leaves every other
test already run."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def test_route_noalloc_matches_allocating_path():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from kestrel_b200 import cuda as kc

    lib = kc.lib()
    ctx = kc.Context(0)
    ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    g = torch.Generator(device="cuda").manual_seed(11)
    E, d, k = 128, 2048, 8
    try:
        for call, n_tok in enumerate((16, 5)):  # two calls in a row, different shapes
            router = torch.randn((E, d), generator=g, device="cuda") * 0.02
            h = torch.randn((n_tok, d), generator=g, device="cuda")
            # Reference: the allocating entry points (context workspace).
            logits = torch.empty((n_tok, E), device="cuda")
            ref_ids = torch.empty((n_tok, k), dtype=torch.int32, device="cuda")
            ref_w = torch.empty((n_tok, k), device="cuda")
            ctx.router_logits_dev(router, h, logits)
            ctx.route_dev(logits, k, ref_ids, ref_w, norm_topk=True)
            # No-allocation entry point.
            ids = torch.full((n_tok, k), -7, dtype=torch.int32, device="cuda")
            w = torch.full((n_tok, k), float("nan"), device="cuda")
            rc = lib.kc_route_noalloc(_ptr(router), E, d, _ptr(h), n_tok, k, 1, 0.0, _ptr(ids), _ptr(w), stream)
            assert rc == 0, lib.kc_last_error(None)
            torch.cuda.synchronize()
            assert torch.equal(ids, ref_ids), f"call {call}: top-k ids differ"
            assert np.array_equal(w.cpu().numpy().view(np.uint32), ref_w.cpu().numpy().view(np.uint32)), \
                f"call {call}: weights differ"
        # Larger than the fixed scratch: refused with a clear error, nothing launched.
        big = torch.empty((1024, 64), device="cuda")
        rc = lib.kc_route_noalloc(_ptr(torch.empty((128, 64), device="cuda")), 128, 64, _ptr(big), 1024, 8, 1, 0.0,
                                  _ptr(torch.empty((1024, 8), dtype=torch.int32, device="cuda")),
                                  _ptr(torch.empty((1024, 8), device="cuda")), stream)
        assert rc == 2 and b"65536" in lib.kc_last_error(None)
    finally:
        ctx.close()

"""Layer parity at the full shapes of the benchmarked configurations against
the CPU oracle (run with -m gpu), at every batch size the bench reports:

* configs[1] (Qwen3-30B-A3B layer: d=2048, 128 experts, top-8, ff=768) at
  B = 1, 16, 128, 512;
* configs[2] (Mixtral-8x7B layer: d=4096, 8 experts, top-2, ff=14336) at
  B = 1, 3, 8, 512, 2048, 4096;
* configs[4] (Qwen3-235B-A22B layer: d=4096, 128 experts, top-8, ff=1536,
  Zipf-skewed routing) at B = 1, 4, 64, 2048.

The large batches run the tensor-core grouped kernel with its batch-dependent
split-K factors and slot tiles. Every case checks identical top-k ids and the
reference's criterion max|d| <= 1e-3 * max(max|ref|, 1)
(crates/kestrel-engine/tests/oracle.rs:75-78); the elementwise relative error
is printed beside it. Weights: Q4_K gate/up + Q6_K down quantised from
N(0, 0.02) on the GPU with this library's quantizer, copied to the host for
the oracle."""
import os

import numpy as np
import pytest

import oracle

from gpu_util import gpu_layer, layer_input, rel_report, tol_ok

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from kestrel_b200.cuda import Context
    c = Context(0)
    c.set_stream(torch.cuda.current_stream().cuda_stream)
    oracle.set_threads(os.cpu_count() or 1)
    yield c
    c.close()
    oracle.set_threads(1)


def check(ctx, lid, host, n, seed):
    h = layer_input(host, n, seed)
    out, ids, w = ctx.moe_ffn(lid, h)
    r_out, r_ids, r_w = oracle.moe_ffn(h, host["router"], host["k"], 12, host["gate"], 12, host["up"], 14,
                                       host["down"], host["ff"])
    assert np.array_equal(ids, r_ids), f"n={n}: top-k ids differ"
    ok, err, scale = tol_ok(out, r_out)
    med, mx = rel_report(out, r_out)
    print(f"\n  E={host['E']} d={host['d']} ff={host['ff']} n={n}: max|d| {err:.3g} = {err / scale:.3g} of scale "
          f"{scale:.3g}; elementwise rel. error median {med:.3g}, max {mx:.3g}")
    assert ok, f"n={n}: max err {err} vs scale {scale}"
    return ids


def test_config1_full_shape(ctx):
    host = gpu_layer(ctx, 710, 128, 8, 2048, 768, seed=1)
    for n, seed in ((1, 11), (16, 12), (128, 13), (512, 14)):
        check(ctx, 710, host, n, seed)


def test_config2_mixtral_shape(ctx):
    host = gpu_layer(ctx, 700, 8, 2, 4096, 14336, seed=2)
    # n=1, 3: int8 path; n=8 puts >= 4 rows on some experts; 512-4096: prefill.
    for n, seed in ((1, 1), (3, 2), (8, 3), (512, 4), (2048, 5), (4096, 6)):
        check(ctx, 700, host, n, seed)


def test_config4_skewed_routing(ctx):
    E, k = 128, 8
    host = gpu_layer(ctx, 701, E, k, 4096, 1536, seed=4, zipf=True)
    for n, seed in ((1, 1), (4, 2)):
        check(ctx, 701, host, n, seed)
    ids = check(ctx, 701, host, 64, 3)
    cnt = np.sort(np.bincount(ids.reshape(-1), minlength=E))[::-1]
    # The skew shows: the most popular expert gets several times the mean load.
    assert cnt[0] >= 4 * (64 * k / E)
    check(ctx, 701, host, 2048, 7)

"""KC_OPT_F32_PREFILL: products with >= 4 rows in the reference's exact f32
order (dequant_row, then avx2::gemm_f32 on 48-row tiles with its 3-row x
4-token blocking and dot_f32 for the rest, quant.rs:241-260,
avx2.rs:230-308), compared bit for bit with the oracle (run with -m gpu)."""
import numpy as np
import pytest

import oracle
from kestrel_b200 import ggml as G

from gpu_util import bits, make_layer, oracle_layer, upload

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from kestrel_b200.cuda import OPT_F32_PREFILL, Context
    c = Context(0)
    c.set_option(OPT_F32_PREFILL, 1)
    yield c
    c.close()


@pytest.mark.parametrize("t,rows,cols", [(G.Q4_K, 100, 512), (G.Q6_K, 96, 768), (G.Q8_0, 61, 1408)],
                         ids=["Q4_K", "Q6_K", "Q8_0-ragged"])
@pytest.mark.parametrize("n", [4, 7, 13])
def test_dense_f32_path_bit_exact(ctx, t, rows, cols, n):
    rng = np.random.default_rng(rows + n)
    w = G.quantize(t, rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.02))
    x = rng.standard_normal((n, cols)).astype(np.float32)
    tid = 700 + t
    ctx.upload_dense(tid, t, w, rows, cols)
    got = ctx.matmul(tid, x)
    ref = oracle.matmul(t, w, rows, cols, x)
    assert np.array_equal(bits(got), bits(ref)), float(np.abs(got - ref).max())


def test_moe_layer_prefill_exact(ctx):
    """A layer whose experts all get >= 4 rows: the grouped f32 products are
    the reference's bit for bit. SwiGLU's exp is a double-precision exp
    rounded to float against the C library's expf, which differ in the last
    bit for ~0.06% of arguments; so nearly all outputs are identical and the
    rest within a few ulps."""
    L = make_layer(8, 2, 512, 768, seed=31)
    upload(ctx, 960, L)
    h = np.random.default_rng(32).standard_normal((64, 512)).astype(np.float32)
    out, ids, _ = ctx.moe_ffn(960, h)
    r_out, r_ids, _ = oracle_layer(oracle, L, h)
    assert np.array_equal(ids, r_ids)
    same = np.mean(bits(out) == bits(r_out))
    err = float(np.abs(out - r_out).max())
    assert same >= 0.99 and err <= 1e-5 * max(float(np.abs(r_out).max()), 1.0), (same, err)

"""GGUF / KGUF container: this package's writer against the library's parser
(kc_gguf_inspect, no GPU), following kestrel-gguf's reader
(crates/kestrel-gguf/src/lib.rs:196-311) and its rejection of corrupt files."""
import os
import struct

import numpy as np
import pytest

from kestrel_b200 import ggml as G
from kestrel_b200 import gguf, synth
from kestrel_b200.cuda import KestrelCudaError, gguf_inspect

SMALL = dict(synth.CONFIG0, n_layer=2, d=256, n_head=4, n_kv=2, head_dim=64, rope_dim=64, n_vocab=512, ff=256)


@pytest.fixture(scope="module")
def model():
    return synth.make_model(SMALL, seed=11)


@pytest.mark.parametrize("prepared", [False, True], ids=["gguf", "kguf-strided"])
def test_round_trip(tmp_path, model, prepared):
    p = str(tmp_path / "m.gguf")
    gguf.write_model(p, model, prepared=prepared)
    info = gguf_inspect(p)
    c = SMALL
    assert info["version"] == 3 and info["prepared"] is prepared and info["alignment"] == 32
    assert info["arch"] == "qwen3moe"
    for k, v in (("n_layer", 2), ("n_embd", 256), ("n_head", 4), ("n_head_kv", 2), ("head_dim", 64),
                 ("n_vocab", 512), ("rope_dim", 64), ("n_expert", 8), ("n_expert_used", 2), ("n_ff_exp", 256)):
        assert info[k] == v, k
    assert info["norm_topk"] is True and abs(info["rope_base"] - 1e4) < 1e-3 and abs(info["rms_eps"] - 1e-6) < 1e-12
    by = {t["name"]: t for t in info["tensors"]}
    assert len(by) == len(model["tensors"])
    data = open(p, "rb").read()
    for layer, name, t, arr, rows, cols in model["tensors"]:
        full = (name if layer < 0 else f"blk.{layer}.{name}") + ".weight"
        ti = by[full]
        assert ti["type"] == t and ti["dims"][0] == cols
        raw = np.ascontiguousarray(arr).reshape(-1).view(np.uint8).tobytes()
        assert ti["size"] == len(raw) and ti["offset"] % 32 == 0
        if ti["stride"]:
            assert prepared and name.endswith("_exps")
            n_sl = ti["dims"][-1]
            sb = len(raw) // n_sl
            assert ti["stride"] > sb and ti["stride"] % 32 == 0
            got = b"".join(data[ti["offset"] + s * ti["stride"]:ti["offset"] + s * ti["stride"] + sb]
                           for s in range(n_sl))
        else:
            got = data[ti["offset"]:ti["offset"] + ti["size"]]
        assert got == raw, full


def _bad(tmp_path, blob, match):
    p = str(tmp_path / "bad.gguf")
    open(p, "wb").write(blob)
    with pytest.raises(KestrelCudaError) as e:
        gguf_inspect(p)
    assert match in str(e.value)


def test_rejects_corrupt_files(tmp_path, model):
    p = str(tmp_path / "m.gguf")
    gguf.write_model(p, model)
    good = open(p, "rb").read()
    _bad(tmp_path, b"GGML" + good[4:], "bad magic")
    _bad(tmp_path, good[:4] + struct.pack("<I", 7) + good[8:], "version 7")
    _bad(tmp_path, good[: len(good) // 2], "past end of file")
    _bad(tmp_path, good[:40], "end of file")
    # A strided tensor in a plain GGUF file.
    g2 = str(tmp_path / "s.gguf")
    gguf.write_gguf(g2, [("general.architecture", gguf.STRING, "qwen3")],
                    [("x.weight", G.F32, [8, 2], np.zeros(16, np.float32))], strides={"x.weight": 64})
    _bad(tmp_path, open(g2, "rb").read(), "strided in a plain GGUF")


def test_unsupported_arch_is_reported_not_fatal(tmp_path):
    p = str(tmp_path / "a.gguf")
    gguf.write_gguf(p, [("general.architecture", gguf.STRING, "gpt2")],
                    [("token_embd.weight", G.F32, [4, 3], np.zeros(12, np.float32))])
    info = gguf_inspect(p)
    assert "gpt2" in info["model_error"] and info["n_tensors"] == 1

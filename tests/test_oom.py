"""The .oom file scan (OomLoader::load, src/quant.rs:320-367) on the CPU: the
library's oomattn_oom_scan and the oracle's restatement against the golden file
(tests/golden/make_golden_oom.py), its f32 and Q8 tensors, and rejection of
damaged images.  No GPU needed."""
import os

import numpy as np
import pytest

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def image():
    with open(os.path.join(GOLD, "golden.oom"), "rb") as f:
        return f.read()


@pytest.fixture(scope="module")
def meta():
    return np.load(os.path.join(GOLD, "golden_oom_meta.npz"))


def test_scan_matches_the_golden_table(image, meta):
    from oomllama_b200 import oom_scan
    t = oom_scan(image)
    assert list(t) == [str(n) for n in meta["names"]]
    for i, m in enumerate(t.values()):
        for k in ("name_offset", "name_len", "quant_type", "num_blocks", "total_values", "data_offset",
                  "data_bytes"):
            assert getattr(m, k) == int(meta[k][i]), (i, k)


def test_oracle_scan_agrees(image, oracle):
    from oomllama_b200 import oom_scan
    lib = [(k, m.quant_type, m.num_blocks, m.total_values, m.data_offset, m.data_bytes)
           for k, m in oom_scan(image).items()]
    assert oracle.oom_scan(image) == lib


def test_tensor_contents(image, meta, oracle):
    from oomllama_b200 import OomFile, q8_unpack
    g = np.load(os.path.join(GOLD, "golden_q8.npz"))
    f = OomFile(image)
    assert np.array_equal(f.f32_tensor("model.norm.weight").numpy(), meta["norm"])
    for name, key, n in (("model.layers.0.mlp.up_proj.weight", "stream", g["w"].size),
                         ("lm_head.weight", "stream", g["w"].size),
                         ("model.layers.0.self_attn.q_proj.bias", "stream_tail", g["tail"].size)):
        blocks = np.asarray(f.blocks(name))
        assert np.array_equal(blocks, g[key])
        d = oracle.q8_dequantize(blocks, n)
        ref = g["deq"] if key == "stream" else g["deq_tail"]
        assert np.array_equal(d.view(np.uint32), ref.view(np.uint32))
        q, sc, mn = q8_unpack(blocks, n)
        assert q.size == n and sc.size == (n + 255) // 256


@pytest.mark.parametrize("cut", [1, 11, 13, 60, 16100, 16500, 16840])
def test_scan_rejects_truncated_images(image, oracle, cut):
    from oomllama_b200 import oom_scan
    from oomllama_b200._lib import OomAttnError
    img = image[:cut]
    with pytest.raises(OomAttnError):
        oom_scan(img)
    with pytest.raises(ValueError):
        oracle.oom_scan(img)


def test_scan_rejects_bad_magic(image):
    from oomllama_b200 import oom_scan
    from oomllama_b200._lib import OomAttnError
    with pytest.raises(OomAttnError):
        oom_scan(b"GGUF" + image[4:])

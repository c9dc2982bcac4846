"""K-E on the CPU: the oracle's restatement of the .oom Q8 format against the
golden vectors (tests/golden/make_golden_q8.py), and the library's host-side
block-stream unpacker (oomattn_q8_unpack) against both.  No GPU needed."""
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden_q8.npz")


@pytest.fixture(scope="module")
def g():
    return np.load(GOLDEN)


def test_oracle_writer_matches_golden_stream(oracle, g):
    # src/gguf2oom.rs:719-770, byte for byte (scale, min, len, q of every block)
    assert np.array_equal(oracle.q8_quantize(g["w"]), g["stream"])
    assert np.array_equal(oracle.q8_quantize(g["tail"]), g["stream_tail"])


def test_oracle_reader_matches_golden_values(oracle, g):
    # min + (f32)q * scale, separately rounded (src/quant.rs:201-224): bit-exact
    d = oracle.q8_dequantize(g["stream"], g["w"].size)
    assert np.array_equal(d.view(np.uint32), g["deq"].view(np.uint32))
    dt = oracle.q8_dequantize(g["stream_tail"], g["tail"].size)
    assert np.array_equal(dt.view(np.uint32), g["deq_tail"].view(np.uint32))


def test_q8_known_answers(oracle):
    # a constant block has scale 0 and dequantises to its value exactly
    s = oracle.q8_quantize(np.full(256, -0.5, np.float32))
    assert np.frombuffer(s[:4].tobytes(), np.float32)[0] == 0.0
    assert np.all(s[12:] == 0)
    assert np.all(oracle.q8_dequantize(s, 256) == -0.5)
    # the block's min maps to q = 0 and its max to q = 255
    v = np.linspace(-1.0, 1.0, 256, dtype=np.float32)
    s = oracle.q8_quantize(v)
    assert s[12] == 0 and s[12 + 255] == 255
    d = oracle.q8_dequantize(s, 256)
    assert d[0] == -1.0
    scale = np.frombuffer(s[:4].tobytes(), np.float32)[0]
    assert np.abs(d - v).max() <= scale / 2 + 1e-7
    # header layout: [f32 scale][f32 min][u32 len]
    assert np.frombuffer(s[4:8].tobytes(), np.float32)[0] == -1.0
    assert np.frombuffer(s[8:12].tobytes(), np.uint32)[0] == 256


def test_oracle_linear_matches_golden(oracle, g):
    w = oracle.q8_dequantize(g["stream"], g["w"].size).reshape(g["w"].shape)
    y = oracle.linear(g["x"], w, g["b"])
    assert np.abs(y - g["y"]).max() <= 1e-5 * max(1.0, np.abs(g["y"]).max())


def test_unpack_matches_oracle(g, oracle):
    from oomllama_b200 import q8_unpack
    n = g["w"].size
    q, scale, mn = q8_unpack(g["stream"], n)
    blk = np.arange(n) // 256
    d = (mn[blk] + (q.astype(np.float32) * scale[blk]).astype(np.float32)).astype(np.float32)
    assert np.array_equal(d.view(np.uint32), g["deq"].view(np.uint32))
    q2, s2, m2 = q8_unpack(g["stream_tail"], g["tail"].size)
    assert q2.size == 300 and s2.size == 2 and m2.size == 2


@pytest.mark.parametrize("cut", [1, 12, 13, 268])
def test_unpack_rejects_truncated_streams(g, cut):
    from oomllama_b200 import q8_unpack
    from oomllama_b200._lib import OomAttnError
    with pytest.raises(OomAttnError) as e:
        q8_unpack(g["stream"][:-cut], g["w"].size)
    assert e.value.code == 1


def test_unpack_rejects_a_wrong_block_length(g):
    from oomllama_b200 import q8_unpack
    from oomllama_b200._lib import OomAttnError
    s = g["stream"].copy()
    s[8:12] = np.frombuffer(np.uint32(255).tobytes(), np.uint8)  # first block claims 255 values
    with pytest.raises(OomAttnError) as e:
        q8_unpack(s, g["w"].size)
    assert "length" in str(e.value)


def test_oracle_rmsnorm_known_answers(oracle):
    # a constant row c normalises to sign(c) * w (up to eps); a row scaled by k gives the same output
    w = np.linspace(-2, 2, 64).astype(np.float32)
    out = oracle.rmsnorm(np.full((1, 64), 3.0, np.float32), w, 1e-6)[0]
    assert np.allclose(out, w, rtol=1e-6, atol=1e-6)
    x = np.random.default_rng(0).standard_normal((3, 64)).astype(np.float32)
    assert np.allclose(oracle.rmsnorm(x, w, 0.0), oracle.rmsnorm(4.0 * x, w, 0.0), rtol=1e-5, atol=1e-6)
    # float64 restatement of src/oomllama.rs:200-211
    ref = x / np.sqrt((x.astype(np.float64) ** 2).mean(-1, keepdims=True) + 1e-6) * w
    assert np.abs(oracle.rmsnorm(x, w, 1e-6) - ref).max() < 1e-5


def test_oracle_swiglu_known_answers(oracle):
    g = np.array([0.0, 1.0, -1.0, 20.0, -20.0], np.float32)
    u = np.array([5.0, 1.0, 2.0, 0.5, 1.0], np.float32)
    out = oracle.swiglu(g, u)
    ref = g.astype(np.float64) / (1.0 + np.exp(-g.astype(np.float64))) * u
    assert out[0] == 0.0
    assert np.abs(out - ref).max() < 1e-6 * max(1.0, np.abs(ref).max())


def test_oracle_argmax_matches_the_scan(oracle):
    # the vectorised argmax against the literal strict-greater scan from element 0
    rng = np.random.default_rng(5)
    x = rng.integers(-3, 4, (64, 40)).astype(np.float32)  # many ties
    x[rng.random(x.shape) < 0.05] = np.nan
    x[::7, 0] = np.nan
    x[3] = -np.inf
    x[5, 10:] = np.inf
    assert oracle.argmax(x).tolist() == [oracle.argmax_scan(r) for r in x]


def test_oracle_embedding_rows(oracle):
    w = np.random.default_rng(2).standard_normal((37, 96)).astype(np.float32)  # blocks straddle rows
    s = oracle.q8_quantize(w)
    full = oracle.q8_dequantize(s, w.size).reshape(37, 96)
    ids = [36, 0, 5, 5]
    assert np.array_equal(oracle.embedding(s, 37, 96, ids), full[ids])

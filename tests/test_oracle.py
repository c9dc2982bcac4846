"""The C oracle against the golden vectors and known-answer identities (CPU only).

Parity is unpinned (the Rust reference cannot run here); these tests pin the
oracle to the reference's formulas through an independent float64 restatement
(tests/golden/make_golden.py) and to the identities attention and RoPE must
satisfy.
"""
import os

import numpy as np
import pytest

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden.npz")


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD)


def test_softmax_sums_to_one(oracle):
    # the reference's own softmax test (src/oom_inference.rs:430-436), through attention_head:
    # with identical values v = 1 the output is sum(p) * 1
    q = np.random.default_rng(0).standard_normal(128).astype(np.float32)
    k = np.random.default_rng(1).standard_normal((3, 128)).astype(np.float32)
    v = np.ones((3, 128), np.float32)
    out, _ = oracle.attention_head(q, k, v)
    assert abs(out.sum() / 128 - 1.0) < 1e-4


@pytest.mark.parametrize("tag,theta", [("qwen", 1e6), ("llama", 5e5)])
def test_rope_table_vs_golden(oracle, gold, tag, theta):
    pos = gold["rope_pos"]
    c, s = oracle.rope_table(theta, 128, int(pos.max()) + 1)
    np.testing.assert_allclose(c[pos], gold[f"rope_cos_{tag}"], atol=2e-6 * 4096)
    np.testing.assert_allclose(s[pos], gold[f"rope_sin_{tag}"], atol=2e-6 * 4096)
    # small positions: f32 angles are exact to ~1 ulp
    np.testing.assert_allclose(c[pos[:4]], gold[f"rope_cos_{tag}"][:4], atol=2e-6)


@pytest.mark.parametrize("tag,theta", [("qwen", 1e6), ("llama", 5e5)])
@pytest.mark.parametrize("variant", ["inter", "split"])
def test_rope_apply_vs_golden(oracle, gold, tag, theta, variant):
    pos = gold["rope_pos"]
    c, s = oracle.rope_table(theta, 128, int(pos.max()) + 1)
    v = oracle.ROPE_INTERLEAVED if variant == "inter" else oracle.ROPE_SPLIT_HALF
    y = oracle.rope_tokens(gold["rope_x"], pos, c, s, v)
    np.testing.assert_allclose(y, gold[f"rope_{variant}_{tag}"], atol=5e-3, rtol=0)
    np.testing.assert_allclose(y[:4], gold[f"rope_{variant}_{tag}"][:4], atol=2e-5, rtol=0)


def test_rope_position_zero_is_identity(oracle):
    x = np.random.default_rng(2).standard_normal((5, 128)).astype(np.float32)
    c, s = oracle.rope_table(1e6, 128, 1)
    for v in (0, 1):
        np.testing.assert_array_equal(oracle.rope_apply(x, c[0], s[0], v), x)


def test_rope_preserves_pair_norms(oracle):
    x = np.random.default_rng(3).standard_normal((4, 128)).astype(np.float32)
    c, s = oracle.rope_table(5e5, 128, 40000)
    for p in (1, 513, 32767, 39999):
        for v in (0, 1):
            y = oracle.rope_apply(x, c[p], s[p], v)
            if v == 1:
                nx = x[:, 0::2] ** 2 + x[:, 1::2] ** 2
                ny = y[:, 0::2] ** 2 + y[:, 1::2] ** 2
            else:
                nx = x[:, :64] ** 2 + x[:, 64:] ** 2
                ny = y[:, :64] ** 2 + y[:, 64:] ** 2
            np.testing.assert_allclose(ny, nx, rtol=1e-5, atol=1e-6)


def test_interleaved_equals_split_half_under_permutation(oracle):
    # interleaved pairs (2i, 2i+1) == split-half pairs (i, i+64) after permuting 2i->i, 2i+1->i+64
    x = np.random.default_rng(4).standard_normal((3, 128)).astype(np.float32)
    perm = np.empty(128, np.int64)
    perm[0::2] = np.arange(64)
    perm[1::2] = np.arange(64) + 64
    c, s = oracle.rope_table(1e6, 128, 800)
    xs = np.empty_like(x)
    xs[:, perm] = x
    yi = oracle.rope_apply(x, c[777], s[777], oracle.ROPE_INTERLEAVED)
    ys = oracle.rope_apply(xs, c[777], s[777], oracle.ROPE_SPLIT_HALF)
    np.testing.assert_array_equal(ys[:, perm], yi)


def test_attention_head_vs_golden(oracle, gold):
    out, lse = oracle.attention_head(gold["head_q"], gold["head_k"], gold["head_v"])
    np.testing.assert_allclose(out, gold["head_out"], atol=2e-6)
    assert abs(lse - float(gold["head_lse"])) < 1e-5


def test_gqa_causal_vs_golden(oracle, gold):
    out, lse = oracle.gqa_attention(gold["gqa_q"], gold["gqa_k"], gold["gqa_v"], causal=True, with_lse=True)
    np.testing.assert_allclose(out, gold["gqa_out"], atol=3e-6)
    np.testing.assert_allclose(lse, gold["gqa_lse"], atol=3e-5)


def test_layer_attention_vs_golden(oracle, gold):
    g = {k[6:]: gold[k] for k in gold.files if k.startswith("layer_")}
    c, s = oracle.rope_table(1e6, 128, 64)
    out, kn, vn = oracle.layer_attention(g["x"], g["wq"], g["wk"], g["wv"], g["bq"], g["bk"], g["bv"], 4, 2,
                                         g["kc"], g["vc"], c, s, oracle.ROPE_INTERLEAVED)
    np.testing.assert_allclose(out, g["out"], atol=2e-5)
    np.testing.assert_array_equal(kn[:, :, :21], g["kc"])


def test_merge_vs_golden(oracle, gold):
    out, lse = oracle.merge_partials(gold["merge_parts"], gold["merge_lses"])
    np.testing.assert_allclose(out, gold["merge_out"], atol=2e-6)
    np.testing.assert_allclose(lse, gold["merge_lse"], atol=2e-6)


def test_single_key_returns_v(oracle):
    rng = np.random.default_rng(5)
    q, k, v = (rng.standard_normal((1, 128)).astype(np.float32) for _ in range(3))
    out, lse = oracle.attention_head(q[0], k, v)
    np.testing.assert_array_equal(out, v[0])


def test_identical_keys_average_v(oracle):
    rng = np.random.default_rng(6)
    q = rng.standard_normal(128).astype(np.float32)
    k = np.repeat(rng.standard_normal((1, 128)).astype(np.float32), 10, 0)
    v = rng.standard_normal((10, 128)).astype(np.float32)
    out, _ = oracle.attention_head(q, k, v)
    np.testing.assert_allclose(out, v.mean(0), atol=1e-6)


def test_causal_first_row_sees_only_first_key(oracle):
    rng = np.random.default_rng(7)
    q = rng.standard_normal((6, 4, 128)).astype(np.float32)
    k = rng.standard_normal((1, 6, 128)).astype(np.float32)
    v = rng.standard_normal((1, 6, 128)).astype(np.float32)
    out = oracle.gqa_attention(q, k, v, causal=True)
    for h in range(4):
        np.testing.assert_array_equal(out[0, h], v[0, 0])


def test_gqa_grouping_repeat_interleave(oracle):
    # q head h reads kv head h // 7 (src/oomllama_turbo.rs:313-316): mark kv head 2 with V = 5
    rng = np.random.default_rng(8)
    q = rng.standard_normal((1, 28, 128)).astype(np.float32)
    k = rng.standard_normal((4, 9, 128)).astype(np.float32)
    v = np.zeros((4, 9, 128), np.float32)
    v[2] = 5.0
    out = oracle.gqa_attention(q, k, v, causal=False)
    for h in range(28):
        np.testing.assert_allclose(out[0, h], 5.0 if h // 7 == 2 else 0.0, atol=2e-6)


def test_split_context_merge_equals_unsplit(oracle):
    rng = np.random.default_rng(9)
    q = rng.standard_normal((1, 7, 128)).astype(np.float32)
    k = rng.standard_normal((1, 300, 128)).astype(np.float32)
    v = rng.standard_normal((1, 300, 128)).astype(np.float32)
    full, lse_full = oracle.gqa_attention(q, k, v, causal=False, with_lse=True)
    parts, lses = [], []
    for a, b in ((0, 100), (100, 250), (250, 300)):
        o, l = oracle.gqa_attention(q, k[:, a:b], v[:, a:b], causal=False, with_lse=True)
        parts.append(o[0])
        lses.append(l[0])
    out, lse = oracle.merge_partials(np.stack(parts), np.stack(lses))
    np.testing.assert_allclose(out, full[0], atol=2e-6)
    np.testing.assert_allclose(lse, lse_full[0], atol=2e-6)


def test_decode_batch_threads_agree(oracle):
    rng = np.random.default_rng(10)
    Ls = [5, 33, 128]
    q = rng.standard_normal((3, 8, 128)).astype(np.float32)
    ks = [rng.standard_normal((2, L, 128)).astype(np.float32) for L in Ls]
    vs = [rng.standard_normal((2, L, 128)).astype(np.float32) for L in Ls]
    a = oracle.decode_batch(q, ks, vs, n_threads=1)
    b = oracle.decode_batch(q, ks, vs, n_threads=4)
    np.testing.assert_array_equal(a, b)
    for i in range(3):
        np.testing.assert_array_equal(a[i], oracle.gqa_attention(q[i:i + 1], ks[i], vs[i], causal=False)[0])


def test_bf16_rounding(oracle):
    x = np.array([1.0, 1.00390625, 1.005859375, -3.1415927, 65504.0, 1e-40, np.inf, -np.inf], np.float32)
    bits = oracle.f32_to_bf16_bits(x)
    back = oracle.bf16_bits_to_f32(bits)
    np.testing.assert_array_equal(back, oracle.round_bf16(x))
    assert back[0] == 1.0 and back[1] == 1.0  # tie rounds to even
    assert back[2] == np.float32(1.0078125)
    assert np.isinf(back[6]) and np.isinf(back[7])
    assert np.isnan(oracle.bf16_bits_to_f32(oracle.f32_to_bf16_bits(np.array([np.nan], np.float32))))[0]

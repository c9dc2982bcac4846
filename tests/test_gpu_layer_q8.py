"""The layer steps around attention on resident Q8 weights, against the oracle:
RMSNorm (src/oomllama.rs:200-211), the gated MLP with its residual add
(src/oomllama.rs:230-242, :401) and the whole decode step of a decoder layer
(GhostDecoderLayer::forward_turbo, src/oomllama.rs:387-402) composed from the
oracle's RMSNorm, Q8 dequantise + matvec, RoPE, GQA attention and SwiGLU.
f32 KV: max-abs <= 1e-4 (scaled by the output's magnitude where it exceeds 1);
bf16 KV: the bf16 tolerance."""
import numpy as np
import pytest
import torch

from helpers import BF16_ATOL, BF16_RTOL, F32_ATOL, assert_close, make_engine

pytestmark = pytest.mark.gpu


def _q8(oracle, rows, cols, rng, scale=0.05):
    from oomllama_b200 import Q8Matrix
    w = (rng.standard_normal((rows, cols)) * scale).astype(np.float32)
    stream = oracle.q8_quantize(w)
    return Q8Matrix.from_oom_stream(stream, rows, cols, device=0), oracle.q8_dequantize(stream, rows * cols).reshape(
        rows, cols)


def test_rmsnorm(oracle):
    eng = make_engine(2, 1, [16])
    rng = np.random.default_rng(1)
    for T, H in [(1, 3584), (5, 256), (16, 4096)]:
        x = (rng.standard_normal((T, H)) * 3).astype(np.float32)
        w = rng.standard_normal(H).astype(np.float32)
        out = eng.rmsnorm(torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda(), 1e-6)
        eng.sync()
        assert_close(out.cpu().numpy(), oracle.rmsnorm(x, w, 1e-6), F32_ATOL, what=f"rmsnorm {T}x{H}")
    eng.close()


@pytest.mark.parametrize("T,H,inter", [(1, 256, 512), (3, 512, 1408), (9, 256, 640), (12, 2048, 8192),
                                         (10, 1024, 20480), (5, 2048, 8192)])
def test_q8_mlp_with_residual(oracle, T, H, inter):
    # (12, 2048, 8192), (10, 1024, 20480) and (5, 2048, 8192): gate+up runs as
    # one launch of the shared-memory-x form over both matrices' row groups,
    # with one and with two row tiles per warp, and with one token tile
    eng = make_engine(2, 1, [16])
    rng = np.random.default_rng(T + H)
    gate, gd = _q8(oracle, inter, H, rng)
    up, ud = _q8(oracle, inter, H, rng)
    down, dd = _q8(oracle, H, inter, rng)
    x = rng.standard_normal((T, H)).astype(np.float32)
    res = rng.standard_normal((T, H)).astype(np.float32)
    y = eng.q8_mlp(gate, up, down, torch.from_numpy(x).cuda(), torch.from_numpy(res).cuda())
    eng.sync()
    ref = oracle.linear(oracle.swiglu(oracle.linear(x, gd), oracle.linear(x, ud)), dd) + res
    assert_close(y.cpu().numpy(), ref, F32_ATOL * max(1.0, np.abs(ref).max()), what=f"q8 mlp T={T}")
    eng.close()


def _layer_case(oracle, kv_dtype, variant, theta, lens, seed, hq=2, hkv=1, inter=512):
    from oomllama_b200 import Q8DecoderLayer
    D, eps = 128, 1e-6
    H = hq * D
    B = len(lens)
    rng = np.random.default_rng(seed)
    mats = {}
    for name, (r, c) in {"q": (hq * D, H), "k": (hkv * D, H), "v": (hkv * D, H), "o": (H, hq * D),
                         "gate": (inter, H), "up": (inter, H), "down": (H, inter)}.items():
        mats[name] = _q8(oracle, r, c, rng)
    bq, bk, bv = [(rng.standard_normal(n) * 0.1).astype(np.float32) for n in (hq * D, hkv * D, hkv * D)]
    n1, n2 = (1 + 0.1 * rng.standard_normal((2, H))).astype(np.float32)
    eng = make_engine(hq, hkv, [L + 1 for L in lens], kv_dtype=kv_dtype, variant=variant, theta=theta, hidden=H,
                      shuffle_seed=seed)
    # cached tokens (already rotated), written through the public cache API
    kc = [(rng.standard_normal((L, hkv, D))).astype(np.float32) for L in lens]
    vc = [(rng.standard_normal((L, hkv, D))).astype(np.float32) for L in lens]
    for b in range(B):
        eng.kv_write(0, b, torch.from_numpy(kc[b]).cuda(), torch.from_numpy(vc[b]).cuda())
    dev = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    w = Q8DecoderLayer(q=mats["q"][0], k=mats["k"][0], v=mats["v"][0], o=mats["o"][0], gate=mats["gate"][0],
                       up=mats["up"][0], down=mats["down"][0], input_norm=dev(n1), post_norm=dev(n2), eps=eps,
                       bq=dev(bq), bk=dev(bk), bv=dev(bv))
    x = rng.standard_normal((B, H)).astype(np.float32)
    out = eng.decoder_layer_q8(0, list(range(B)), dev(x), w)
    eng.sync()
    lens_after = [eng.seq_len(0, b) for b in range(B)]
    eng.close()
    # the oracle's decode step
    var = oracle.ROPE_INTERLEAVED if variant == "interleaved" else oracle.ROPE_SPLIT_HALF
    cos_t, sin_t = oracle.rope_table(theta, D, max(lens) + 1)
    wd = {name: m[1] for name, m in mats.items()}
    wd.update(bq=bq, bk=bk, bv=bv, n1=n1, n2=n2, eps=eps)
    ref = oracle.decoder_layer_decode(x, wd, kc, vc, lens, hq, hkv, cos_t, sin_t, var, kv_dtype == "bf16")
    return out.cpu().numpy(), ref, lens_after


def test_decoder_layer_q8_f32_cache(oracle):
    out, ref, lens_after = _layer_case(oracle, "f32", "interleaved", 1e6, [5, 17, 40], seed=3)
    assert lens_after == [6, 18, 41]
    assert_close(out, ref, F32_ATOL * max(1.0, np.abs(ref).max()), what="decoder layer f32 KV")


def test_decoder_layer_q8_bf16_cache_split_half(oracle):
    out, ref, _ = _layer_case(oracle, "bf16", "split_half", 5e5, [1, 33, 200, 64], seed=4)
    assert_close(out, ref, BF16_ATOL * max(1.0, np.abs(ref).max()), BF16_RTOL, what="decoder layer bf16 KV")


def test_decoder_layer_q8_qkv_on_tensor_cores(oracle):
    # 40 q / 8 kv heads over hidden 5120 for 12 sequences: q, k and v (36.7 M weights) run as ONE
    # tensor-core pass over the three matrices (their row tiles in one persistent grid, tiles cut
    # between CTAs merged in order) with the RMSNorm folded into the digit split and the biases in
    # the epilogue; against the composed oracle
    lens = [3, 40, 77, 16, 100, 5, 9, 64, 31, 2, 18, 50]
    out, ref, lens_after = _layer_case(oracle, "bf16", "interleaved", 1e6, lens, seed=6, hq=40, hkv=8, inter=512)
    assert lens_after == [L + 1 for L in lens]
    assert_close(out, ref, BF16_ATOL * max(1.0, np.abs(ref).max()), BF16_RTOL, what="decoder layer, q/k/v on tcgen05")

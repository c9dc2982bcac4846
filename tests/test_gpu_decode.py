"""K-B / K-B2 parity: split-KV GQA decode over the paged cache vs the oracle
(oom_inference.rs:240-272 per (sequence, q head), GQA grouping
oomllama_turbo.rs:313-316).  Calls go through the C ABI."""
import numpy as np
import pytest
import torch

from helpers import BF16_ATOL, BF16_RTOL, F32_ATOL, as_f32_np, assert_close, make_engine, randn

pytestmark = pytest.mark.gpu


def _run_decode(oracle, n_heads, n_kv, lens, kv_dtype, seed=0, with_lse=False):
    eng = make_engine(n_heads, n_kv, lens, kv_dtype=kv_dtype, shuffle_seed=seed)
    dt = torch.bfloat16 if kv_dtype == "bf16" else torch.float32
    ks, vs = [], []
    for s, L in enumerate(lens):
        k = randn((L, n_kv, 128), seed * 1000 + 2 * s, dt)
        v = randn((L, n_kv, 128), seed * 1000 + 2 * s + 1, dt)
        if L:
            eng.kv_write(0, s, k.cuda(), v.cuda())
        ks.append(as_f32_np(k).transpose(1, 0, 2).copy())
        vs.append(as_f32_np(v).transpose(1, 0, 2).copy())
    q = randn((len(lens), n_heads, 128), seed + 77)
    res = eng.decode(0, list(range(len(lens))), q.cuda(), with_lse=with_lse)
    eng.sync()
    outs, lses = [], []
    for s in range(len(lens)):
        if lens[s] == 0:
            outs.append(np.zeros((n_heads, 128), np.float32))
            lses.append(np.full(n_heads, -np.inf, np.float32))
            continue
        o, l = oracle.gqa_attention(as_f32_np(q[s:s + 1]), ks[s], vs[s], causal=False, with_lse=True)
        outs.append(o[0])
        lses.append(l[0])
    eng.close()
    return res, np.stack(outs), np.stack(lses)


def test_decode_f32_qwen_513(oracle):
    # single-layer Qwen2.5-7B decode shape: 28q/4kv, 512 cached + 1 new, f32 cache
    out, ref, _ = _run_decode(oracle, 28, 4, [513], "f32", seed=1)
    assert_close(out.cpu().numpy(), ref, F32_ATOL, what="f32 decode 513")


@pytest.mark.parametrize("lens", [[1], [16], [17], [31, 2, 100], [4096]])
def test_decode_f32_edges(oracle, lens):
    out, ref, _ = _run_decode(oracle, 28, 4, lens, "f32", seed=2)
    assert_close(out.cpu().numpy(), ref, F32_ATOL, what=f"f32 decode {lens}")


@pytest.mark.parametrize("lens", [[1], [15], [16], [17], [513], [1000, 1, 37, 4097]])
def test_decode_bf16_edges(oracle, lens):
    out, ref, _ = _run_decode(oracle, 28, 4, lens, "bf16", seed=3)
    assert_close(out.cpu().numpy(), ref, BF16_ATOL, BF16_RTOL, what=f"bf16 decode {lens}")


def test_decode_bf16_batched_shuffled_pages(oracle):
    # batched decode, shuffled 16-token pages, varied lengths (scaled-down batch of 64 x U[1024, 8192])
    rng = np.random.default_rng(4)
    lens = rng.integers(1024, 8193, size=12).tolist()
    out, ref, _ = _run_decode(oracle, 28, 4, lens, "bf16", seed=4)
    assert_close(out.cpu().numpy(), ref, BF16_ATOL, BF16_RTOL, what="bf16 batched decode")


def test_decode_bf16_llama_long_context(oracle):
    # Llama-3-8B shape 32q/8kv at 32768 context (2 sequences: exercises the split-KV merge)
    out, ref, _ = _run_decode(oracle, 32, 8, [32768, 20000], "bf16", seed=5)
    assert_close(out.cpu().numpy(), ref, BF16_ATOL, BF16_RTOL, what="bf16 llama 32k decode")


def test_decode_lse_and_empty_row(oracle):
    (out, lse), ref, ref_lse = _run_decode(oracle, 8, 1, [0, 300], "bf16", seed=6, with_lse=True)
    out, lse = out.cpu().numpy(), lse.cpu().numpy()
    assert (out[0] == 0).all() and np.isneginf(lse[0]).all()
    assert_close(out[1], ref[1], BF16_ATOL, BF16_RTOL, what="bf16 decode row 1")
    assert_close(lse[1], ref_lse[1], 1e-3, what="lse")


@pytest.mark.parametrize("kv_dtype", ["bf16", "f32"])
def test_decode_ragged_rows_longest_first(oracle, kv_dtype):
    # rows of very different lengths, empty ones among them: the work items are
    # reordered longest first and each row's pages split into near-equal ranges
    lens = [0, 5000, 17, 1, 0, 800, 3000, 16, 33, 12000, 2]
    (out, lse), ref, ref_lse = _run_decode(oracle, 28, 4, lens, kv_dtype, seed=8, with_lse=True)
    out, lse = out.cpu().numpy(), lse.cpu().numpy()
    tol = (BF16_ATOL, BF16_RTOL) if kv_dtype == "bf16" else (F32_ATOL, None)
    for r, L in enumerate(lens):
        if L == 0:
            assert (out[r] == 0).all() and np.isneginf(lse[r]).all()
        else:
            assert_close(out[r], ref[r], *tol, what=f"{kv_dtype} ragged row {r} (len {L})")
            assert_close(lse[r], ref_lse[r], 1e-3, what=f"lse row {r}")


def test_decode_gqa_marker():
    # q head h must read kv head h // group: V of kv head 2 is 5, others 0
    eng = make_engine(28, 4, [40], kv_dtype="bf16")
    k = randn((40, 4, 128), 9, torch.bfloat16)
    v = torch.zeros(40, 4, 128, dtype=torch.bfloat16)
    v[:, 2] = 5.0
    eng.kv_write(0, 0, k.cuda(), v.cuda())
    out = eng.decode(0, [0], randn((1, 28, 128), 10).cuda()).cpu().numpy()
    eng.sync()
    for h in range(28):
        np.testing.assert_allclose(out[0, h], 5.0 if h // 7 == 2 else 0.0, atol=1e-5)
    eng.close()


def test_merge_partials_vs_oracle(oracle):
    from oomllama_b200 import TurboConfig, TurboEngine
    eng = TurboEngine(TurboConfig(n_layers=1, hidden_size=0, n_heads=8, n_kv_heads=1, max_seq_len=16,
                                  kv_dtype="bf16"))
    parts = randn((3, 40, 128), 11)
    lses = randn((3, 40), 12, scale=3.0)
    lses[1, 5] = float("-inf")
    lses[:, 7] = float("-inf")
    out, lse = eng.merge_partials(parts.cuda(), lses.cuda())
    eng.sync()
    ro, rl = oracle.merge_partials(parts.numpy(), lses.numpy())
    np.testing.assert_allclose(out.cpu().numpy(), ro, atol=1e-5)
    np.testing.assert_allclose(lse.cpu().numpy(), rl, atol=1e-5)
    eng.close()


def test_decode_out_of_range_rejected_on_host():
    from oomllama_b200._lib import OomAttnError
    eng = make_engine(28, 4, [32])
    with pytest.raises(OomAttnError) as e:
        eng.decode(0, [0], torch.zeros(1, 28, 128, device="cuda"), lens=[33])
    assert e.value.code == 3
    with pytest.raises(OomAttnError):
        eng.decode(0, [5], torch.zeros(1, 28, 128, device="cuda"))
    eng.close()

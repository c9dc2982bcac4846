"""K-C parity: the tcgen05/TMEM causal prefill vs the oracle
(flash_attention_forward with causal=true, oomllama_turbo.rs:304-369; mask
aligned to the end of the cache).  Q is bf16 after RoPE by contract, the
cache is bf16; the oracle sees the same bf16 values."""
import numpy as np
import pytest
import torch

from helpers import BF16_ATOL, BF16_RTOL, as_f32_np, assert_close, make_engine, randn

pytestmark = pytest.mark.gpu


def _prefill_case(oracle, n_heads, n_kv, prefix, n_new, seed, rows=None, out_dtype=torch.float32):
    L = prefix + n_new
    eng = make_engine(n_heads, n_kv, [L], kv_dtype="bf16", shuffle_seed=seed)
    k = randn((L, n_kv, 128), seed + 1, torch.bfloat16)
    v = randn((L, n_kv, 128), seed + 2, torch.bfloat16)
    eng.kv_write(0, 0, k.cuda(), v.cuda())
    q = randn((n_new, n_heads, 128), seed + 3, torch.bfloat16)
    out, lse = eng.prefill(0, 0, q.cuda(), out_dtype=out_dtype, with_lse=True)
    eng.sync()
    kf = as_f32_np(k).transpose(1, 0, 2).copy()
    vf = as_f32_np(v).transpose(1, 0, 2).copy()
    qf = as_f32_np(q)
    out = as_f32_np(out)
    if rows is None:
        ref, ref_lse = oracle.gqa_attention(qf, kf, vf, causal=True, with_lse=True)
        eng.close()
        return out, ref, lse.cpu().numpy(), ref_lse
    r, h = rows
    ref = oracle.gqa_attention_rows(qf, kf, vf, r, h, causal=True)
    eng.close()
    return out[r, h], ref, None, None


@pytest.mark.parametrize("n_new", [1, 100, 128, 129, 256, 300, 512])
def test_prefill_small(oracle, n_new):
    out, ref, lse, ref_lse = _prefill_case(oracle, 28, 4, 0, n_new, seed=n_new)
    assert_close(out, ref, BF16_ATOL, BF16_RTOL, what=f"prefill n={n_new}")
    assert_close(lse, ref_lse, 2e-3, what="prefill lse")


@pytest.mark.parametrize("prefix,n_new", [(16, 100), (200, 300), (1000, 257)])
def test_prefill_chunk_on_cached_prefix(oracle, prefix, n_new):
    out, ref, lse, ref_lse = _prefill_case(oracle, 28, 4, prefix, n_new, seed=prefix)
    assert_close(out, ref, BF16_ATOL, BF16_RTOL, what=f"chunked prefill P={prefix} n={n_new}")


def test_prefill_llama_heads_bf16_out(oracle):
    out, ref, _, _ = _prefill_case(oracle, 32, 8, 0, 384, seed=5, out_dtype=torch.bfloat16)
    # a bf16 output adds one rounding to nearest: at most 2^-8 of |out| (unit roundoff of an 8-bit significand)
    excess = np.abs(out - ref) - (BF16_ATOL + np.abs(ref) * 2.0 ** -8)
    assert excess.max() <= 0, f"bf16-out prefill exceeds tolerance by {excess.max():.2e}"
    assert_close(out, ref, 1.0, BF16_RTOL, what="prefill 32q/8kv bf16 out (norm-relative)")


def test_prefill_full_size_sampled_rows(oracle):
    # Qwen2.5-7B causal prefill at 4096 tokens; oracle on 384 sampled (row, head) pairs
    rng = np.random.default_rng(6)
    rows = np.concatenate([[0, 1, 127, 128, 255, 256, 4095], rng.integers(0, 4096, 377)]).astype(np.int32)
    heads = rng.integers(0, 28, rows.size).astype(np.int32)
    out, ref, _, _ = _prefill_case(oracle, 28, 4, 0, 4096, seed=7, rows=(rows, heads))
    assert_close(out, ref, BF16_ATOL, BF16_RTOL, what="prefill 4096 sampled rows")


def test_prefill_reports_v_outside_fp16_range():
    # P.V runs in fp16; a cached V of magnitude >= 65536 has no fp16 image and
    # must surface as a device-check error, not as a silent inf.
    from oomllama_b200._lib import OomAttnError
    eng = make_engine(28, 4, [128], kv_dtype="bf16")
    k = randn((128, 4, 128), 1, torch.bfloat16)
    v = randn((128, 4, 128), 2, torch.bfloat16)
    v[5, 1, 7] = 70000.0
    eng.kv_write(0, 0, k.cuda(), v.cuda())
    eng.prefill(0, 0, randn((128, 28, 128), 3, torch.bfloat16).cuda())
    with pytest.raises(OomAttnError) as e:
        eng.sync()
    assert e.value.code == 9
    eng.sync()  # the status word is cleared after it is reported
    eng.close()


def test_prefill_rejects_f32_cache():
    from oomllama_b200._lib import OomAttnError
    eng = make_engine(28, 4, [32], kv_dtype="f32")
    eng.kv_write(0, 0, torch.zeros(8, 4, 128, device="cuda"), torch.zeros(8, 4, 128, device="cuda"))
    with pytest.raises(OomAttnError) as e:
        eng.prefill(0, 0, torch.zeros(8, 28, 128, dtype=torch.bfloat16, device="cuda"))
    assert e.value.code == 8
    eng.close()


@pytest.mark.parametrize("prefix,n_new", [(0, 700), (300, 513)])
def test_prefill_growing_scores_rescales_o(oracle, prefix, n_new):
    # Keys grow in magnitude along the sequence, so a row's running maximum
    # climbs by far more than 2^8 across its key tiles and the lazy O rescale
    # runs in most steps (both key halves of a row must agree on it).
    L = prefix + n_new
    eng = make_engine(8, 1, [L], kv_dtype="bf16", shuffle_seed=11)
    growth = torch.linspace(1.0, 24.0, L).reshape(L, 1, 1)
    k = (randn((L, 1, 128), 12, torch.float32) * growth).to(torch.bfloat16)
    v = randn((L, 1, 128), 13, torch.bfloat16)
    eng.kv_write(0, 0, k.cuda(), v.cuda())
    q = randn((n_new, 8, 128), 14, torch.bfloat16)
    out, lse = eng.prefill(0, 0, q.cuda(), with_lse=True)
    eng.sync()
    ref, ref_lse = oracle.gqa_attention(as_f32_np(q), as_f32_np(k).transpose(1, 0, 2).copy(),
                                        as_f32_np(v).transpose(1, 0, 2).copy(), causal=True, with_lse=True)
    eng.close()
    assert_close(as_f32_np(out), ref, BF16_ATOL, BF16_RTOL, what=f"growing-score prefill P={prefix} n={n_new}")
    assert_close(lse.cpu().numpy(), ref_lse, 2e-3 * 24, BF16_RTOL, what="growing-score prefill lse")


def test_prefill_query_block_ranges_match_whole_launch():
    # the sharded prefill's per-rank launch: only the blocks of its ranges are written, and they match
    # the whole launch's rows (a launch of few blocks may cut the heaviest blocks' keys into chunks
    # merged by their lse, so the match is to the bf16 tolerance rather than bit for bit)
    from oomllama_b200.shard import PrefillShardPlan
    n_new = 2000  # 8 blocks, the last one ragged
    eng = make_engine(28, 4, [n_new], kv_dtype="bf16", shuffle_seed=3)
    k = randn((n_new, 4, 128), 31, torch.bfloat16)
    v = randn((n_new, 4, 128), 32, torch.bfloat16)
    eng.kv_write(0, 0, k.cuda(), v.cuda())
    q = randn((n_new, 28, 128), 33, torch.bfloat16).cuda()
    full, full_lse = eng.prefill(0, 0, q, with_lse=True)
    for plan in (PrefillShardPlan(28, 4, 8, 0), PrefillShardPlan(28, 4, 8, 1), PrefillShardPlan(28, 4, 4, 0)):
        blocks = plan.blocks(n_new)
        part = torch.full_like(full, float("nan"))
        part, lse = eng.prefill(0, 0, q, out=part, with_lse=True, blocks=blocks)
        eng.sync()
        rows = torch.zeros(n_new, dtype=torch.bool)
        for lo, hi in blocks:
            rows[256 * lo:min(n_new, 256 * hi)] = True
        rows = rows.cuda()
        assert_close(part[rows].cpu().numpy(), full[rows].cpu().numpy(), BF16_ATOL, BF16_RTOL, what=f"{blocks}")
        assert_close(lse[rows].cpu().numpy(), full_lse[rows].cpu().numpy(), 1e-3, what=f"lse {blocks}")
        assert torch.isnan(part[~rows]).all()
    # every block covered once by the two zig-zag ranks of a kv head
    cover = np.zeros(8, int)
    for r in range(2):
        for lo, hi in PrefillShardPlan(28, 4, 8, r).blocks(n_new):
            cover[lo:hi] += 1
    assert (cover == 1).all()
    from oomllama_b200._lib import OomAttnError
    with pytest.raises(OomAttnError):
        eng.prefill(0, 0, q, blocks=[(0, 9)])  # past the last block
    with pytest.raises(OomAttnError):
        eng.prefill(0, 0, q, blocks=[(0, 4), (3, 6)])  # overlapping
    eng.close()


@pytest.mark.parametrize("prefix,n_new,out_dtype", [(0, 4096, torch.float32), (700, 3000, torch.float32),
                                                    (0, 2500, torch.bfloat16)])
def test_prefill_key_split_few_heads(oracle, prefix, n_new, out_dtype):
    # a launch with few heads (a sharded rank's share): the heaviest query blocks would set the launch
    # time, so their key range is cut into chunks whose partials are merged; rows of blocks with few
    # keys are written directly -- every row checked against the oracle on sampled (row, head) pairs
    n_heads, n_kv = 4, 1
    L = prefix + n_new
    eng = make_engine(n_heads, n_kv, [L], kv_dtype="bf16", shuffle_seed=21)
    k = randn((L, n_kv, 128), 41, torch.bfloat16)
    v = randn((L, n_kv, 128), 42, torch.bfloat16)
    eng.kv_write(0, 0, k.cuda(), v.cuda())
    q = randn((n_new, n_heads, 128), 43, torch.bfloat16)
    out, lse = eng.prefill(0, 0, q.cuda(), out_dtype=out_dtype, with_lse=True)
    eng.sync()
    kf, vf = as_f32_np(k).transpose(1, 0, 2).copy(), as_f32_np(v).transpose(1, 0, 2).copy()
    qf = as_f32_np(q)
    rng = np.random.default_rng(n_new)
    rows = np.concatenate([rng.integers(0, n_new, 200), [0, n_new - 1, n_new - 129]]).astype(np.int32)
    heads = rng.integers(0, n_heads, rows.size).astype(np.int32)
    # the oracle's rows are positions prefix + row of a causal prefill over the whole cache
    qfull = np.zeros((L, n_heads, 128), np.float32)
    qfull[prefix:] = qf
    ref = oracle.gqa_attention_rows(qfull, kf, vf, rows + prefix, heads, causal=True)
    got = as_f32_np(out)[rows, heads]
    if out_dtype == torch.bfloat16:
        assert np.abs(got - ref).max() <= BF16_ATOL + 2.0 ** -8 * np.abs(ref).max()
    else:
        assert_close(got, ref, BF16_ATOL, BF16_RTOL, what=f"key-split prefill P={prefix} n={n_new}")
    assert np.isfinite(lse.cpu().numpy()).all()
    eng.close()

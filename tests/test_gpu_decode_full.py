"""Full-size decode parity against the oracle: the batched Qwen2.5-7B decode (64 sequences, cached
lengths U{1024..8192}, shuffled 16-token pages, interleaved RoPE theta=1e6) and the Llama-3-8B long
context (8 x 32768, 32q/8kv, split-half RoPE theta=5e5), each as one step of the reference's order --
the new token's K-A append (bias + RoPE + paged append, src/oomllama_turbo.rs:647-681), then the
split-KV decode over the whole context (src/oomllama_turbo.rs:680-695, attention per (sequence, q head)
as src/oom_inference.rs:240-272, GQA grouping src/oomllama_turbo.rs:313-316).  Every q head of a
seeded sample of rows is compared; the rotated q and the appended K/V are checked bit for bit.
Also: the packed (O, lse) decode equals the unpacked one, and the packed merge equals the merge of
separate arrays."""
import numpy as np
import pytest
import torch

from helpers import BF16_ATOL, BF16_RTOL, assert_close

pytestmark = pytest.mark.gpu


def _full_step(oracle, hq, hkv, cached, variant, theta, seed, sample_rows):
    from oomllama_b200 import TurboConfig, TurboEngine
    B = len(cached)
    pages = [-(-(L + 1) // 16) for L in cached]
    cfg = TurboConfig(n_layers=1, hidden_size=0, n_heads=hq, n_kv_heads=hkv, max_seq_len=max(cached) + 16,
                      max_seqs=B, n_pages=sum(pages), kv_dtype="bf16", rope_variant=variant, rope_theta=theta)
    eng = TurboEngine(cfg, device=0, assign_pages=False)
    perm = np.random.default_rng(seed).permutation(sum(pages))
    tables, o = [], 0
    for s in range(B):
        tables.append(perm[o:o + pages[s]])
        eng.set_block_table(s, tables[s].tolist())
        eng.set_seq_len(0, s, cached[s])
        o += pages[s]
    kp, vp = eng.kv_pool()
    g = torch.Generator(device="cuda").manual_seed(seed)
    kp.normal_(generator=g)
    vp.normal_(generator=g)
    kp[:, -1].zero_()
    vp[:, -1].zero_()
    q = torch.randn(B, hq * 128, generator=g, device="cuda")
    k = torch.randn(B, hkv * 128, generator=g, device="cuda")
    v = torch.randn(B, hkv * 128, generator=g, device="cuda")
    qr = eng.rope_append(0, list(range(B)), q, k, v)  # appends at slot cached[s], position cached[s]
    out = eng.decode(0, list(range(B)), qr)
    eng.sync()
    assert all(eng.seq_len(0, s) == cached[s] + 1 for s in range(B))
    c, s_ = oracle.rope_table(theta, 128, max(cached) + 1)
    var = oracle.ROPE_INTERLEAVED if variant == "interleaved" else oracle.ROPE_SPLIT_HALF
    pos = np.array(cached)
    q_ref = oracle.rope_tokens(q.cpu().numpy().reshape(B, hq, 128), pos, c, s_, var)
    k_ref = oracle.round_bf16(oracle.rope_tokens(k.cpu().numpy().reshape(B, hkv, 128), pos, c, s_, var))
    np.testing.assert_array_equal(qr.cpu().numpy(), q_ref)
    rows = np.random.default_rng(seed + 100).choice(B, size=min(sample_rows, B), replace=False)
    for r in rows:
        L = cached[r] + 1
        pg = torch.from_numpy(tables[r].astype(np.int64)).cuda()
        kr = kp[0].index_select(0, pg).permute(1, 0, 2, 3).reshape(hkv, -1, 128)[:, :L].float().cpu().numpy()
        vr = vp[0].index_select(0, pg).permute(1, 0, 2, 3).reshape(hkv, -1, 128)[:, :L].float().cpu().numpy()
        # the appended slot holds the oracle's rotated, bf16-rounded k and the bf16-rounded v
        np.testing.assert_array_equal(kr[:, L - 1], k_ref[r])
        np.testing.assert_array_equal(vr[:, L - 1], oracle.round_bf16(v[r].cpu().numpy().reshape(hkv, 128)))
        ref = oracle.gqa_attention(q_ref[r:r + 1], kr, vr, causal=False)[0]
        assert_close(out[r].cpu().numpy(), ref, BF16_ATOL, BF16_RTOL, what=f"row {r} (L {L})")
    eng.close()
    return rows


def test_full_size_batched_qwen_decode(oracle):
    # 64 sequences, cached lengths U{1024..8192} (seed 2), plus the new token
    cached = np.random.default_rng(2).integers(1024, 8193, size=64).tolist()
    _full_step(oracle, 28, 4, cached, "interleaved", 1e6, seed=2, sample_rows=10)


def test_full_size_llama_32k_decode(oracle):
    # 8 sequences x 32768 slots (32767 cached + the new one), 32q/8kv, split-half theta=5e5
    _full_step(oracle, 32, 8, [32767] * 8, "split_half", 5e5, seed=3, sample_rows=3)


def test_packed_decode_and_merge_match_unpacked():
    from oomllama_b200 import TurboConfig, TurboEngine
    from oomllama_b200._lib import PACKED_STRIDE
    lens = [0, 5, 900, 3000]
    pages = [max(1, -(-L // 16)) for L in lens]
    eng = TurboEngine(TurboConfig(n_layers=1, hidden_size=0, n_heads=28, n_kv_heads=4, max_seq_len=3008,
                                  max_seqs=4, n_pages=sum(pages), kv_dtype="bf16"), device=0, assign_pages=False)
    o = 0
    for s, n in enumerate(pages):
        eng.set_block_table(s, range(o, o + n))
        eng.set_seq_len(0, s, lens[s])
        o += n
    kp, vp = eng.kv_pool()
    g = torch.Generator(device="cuda").manual_seed(9)
    kp[:, :-1].normal_(generator=g)
    vp[:, :-1].normal_(generator=g)
    q = torch.randn(4, 28, 128, generator=g, device="cuda")
    out, lse = eng.decode(0, range(4), q, with_lse=True)
    packed = eng.decode_packed(0, range(4), q)
    eng.sync()
    assert packed.shape == (4, 28, PACKED_STRIDE)
    assert torch.equal(packed[..., :128], out) and torch.equal(packed[..., 128], lse)
    # a merge of three copies with shifted lse equals the merge of the separate arrays
    parts = torch.stack([packed, packed, packed]).reshape(3, 4 * 28, PACKED_STRIDE).clone()
    parts[1, :, 128] -= 0.5
    parts[2, :, :128] *= -1.0
    m1, _ = eng.merge_packed(parts, 3)
    m2, _ = eng.merge_partials(parts[..., :128].contiguous(), parts[..., 128].contiguous())
    eng.sync()
    assert torch.equal(m1, m2)
    eng.close()


def test_rope_q_matches_rope_append_q():
    from oomllama_b200 import TurboConfig, TurboEngine
    for variant in ("interleaved", "split_half"):
        eng = TurboEngine(TurboConfig(n_layers=1, hidden_size=0, n_heads=28, n_kv_heads=4, max_seq_len=2048,
                                      max_seqs=3, kv_dtype="bf16", rope_variant=variant, rope_theta=1e6), device=0)
        for s, L in enumerate((0, 100, 2000)):
            eng.set_seq_len(0, s, L)
        g = torch.Generator(device="cuda").manual_seed(4)
        q = torch.randn(3, 28 * 128, generator=g, device="cuda")
        k = torch.randn(3, 4 * 128, generator=g, device="cuda")
        bq = torch.randn(28 * 128, generator=g, device="cuda")
        a = eng.rope_append(0, [0, 1, 2], q, k, k.clone(), bq=bq)
        b = eng.rope_q([0, 100, 2000], q, bq=bq)
        eng.sync()
        assert torch.equal(a, b), variant
        assert [eng.seq_len(0, s) for s in range(3)] == [1, 101, 2001]
        eng.close()

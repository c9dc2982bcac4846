"""Multi-GPU decode (K-D) on real GPUs: two ranks over NCCL.

A 1-kv-head shape on 2 GPUs forces the split-context path: each rank holds
half of every sequence's pages, decodes its slice with oomattn_decode (LSE
out), the pair all-gathers the (O, lse) partials over NCCL and merges them
with oomattn_merge_partials.  The merged output must match the oracle over the
whole context.  A 4-kv-head shape on 2 GPUs checks the kv-head-group split
(no collective).  Skipped on hosts with fewer than 2 GPUs.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, n_heads, n_kv, lens, out_dir):
    import datetime

    import torch.distributed as dist

    from oomllama_b200 import TurboConfig, TurboEngine
    from oomllama_b200.shard import DecodeShardPlan, new_group_comms, sharded_decode
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device(f"cuda:{rank}"))
    plan = DecodeShardPlan(n_heads, n_kv, world, rank)
    comms = new_group_comms(plan, dist)
    g = torch.Generator().manual_seed(0)
    B = len(lens)
    q = torch.randn(B, n_heads, 128, generator=g)
    ks = [torch.randn(n_kv, L, 128, generator=g).to(torch.bfloat16) for L in lens]
    vs = [torch.randn(n_kv, L, 128, generator=g).to(torch.bfloat16) for L in lens]
    kvh, qh = plan.kv_heads, plan.q_heads
    local = [plan.context_slice(L) for L in lens]
    n_pages = sum(-(-(b - a) // 16) for a, b in local)
    eng = TurboEngine(TurboConfig(n_layers=1, hidden_size=0, n_heads=len(qh), n_kv_heads=len(kvh),
                                  max_seq_len=max(lens) + 16, max_seqs=B, n_pages=max(1, n_pages), kv_dtype="bf16"),
                      device=rank, assign_pages=False)
    o = 0
    for s, (a, b) in enumerate(local):
        np_s = -(-(b - a) // 16)
        eng.set_block_table(s, list(range(o, o + np_s)))
        o += np_s
        if b > a:
            eng.kv_write(0, s, ks[s][kvh.start:kvh.stop, a:b].transpose(0, 1).contiguous().cuda(),
                         vs[s][kvh.start:kvh.stop, a:b].transpose(0, 1).contiguous().cuda())
    out = sharded_decode(eng, 0, list(range(B)), q[:, qh.start:qh.stop].contiguous().cuda(), plan, dist,
                         comms[plan.group])
    eng.sync()
    np.save(os.path.join(out_dir, f"out{rank}.npy"), out.cpu().numpy())
    dist.barrier()
    eng.close()
    dist.destroy_process_group()


@pytest.mark.parametrize("n_heads,n_kv", [(8, 1), (28, 4)])
def test_two_gpu_sharded_decode(tmp_path, oracle, n_heads, n_kv):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from oomllama_b200.shard import DecodeShardPlan
    world = 2
    lens = [1, 17, 700, 5000]
    mp.spawn(_rank, args=(world, _free_port(), n_heads, n_kv, lens, str(tmp_path)), nprocs=world, join=True)
    g = torch.Generator().manual_seed(0)
    B = len(lens)
    q = torch.randn(B, n_heads, 128, generator=g)
    ks = [torch.randn(n_kv, L, 128, generator=g).to(torch.bfloat16) for L in lens]
    vs = [torch.randn(n_kv, L, 128, generator=g).to(torch.bfloat16) for L in lens]
    for r in range(world):
        plan = DecodeShardPlan(n_heads, n_kv, world, r)
        got = np.load(tmp_path / f"out{r}.npy")
        for b in range(B):
            ref = oracle.gqa_attention(q[b:b + 1].numpy(), ks[b].float().numpy(), vs[b].float().numpy(),
                                       causal=False)[0, plan.q_heads.start:plan.q_heads.stop]
            err = float(np.abs(got[b] - ref).max())
            assert err <= 2e-3, f"rank {r} seq {b}: max-abs {err:.2e}"


def _step_rank(rank, world, port, n_heads, n_kv, lens, steps, out_dir):
    """Decode steps with the new token appended on the owning rank only (ShardedDecodeStep)."""
    import datetime

    import torch.distributed as dist

    from oomllama_b200 import TurboConfig, TurboEngine
    from oomllama_b200.shard import DecodeShardPlan, ShardedDecodeStep, new_group_comms
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device(f"cuda:{rank}"))
    plan = DecodeShardPlan(n_heads, n_kv, world, rank)
    comms = new_group_comms(plan, dist)
    g = torch.Generator().manual_seed(0)
    B = len(lens)
    ks = [torch.randn(n_kv, L, 128, generator=g).to(torch.bfloat16) for L in lens]
    vs = [torch.randn(n_kv, L, 128, generator=g).to(torch.bfloat16) for L in lens]
    new = [(torch.randn(B, n_heads * 128, generator=g), torch.randn(B, n_kv * 128, generator=g),
            torch.randn(B, n_kv * 128, generator=g)) for _ in range(steps)]
    kvh, qh = plan.kv_heads, plan.q_heads
    local = [plan.context_slice(L) for L in lens]
    cap = [b - a + (steps if plan.slice_index == plan.ctx_split - 1 else 0) for a, b in local]
    n_pages = sum(-(-c // 16) for c in cap)
    eng = TurboEngine(TurboConfig(n_layers=1, hidden_size=0, n_heads=len(qh), n_kv_heads=len(kvh),
                                  max_seq_len=max(lens) + steps + 16, max_seqs=B, n_pages=max(1, n_pages),
                                  kv_dtype="bf16", rope_variant="interleaved", rope_theta=1e6),
                      device=rank, assign_pages=False)
    o = 0
    for s, (a, b) in enumerate(local):
        np_s = -(-cap[s] // 16)
        eng.set_block_table(s, list(range(o, o + np_s)))
        o += np_s
        if b > a:
            eng.kv_write(0, s, ks[s][kvh.start:kvh.stop, a:b].transpose(0, 1).contiguous().cuda(),
                         vs[s][kvh.start:kvh.stop, a:b].transpose(0, 1).contiguous().cuda())
    step = ShardedDecodeStep(eng, plan, 0, range(B), lens, dist, comms[plan.group])
    outs = []
    for q, k, v in new:
        sl = lambda t, hs: t.view(B, -1, 128)[:, hs.start:hs.stop].reshape(B, -1).contiguous().cuda()  # noqa
        outs.append(step(sl(q, qh), sl(k, kvh), sl(v, kvh)).clone())
    eng.sync()
    np.save(os.path.join(out_dir, f"step{rank}.npy"), torch.stack(outs).cpu().numpy())
    np.save(os.path.join(out_dir, f"len{rank}.npy"), np.array([eng.seq_len(0, s) for s in range(B)]))
    dist.barrier()
    eng.close()
    dist.destroy_process_group()


@pytest.mark.parametrize("n_heads,n_kv", [(8, 1), (28, 4)])
def test_two_gpu_decode_steps_append_on_owner(tmp_path, oracle, n_heads, n_kv):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from oomllama_b200.shard import DecodeShardPlan
    world, steps = 2, 3
    lens = [1, 17, 700, 5000]
    mp.spawn(_step_rank, args=(world, _free_port(), n_heads, n_kv, lens, steps, str(tmp_path)), nprocs=world,
             join=True)
    g = torch.Generator().manual_seed(0)
    B = len(lens)
    ks = [torch.randn(n_kv, L, 128, generator=g).to(torch.bfloat16).float().numpy() for L in lens]
    vs = [torch.randn(n_kv, L, 128, generator=g).to(torch.bfloat16).float().numpy() for L in lens]
    new = [(torch.randn(B, n_heads * 128, generator=g), torch.randn(B, n_kv * 128, generator=g),
            torch.randn(B, n_kv * 128, generator=g)) for _ in range(steps)]
    c, s_ = oracle.rope_table(1e6, 128, max(lens) + steps + 1)
    refs = []
    for t, (q, k, v) in enumerate(new):
        pos = np.array(lens) + t
        qr = oracle.rope_tokens(q.numpy().reshape(B, n_heads, 128), pos, c, s_, oracle.ROPE_INTERLEAVED)
        kr = oracle.round_bf16(oracle.rope_tokens(k.numpy().reshape(B, n_kv, 128), pos, c, s_,
                                                  oracle.ROPE_INTERLEAVED))
        vr = oracle.round_bf16(v.numpy().reshape(B, n_kv, 128))
        step_ref = []
        for b in range(B):
            ks[b] = np.concatenate([ks[b], kr[b][:, None]], axis=1)
            vs[b] = np.concatenate([vs[b], vr[b][:, None]], axis=1)
            step_ref.append(oracle.gqa_attention(qr[b:b + 1], ks[b], vs[b], causal=False)[0])
        refs.append(np.stack(step_ref))
    for r in range(world):
        plan = DecodeShardPlan(n_heads, n_kv, world, r)
        got = np.load(tmp_path / f"step{r}.npy")
        lens_r = np.load(tmp_path / f"len{r}.npy")
        for b, L in enumerate(lens):
            a, e = plan.context_slice(L)
            grew = steps if plan.slice_index == plan.ctx_split - 1 else 0
            assert lens_r[b] == e - a + grew  # only the owner of the tail appended
        for t in range(steps):
            err = float(np.abs(got[t] - refs[t][:, plan.q_heads.start:plan.q_heads.stop]).max())
            assert err <= 2e-3, f"rank {r} step {t}: max-abs {err:.2e}"


def _prefill_rank(rank, world, port, n_new, out_dir):
    """One sequence's causal prefill sharded by PrefillShardPlan (kv-head groups, then zig-zag blocks)."""
    from oomllama_b200 import TurboConfig, TurboEngine
    from oomllama_b200.shard import PrefillShardPlan
    torch.cuda.set_device(rank)
    plan = PrefillShardPlan(8, 1, world, rank)
    g = torch.Generator().manual_seed(5)
    q = torch.randn(n_new, 8, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(n_new, 1, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(n_new, 1, 128, generator=g).to(torch.bfloat16)
    eng = TurboEngine(TurboConfig(n_layers=1, hidden_size=0, n_heads=len(plan.q_heads),
                                  n_kv_heads=len(plan.kv_heads), max_seq_len=n_new, kv_dtype="bf16"), device=rank)
    qh, kvh = plan.q_heads, plan.kv_heads
    qr = eng.rope_append(0, [0], q[:, qh.start:qh.stop].reshape(n_new, -1).contiguous().cuda(),
                         k[:, kvh.start:kvh.stop].reshape(n_new, -1).contiguous().cuda(),
                         v[:, kvh.start:kvh.stop].reshape(n_new, -1).contiguous().cuda(), q_out_dtype=torch.bfloat16)
    out = torch.full((n_new, len(qh), 128), float("nan"), device=f"cuda:{rank}")
    eng.prefill(0, 0, qr, out=out, blocks=plan.blocks(n_new))
    eng.sync()
    np.save(os.path.join(out_dir, f"pf{rank}.npy"), out.cpu().numpy())
    np.save(os.path.join(out_dir, f"qr{rank}.npy"), qr.float().cpu().numpy())
    eng.close()


def test_two_gpu_sharded_prefill_zigzag(tmp_path, oracle):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    n_new, world = 1500, 2
    mp.spawn(_prefill_rank, args=(world, 0, n_new, str(tmp_path)), nprocs=world, join=True)
    g = torch.Generator().manual_seed(5)
    q = torch.randn(n_new, 8, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(n_new, 1, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(n_new, 1, 128, generator=g).to(torch.bfloat16)
    c, s_ = oracle.rope_table(1e6, 128, n_new)
    pos = np.arange(n_new)
    qr = oracle.round_bf16(oracle.rope_tokens(q.float().numpy(), pos, c, s_, oracle.ROPE_INTERLEAVED))
    kr = oracle.round_bf16(oracle.rope_tokens(k.float().numpy(), pos, c, s_, oracle.ROPE_INTERLEAVED))
    merged = np.full((n_new, 8, 128), np.nan, np.float32)
    for r in range(world):
        got = np.load(tmp_path / f"pf{r}.npy")
        np.testing.assert_array_equal(np.load(tmp_path / f"qr{r}.npy"), qr)
        done = ~np.isnan(got[:, 0, 0])
        assert not (done & ~np.isnan(merged[:, 0, 0])).any()  # no row computed twice
        merged[done] = got[done]
    assert not np.isnan(merged).any()  # every row computed once
    rows = np.random.default_rng(0).integers(0, n_new, 64)
    heads = np.random.default_rng(1).integers(0, 8, 64)
    ref = oracle.gqa_attention_rows(qr, kr.transpose(1, 0, 2).copy(),
                                    v.float().numpy().transpose(1, 0, 2).copy(), rows, heads, causal=True)
    err = float(np.abs(merged[rows, heads] - ref).max())
    assert err <= 2e-3, f"sharded prefill max-abs {err:.2e}"

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

"""Multi-GPU sharding logic on CPU ranks (gloo): the decode shard plan, the
partial all-gather of split contexts and the LSE merge reproduce the unsharded
attention.  The per-rank attention and the merge are computed by the oracle
here (no GPU); on GPUs the same plan drives oomattn_decode + NCCL +
oomattn_merge_partials."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oomllama_b200.shard import DecodeShardPlan, gather_partials, new_group_comms


def test_plan_partitions_heads_and_slots():
    for n_heads, n_kv, world in ((28, 4, 1), (28, 4, 2), (28, 4, 4), (28, 4, 8), (32, 8, 8), (32, 8, 2)):
        plans = [DecodeShardPlan(n_heads, n_kv, world, r) for r in range(world)]
        grp = n_heads // n_kv
        for p in plans:
            assert all(h // grp in p.kv_heads for h in p.q_heads)
        # every (q head, slot) pair has exactly one owner
        for L in (1, 15, 16, 17, 1000, 8193):
            cover = np.zeros((n_heads, L), np.int32)
            for p in plans:
                a, b = p.context_slice(L)
                assert a % 16 == 0
                cover[p.q_heads.start:p.q_heads.stop, a:b] += 1
            assert (cover == 1).all()
    with pytest.raises(ValueError):
        DecodeShardPlan(28, 4, 3, 0)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, n_heads, n_kv, lens, result_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    from oracle import oracle as O
    plan = DecodeShardPlan(n_heads, n_kv, world, rank)
    comms = new_group_comms(plan, dist)
    rng = np.random.default_rng(0)
    B = len(lens)
    q = rng.standard_normal((B, n_heads, 128)).astype(np.float32)
    ks = [rng.standard_normal((n_kv, L, 128)).astype(np.float32) for L in lens]
    vs = [rng.standard_normal((n_kv, L, 128)).astype(np.float32) for L in lens]
    qh, kvh = plan.q_heads, plan.kv_heads
    outs, lses = [], []
    for b, L in enumerate(lens):
        a, e = plan.context_slice(L)
        k = ks[b][kvh.start:kvh.stop, a:e]
        v = vs[b][kvh.start:kvh.stop, a:e]
        if e > a:
            o, l = O.gqa_attention(q[b:b + 1, qh.start:qh.stop], k, v, causal=False, with_lse=True)
            outs.append(o[0])
            lses.append(l[0])
        else:
            outs.append(np.zeros((len(qh), 128), np.float32))
            lses.append(np.full(len(qh), -np.inf, np.float32))
    out_t = torch.from_numpy(np.stack(outs))
    lse_t = torch.from_numpy(np.stack(lses))
    parts, pl = gather_partials(out_t, lse_t, plan, dist, comms[plan.group])
    merged, _ = O.merge_partials(parts.numpy(), pl.numpy())
    merged = merged.reshape(B, len(qh), 128)
    err = 0.0
    for b in range(B):
        ref = O.gqa_attention(q[b:b + 1], ks[b], vs[b], causal=False)[0, qh.start:qh.stop]
        err = max(err, float(np.abs(merged[b] - ref).max()))
    np.save(os.path.join(result_dir, f"err{rank}.npy"), np.array(err))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,n_heads,n_kv", [(2, 28, 4), (4, 28, 2), (4, 8, 1)])
def test_split_context_merge_gloo(tmp_path, world, n_heads, n_kv):
    lens = [1, 17, 300, 1025]
    mp.spawn(_worker, args=(world, _free_port(), n_heads, n_kv, lens, str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        assert float(np.load(tmp_path / f"err{r}.npy")) < 2e-5

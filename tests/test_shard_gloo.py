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


def test_owner_of_slot_prompt_slices_then_tail():
    for world, n_heads, n_kv in ((8, 28, 4), (2, 8, 1), (4, 28, 2)):
        plans = [DecodeShardPlan(n_heads, n_kv, world, r) for r in range(world)]
        for P in (1, 16, 17, 300, 1025):
            for slot in list(range(0, P, 7)) + [P - 1, P, P + 5, P + 400]:
                owners = [p for p in plans if p.group == 0 and p.appends_here(P, slot)]
                assert len(owners) == 1
                s = owners[0].slice_index
                if slot >= P:
                    assert s == plans[0].ctx_split - 1
                else:
                    a, b = owners[0].slice_of(P, s)
                    assert a <= slot < b


class _OracleEngine:
    """CPU stand-in for TurboEngine with the calls ShardedDecodeStep makes, computed by the oracle: the
    step's host logic (which rank appends, the positions, the packed all-gather and the merge) runs
    unchanged on gloo ranks."""

    def __init__(self, n_heads, n_kv, cos_t, sin_t, variant):
        from types import SimpleNamespace
        self.config = SimpleNamespace(n_heads=n_heads, n_kv_heads=n_kv)
        self.cos, self.sin, self.variant = cos_t, sin_t, variant
        self.k, self.v, self.off = {}, {}, {}

    def load(self, s, k, v):
        self.k[s], self.v[s] = k.copy(), v.copy()

    def set_position_offset(self, s, a):
        self.off[s] = a

    def _rope(self, x, pos):
        from oracle import oracle as O
        return O.rope_apply(x, self.cos[pos], self.sin[pos], self.variant)

    def rope_append(self, layer, seq_ids, q, k, v, bq=None, bk=None, bv=None):
        hq, hkv = self.config.n_heads, self.config.n_kv_heads
        out = []
        for i, s in enumerate(seq_ids):
            pos = self.off[s] + self.k[s].shape[1]
            out.append(self._rope(q[i].numpy().reshape(hq, 128), pos))
            kr = self._rope(k[i].numpy().reshape(hkv, 128), pos)
            self.k[s] = np.concatenate([self.k[s], kr[:, None]], axis=1)
            self.v[s] = np.concatenate([self.v[s], v[i].numpy().reshape(hkv, 1, 128)], axis=1)
        return torch.from_numpy(np.stack(out))

    def rope_q(self, positions, q, bq=None):
        hq = self.config.n_heads
        return torch.from_numpy(np.stack([self._rope(q[i].numpy().reshape(hq, 128), p)
                                          for i, p in enumerate(positions)]))

    def decode_packed(self, layer, seq_ids, q, lens=None, out=None):
        from oracle import oracle as O
        for i, s in enumerate(seq_ids):
            if self.k[s].shape[1] == 0:
                out[i, :, :128] = 0.0
                out[i, :, 128] = float("-inf")
                continue
            o, l = O.gqa_attention(q[i:i + 1].numpy(), self.k[s], self.v[s], causal=False, with_lse=True)
            out[i, :, :128] = torch.from_numpy(o[0])
            out[i, :, 128] = torch.from_numpy(l[0])
        return out

    def merge_packed(self, packed, n_parts, out=None, lse=None):
        from oracle import oracle as O
        o, _ = O.merge_partials(packed[..., :128].numpy(), packed[..., 128].numpy())
        out.copy_(torch.from_numpy(o))
        return out, None

    def decode(self, layer, seq_ids, q, lens=None):
        from oracle import oracle as O
        return torch.from_numpy(np.stack([O.gqa_attention(q[i:i + 1].numpy(), self.k[s], self.v[s],
                                                          causal=False)[0] for i, s in enumerate(seq_ids)]))


def _step_worker(rank, world, port, n_heads, n_kv, lens, steps, result_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    from oracle import oracle as O
    from oomllama_b200.shard import ShardedDecodeStep
    plan = DecodeShardPlan(n_heads, n_kv, world, rank)
    comms = new_group_comms(plan, dist)
    cos_t, sin_t = O.rope_table(1e6, 128, max(lens) + steps + 1)
    rng = np.random.default_rng(1)
    B = len(lens)
    # the prompt's K/V, already rotated, identical on every rank (same seed)
    ks = [rng.standard_normal((n_kv, L, 128)).astype(np.float32) for L in lens]
    vs = [rng.standard_normal((n_kv, L, 128)).astype(np.float32) for L in lens]
    qh, kvh = plan.q_heads, plan.kv_heads
    eng = _OracleEngine(len(qh), len(kvh), cos_t, sin_t, O.ROPE_INTERLEAVED)
    for b, L in enumerate(lens):
        a, e = plan.context_slice(L)
        eng.load(b, ks[b][kvh.start:kvh.stop, a:e], vs[b][kvh.start:kvh.stop, a:e])
    step = ShardedDecodeStep(eng, plan, 0, range(B), lens, dist, comms[plan.group])
    err = 0.0
    for t in range(steps):
        q = rng.standard_normal((B, n_heads, 128)).astype(np.float32)
        k = rng.standard_normal((B, n_kv, 128)).astype(np.float32)
        v = rng.standard_normal((B, n_kv, 128)).astype(np.float32)
        got = step(torch.from_numpy(q[:, qh.start:qh.stop].reshape(B, -1).copy()),
                   torch.from_numpy(k[:, kvh.start:kvh.stop].reshape(B, -1).copy()),
                   torch.from_numpy(v[:, kvh.start:kvh.stop].reshape(B, -1).copy()))
        for b in range(B):  # unsharded reference: append then attend over the whole context
            pos = lens[b] + t
            kr = O.rope_apply(k[b], cos_t[pos], sin_t[pos], O.ROPE_INTERLEAVED)
            ks[b] = np.concatenate([ks[b], kr[:, None]], axis=1)
            vs[b] = np.concatenate([vs[b], v[b][:, None]], axis=1)
            qr = O.rope_apply(q[b], cos_t[pos], sin_t[pos], O.ROPE_INTERLEAVED)
            ref = O.gqa_attention(qr[None], ks[b], vs[b], causal=False)[0, qh.start:qh.stop]
            err = max(err, float(np.abs(got[b].numpy() - ref).max()))
    appended = sum(eng.k[b].shape[1] for b in range(B)) - sum(b_ - a_ for a_, b_ in
                                                                (plan.context_slice(L) for L in lens))
    np.save(os.path.join(result_dir, f"step{rank}.npy"), np.array([err, appended]))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,n_heads,n_kv", [(2, 8, 1), (4, 28, 2), (2, 28, 4)])
def test_sharded_decode_step_appends_on_owner_gloo(tmp_path, world, n_heads, n_kv):
    lens, steps = [1, 17, 300, 1025], 3
    mp.spawn(_step_worker, args=(world, _free_port(), n_heads, n_kv, lens, steps, str(tmp_path)), nprocs=world,
             join=True)
    split = DecodeShardPlan(n_heads, n_kv, world, 0).ctx_split
    for r in range(world):
        err, appended = np.load(tmp_path / f"step{r}.npy")
        assert err < 2e-5, f"rank {r}: max-abs {err}"
        # only the last slice of each group stores the steps' tokens
        plan = DecodeShardPlan(n_heads, n_kv, world, r)
        assert appended == (len(lens) * steps if plan.slice_index == split - 1 else 0)

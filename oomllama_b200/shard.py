"""Multi-GPU sharding of the decode step (K-D host logic).

One process per GPU.  Work units are (sequence, kv-head group): the reference
has no multi-GPU attention at all (its only multi-GPU feature is even/odd layer
placement, src/oomllama.rs:474-501), so this is new.

  * world <= n_kv: rank r owns kv heads [r*n_kv/world, (r+1)*n_kv/world) and
    their q heads (h -> h / group keeps a q head with its kv head), for every
    sequence.  No data-path collective: each rank's output heads are final.
  * world > n_kv (e.g. 4 kv heads on 8 GPUs): ranks form n_kv groups of
    world/n_kv; inside a group each rank holds a contiguous page-aligned slice
    of every sequence's context.  Each rank's decode yields a partial
    (normalised O, natural-log lse) per (sequence, q head); the group
    all-gathers them over NCCL and merges with oomattn_merge_partials (K-B2):
      M = max lse_p ; O = sum e^(lse_p - M) O_p / sum e^(lse_p - M).
KV never moves between GPUs: K-A appends a token on the rank whose slice
holds its slot, so only ~0.5 KB per (sequence, q head) crosses NVLink per step.
"""
from __future__ import annotations

from dataclasses import dataclass

PAGE = 16


@dataclass(frozen=True)
class DecodeShardPlan:
    n_heads: int
    n_kv: int
    world: int
    rank: int

    def __post_init__(self):
        if self.n_heads % self.n_kv:
            raise ValueError("n_heads must be a multiple of n_kv")
        if self.world <= 0 or not 0 <= self.rank < self.world:
            raise ValueError("bad rank / world")
        g = self.groups
        if self.n_kv % g or self.world % g:
            raise ValueError(f"{self.world} GPUs cannot shard {self.n_kv} kv heads evenly")

    @property
    def groups(self) -> int:
        """Number of kv-head groups (= GPUs per context slice set)."""
        return min(self.world, self.n_kv)

    @property
    def ctx_split(self) -> int:
        """Context slices per sequence (1 unless GPUs outnumber kv heads)."""
        return self.world // self.groups

    @property
    def group(self) -> int:
        return self.rank // self.ctx_split

    @property
    def slice_index(self) -> int:
        return self.rank % self.ctx_split

    @property
    def kv_heads(self) -> range:
        per = self.n_kv // self.groups
        return range(self.group * per, (self.group + 1) * per)

    @property
    def q_heads(self) -> range:
        grp = self.n_heads // self.n_kv
        kv = self.kv_heads
        return range(kv.start * grp, kv.stop * grp)

    def group_ranks(self, group: int | None = None) -> list[int]:
        g = self.group if group is None else group
        return list(range(g * self.ctx_split, (g + 1) * self.ctx_split))

    def context_slice(self, length: int) -> tuple[int, int]:
        """Cache slots [start, end) of a sequence of `length` slots held by this rank
        (whole pages; the last slice takes the remainder)."""
        pages = -(-length // PAGE)
        s, n = self.slice_index, self.ctx_split
        p0, p1 = pages * s // n, pages * (s + 1) // n
        return min(length, p0 * PAGE), min(length, p1 * PAGE)

    def owner_of_slot(self, length_after: int, slot: int) -> int:
        """Slice index that stores `slot` when the sequence holds `length_after` slots."""
        for s in range(self.ctx_split):
            plan = DecodeShardPlan(self.n_heads, self.n_kv, self.world, self.group * self.ctx_split + s)
            a, b = plan.context_slice(length_after)
            if a <= slot < b:
                return s
        raise ValueError("slot outside the sequence")


def new_group_comms(plan: DecodeShardPlan, dist):
    """Process groups of every kv-head group (all ranks must call this, in order)."""
    return [dist.new_group(plan.group_ranks(g)) for g in range(plan.groups)]


def gather_partials(out, lse, plan: DecodeShardPlan, dist, comm):
    """All-gather this group's partials: out [rows, Hq_local, 128], lse
    [rows, Hq_local] -> parts [ctx_split, rows*Hq_local, 128], lses [ctx_split, rows*Hq_local]."""
    import torch
    n = plan.ctx_split
    parts = torch.empty((n,) + tuple(out.reshape(-1, out.shape[-1]).shape), dtype=out.dtype, device=out.device)
    lses = torch.empty((n, lse.numel()), dtype=lse.dtype, device=lse.device)
    if n == 1:
        parts[0].copy_(out.reshape(-1, out.shape[-1]))
        lses[0].copy_(lse.reshape(-1))
        return parts, lses
    src_o = out.reshape(-1, out.shape[-1]).contiguous()
    src_l = lse.reshape(-1).contiguous()
    if dist.get_backend(comm) == "nccl":
        dist.all_gather_into_tensor(parts, src_o, group=comm)
        dist.all_gather_into_tensor(lses, src_l, group=comm)
    else:  # gloo (host-side tests)
        dist.all_gather(list(parts.unbind(0)), src_o, group=comm)
        dist.all_gather(list(lses.unbind(0)), src_l, group=comm)
    return parts, lses


def sharded_decode(engine, layer, seq_ids, q_local, plan: DecodeShardPlan, dist=None, comm=None):
    """Decode on this rank's shard; with a split context, gather and merge the
    group's partials.  q_local: [rows, len(plan.q_heads), 128] f32 on this GPU.
    Returns the merged output of this rank's q heads [rows, Hq_local, 128]."""
    if plan.ctx_split == 1:
        return engine.decode(layer, seq_ids, q_local)
    out, lse = engine.decode(layer, seq_ids, q_local, with_lse=True)
    parts, lses = gather_partials(out, lse, plan, dist, comm)
    merged, _ = engine.merge_partials(parts, lses)
    return merged.view_as(out)

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
The prompt's slots are cut into page-aligned slices at the prompt length;
tokens appended by decode steps belong to the last slice, so no slice
boundary moves while a sequence grows.  The ranks that do not append a step's
token rotate its query at the same global position (oomattn_rope_q) and
attend over their own slices.  Each rank's decode writes O and lse packed per
(sequence, q head) (oomattn_decode_packed), so the group exchanges them with
one all-gather into a preallocated buffer before the merge.
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
        return self.slice_of(length, self.slice_index)

    def slice_of(self, prompt_len: int, s: int) -> tuple[int, int]:
        """Prompt slots [start, end) of slice s (whole pages; the last slice takes the remainder)."""
        pages = -(-prompt_len // PAGE)
        n = self.ctx_split
        p0, p1 = pages * s // n, pages * (s + 1) // n
        return min(prompt_len, p0 * PAGE), min(prompt_len, p1 * PAGE)

    def owner_of_slot(self, prompt_len: int, slot: int) -> int:
        """Slice index that stores `slot` of a sequence whose prompt held `prompt_len` slots: prompt
        slots by their page-aligned slice, every later (decode-appended) slot in the last slice."""
        if slot < 0:
            raise ValueError("negative slot")
        if slot >= prompt_len:
            return self.ctx_split - 1
        for s in range(self.ctx_split):
            a, b = self.slice_of(prompt_len, s)
            if a <= slot < b:
                return s
        raise ValueError("slot outside the sequence")

    def appends_here(self, prompt_len: int, slot: int) -> bool:
        """Whether this rank's slice stores `slot` (and so appends the token written there)."""
        return self.owner_of_slot(prompt_len, slot) == self.slice_index


@dataclass(frozen=True)
class PrefillShardPlan:
    """Sharding of one sequence's causal prefill (flash_attention_forward's causal path,
    src/oomllama_turbo.rs:344-368) over `world` GPUs.  Up to n_kv GPUs, rank r owns the kv heads
    [r*n_kv/world, (r+1)*n_kv/world) with their q heads and every query row.  Beyond that the ranks
    of a kv-head group also split the 256-row query blocks zig-zag: the blocks are cut into
    2 * q_split contiguous chunks and slice s takes chunks s and 2 * q_split - 1 - s, so every rank
    gets an equal share of the causal work (early rows see few keys, late rows many).  Each rank
    holds the whole K/V of its heads, so no collective is needed."""
    n_heads: int
    n_kv: int
    world: int
    rank: int

    def __post_init__(self):
        DecodeShardPlan(self.n_heads, self.n_kv, self.world, self.rank)  # same validation

    @property
    def groups(self) -> int:
        return min(self.world, self.n_kv)

    @property
    def q_split(self) -> int:
        return self.world // self.groups

    @property
    def group(self) -> int:
        return self.rank // self.q_split

    @property
    def slice_index(self) -> int:
        return self.rank % self.q_split

    @property
    def kv_heads(self) -> range:
        per = self.n_kv // self.groups
        return range(self.group * per, (self.group + 1) * per)

    @property
    def q_heads(self) -> range:
        grp = self.n_heads // self.n_kv
        kv = self.kv_heads
        return range(kv.start * grp, kv.stop * grp)

    def blocks(self, n_new: int) -> list[tuple[int, int]]:
        """This rank's 256-row query blocks as disjoint [lo, hi) ranges (empty ranges dropped)."""
        nb = -(-n_new // 256)
        n, s = self.q_split, self.slice_index
        cut = [nb * i // (2 * n) for i in range(2 * n + 1)]
        ranges = [(cut[s], cut[s + 1]), (cut[2 * n - 1 - s], cut[2 * n - s])]
        if ranges[0][1] == ranges[1][0]:  # the two chunks touch (middle slice): one range
            ranges = [(ranges[0][0], ranges[1][1])]
        return [r for r in ranges if r[1] > r[0]]


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


def gather_packed(packed, plan: DecodeShardPlan, dist, comm, out=None):
    """All-gather this group's packed partials [rows, Hq_local, PACKED_STRIDE] with ONE collective into
    out [ctx_split, rows * Hq_local, PACKED_STRIDE] (allocated when None; pass it back to reuse it)."""
    import torch
    n = plan.ctx_split
    src = packed.reshape(-1, packed.shape[-1])
    if out is None:
        out = torch.empty((n,) + tuple(src.shape), dtype=packed.dtype, device=packed.device)
    if n == 1:
        out[0].copy_(src)
    elif dist.get_backend(comm) == "nccl":
        dist.all_gather_into_tensor(out, src, group=comm)
    else:  # gloo (host-side tests)
        dist.all_gather(list(out.unbind(0)), src.contiguous(), group=comm)
    return out


class SplitContextDecoder:
    """K-D on one rank: decode its shard of every row with the (O, lse) outputs packed, one all-gather of
    the group's partials, then the K-B2 merge.  Buffers are allocated once per batch size."""

    def __init__(self, engine, plan: DecodeShardPlan, dist=None, comm=None):
        self.engine, self.plan, self.dist, self.comm = engine, plan, dist, comm
        self._bufs = {}

    def buffers(self, rows: int, hq: int, device):
        """(packed [rows, hq, PACKED_STRIDE], gathered [ctx_split, rows*hq, PACKED_STRIDE], out [rows, hq, 128])."""
        import torch

        from ._lib import PACKED_STRIDE
        key = (rows, hq)
        if key not in self._bufs:
            n = self.plan.ctx_split
            self._bufs[key] = (torch.empty(rows, hq, PACKED_STRIDE, device=device),
                               torch.empty(n, rows * hq, PACKED_STRIDE, device=device),
                               torch.empty(rows, hq, 128, device=device))
        return self._bufs[key]

    def __call__(self, layer, seq_ids, q_local, lens=None):
        """q_local [rows, Hq_local, 128] f32 (rotated) -> merged output [rows, Hq_local, 128] (a buffer
        this object reuses on the next call with the same row count)."""
        rows, hq = q_local.shape[0], q_local.shape[1]
        if self.plan.ctx_split == 1:
            return self.engine.decode(layer, seq_ids, q_local, lens=lens)
        packed, gathered, out = self.buffers(rows, hq, q_local.device)
        self.engine.decode_packed(layer, seq_ids, q_local, lens=lens, out=packed)
        gather_packed(packed, self.plan, self.dist, self.comm, out=gathered)
        self.engine.merge_packed(gathered, self.plan.ctx_split, out=out.view(rows * hq, 128))
        return out


class ShardedDecodeStep:
    """One decode step of one layer on this rank of a sharded engine, new token included: the token of
    each sequence is appended (K-A: bias + RoPE + paged append, src/oomllama_turbo.rs:647-681) only on
    the rank whose slice stores its slot -- KV never moves -- and every rank attends with the query
    rotated at the token's global position (src/oomllama_turbo.rs:680-695: append, then attend).
    The engine holds this rank's kv heads and its slice of every sequence; `prompt_lens` are the
    sequences' global lengths when the slices were cut (the engine's cached lengths are the slices')."""

    def __init__(self, engine, plan: DecodeShardPlan, layer: int, seq_ids, prompt_lens, dist=None, comm=None):
        self.engine, self.plan, self.layer = engine, plan, layer
        self.seq_ids = list(seq_ids)
        self.prompt_lens = list(prompt_lens)
        self.global_lens = list(prompt_lens)
        self.decoder = SplitContextDecoder(engine, plan, dist, comm)
        for s, L in zip(self.seq_ids, self.prompt_lens):
            a, _ = plan.slice_of(L, plan.slice_index)
            engine.set_position_offset(s, a)  # this slice's slot 0 sits at global position a

    def __call__(self, q, k, v, bq=None, bk=None, bv=None):
        """q [B, Hq_local*128], k, v [B, Hkv_local*128] projected (before bias and RoPE) for the new token
        of each sequence -> attention output [B, Hq_local, 128] over the whole global context."""
        import torch
        B = len(self.seq_ids)
        mine = [self.plan.appends_here(L, g) for L, g in zip(self.prompt_lens, self.global_lens)]
        hq = self.engine.config.n_heads
        if all(mine):
            qr = self.engine.rope_append(self.layer, self.seq_ids, q, k, v, bq, bk, bv)
        else:
            qr = self.engine.rope_q(self.global_lens, q, bq)
            idx = [i for i, m in enumerate(mine) if m]
            if idx:  # the sequences whose new slot lies in this rank's slice
                sel = torch.tensor(idx, device=q.device)
                self.engine.rope_append(self.layer, [self.seq_ids[i] for i in idx], q.index_select(0, sel).contiguous(),
                                        k.index_select(0, sel).contiguous(), v.index_select(0, sel).contiguous(),
                                        bq, bk, bv)
        self.global_lens = [g + 1 for g in self.global_lens]
        return self.decoder(self.layer, self.seq_ids, qr.view(B, hq, 128))


def sharded_decode(engine, layer, seq_ids, q_local, plan: DecodeShardPlan, dist=None, comm=None):
    """Decode on this rank's shard; with a split context, gather and merge the
    group's partials.  q_local: [rows, len(plan.q_heads), 128] f32 on this GPU.
    Returns the merged output of this rank's q heads [rows, Hq_local, 128]."""
    return SplitContextDecoder(engine, plan, dist, comm)(layer, seq_ids, q_local)

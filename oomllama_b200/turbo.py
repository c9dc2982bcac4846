"""TurboEngine-compatible host interface over the oomattn C ABI.

Mirrors the reference's public turbo API (src/oomllama_turbo.rs, re-exported
at src/lib.rs:99): ``TurboConfig`` (:474-516), ``TurboEngine.new`` (:528),
``attention_forward_with_bias`` (:618-723), ``reset`` (:726), ``seq_len``
(:731) and the per-layer cache view of ``LayerKVCache`` / ``ModelKVCache``
(:26-104).  Tensors are torch CUDA tensors used only as device buffers; every
computation runs in liboomattn.so on the caller's current CUDA stream.

Differences from the reference, all deliberate and matching its intended
semantics:
  * RoPE positions come from each layer's own cache length (the reference
    reads layer 0's, :671 with :101-103), and positions are checked against
    max_seq_len (the reference never enforces it, :74-85);
  * GQA uses the KV length (the reference reshapes with q's length, :324);
  * the causal mask is aligned to the end of the cache, so chunked prefill on
    a non-empty cache works (the reference's mask assumes q_len == kv_len);
  * the RoPE variant and theta are configuration, not hard-coded (:746).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import torch

from . import _lib
from ._lib import DTYPE_BF16, DTYPE_F32, ROPE_INTERLEAVED, ROPE_SPLIT_HALF, check, int_array

PAGE_SIZE = 16
HEAD_DIM = 128

_DT = {torch.float32: DTYPE_F32, torch.bfloat16: DTYPE_BF16}


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype not in _DT:
        raise TypeError(f"unsupported dtype {t.dtype}; expected float32 or bfloat16")
    return _DT[t.dtype]


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _dev(t: torch.Tensor, name: str, device: int, dtype=None, numel=None):
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise TypeError(f"{name} must be a CUDA tensor")
    if t.device.index != device:
        raise ValueError(f"{name} is on cuda:{t.device.index}, the engine on cuda:{device}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if dtype is not None and t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if numel is not None and t.numel() != numel:
        raise ValueError(f"{name} has {t.numel()} elements, expected {numel}")
    return t


@dataclass
class TurboConfig:
    """TurboConfig (src/oomllama_turbo.rs:474-497) plus the settings the
    reference hard-codes (theta at :746) or does not have (paging, cache
    dtype, RoPE variant).  The layer-pinning / prefetch fields are kept for
    signature parity; weights are the caller's device tensors here."""

    n_layers: int
    hidden_size: int
    n_heads: int
    n_kv_heads: int
    head_dim: int = HEAD_DIM
    max_seq_len: int = 8192
    vram_budget_gb: float = 0.0
    pin_strategy: object = None
    prefetch_lookahead: int = 0
    use_flash_attention: bool = True
    use_fp16: bool = False
    # new settings
    max_seqs: int = 1
    n_pages: int | None = None          # default: every sequence can reach max_seq_len
    kv_dtype: str = "f32"               # "f32" or "bf16"
    rope_variant: str = "interleaved"   # "interleaved" (apply_rope) or "split_half" (apply_rope_llama)
    rope_theta: float = 1e6
    softmax_scale: float | None = None  # None: 1/sqrt(head_dim)

    @staticmethod
    def qwen32b_dual3060() -> "TurboConfig":
        """The reference's preset (src/oomllama_turbo.rs:500-515)."""
        return TurboConfig(n_layers=64, hidden_size=5120, n_heads=40, n_kv_heads=8, head_dim=128,
                           max_seq_len=8192, vram_budget_gb=20.0, prefetch_lookahead=2, use_fp16=True)

    def pages_per_seq(self) -> int:
        return -(-self.max_seq_len // PAGE_SIZE)

    def to_c(self) -> _lib.Config:
        n_pages = self.n_pages if self.n_pages is not None else self.max_seqs * self.pages_per_seq()
        kv = {"f32": DTYPE_F32, "bf16": DTYPE_BF16}[self.kv_dtype]
        rv = {"split_half": ROPE_SPLIT_HALF, "interleaved": ROPE_INTERLEAVED}[self.rope_variant]
        return _lib.Config(self.n_layers, self.hidden_size, self.n_heads, self.n_kv_heads, self.head_dim,
                           self.max_seq_len, self.max_seqs, PAGE_SIZE, n_pages, kv, rv, float(self.rope_theta),
                           float(self.softmax_scale or 0.0))


def compute_rope_freqs(head_dim: int, max_seq_len: int, rope_theta: float):
    """compute_rope_freqs (src/oomllama_turbo.rs:376-396): (sin, cos) f32 CPU
    tensors [max_seq_len, head_dim/2], computed by the library's host code."""
    if head_dim != HEAD_DIM:
        raise ValueError("head_dim must be 128")
    L = _lib.load()
    cos = torch.empty(max_seq_len, head_dim // 2, dtype=torch.float32)
    sin = torch.empty_like(cos)
    check(None, L.oomattn_compute_rope_table(ctypes.c_float(rope_theta), head_dim, 0, max_seq_len,
                                             _ptr(cos), _ptr(sin)))
    return sin, cos


class TurboEngine:
    """TurboEngine (src/oomllama_turbo.rs:519-787) on one GPU."""

    def __init__(self, config: TurboConfig, device: int = 0, assign_pages: bool = True):
        self.config = config
        self.device = int(device)
        self._L = _lib.load()
        cfg = config.to_c()
        self._n_pages = cfg.n_pages
        ctx = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            stream = torch.cuda.current_stream().cuda_stream
            code = self._L.oomattn_create(ctypes.byref(cfg), self.device, ctypes.c_void_p(stream), ctypes.byref(ctx))
        if code != 0:
            raise _lib.OomAttnError(code, "oomattn_create rejected the configuration or failed to allocate")
        self._ctx = ctx
        if assign_pages:
            pps = config.pages_per_seq()
            if self._n_pages >= config.max_seqs * pps:
                for s in range(config.max_seqs):
                    self.set_block_table(s, range(s * pps, (s + 1) * pps))

    # ------------------------------------------------------------ lifecycle
    def close(self):
        if getattr(self, "_ctx", None):
            self._L.oomattn_destroy(self._ctx)
            self._ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _bind_stream(self):
        s = torch.cuda.current_stream(self.device).cuda_stream
        self._L.oomattn_set_stream(self._ctx, ctypes.c_void_p(s))

    def sync(self):
        """Wait for queued work; raises on a device-side timeout or index-check failure."""
        self._bind_stream()
        check(self._ctx, self._L.oomattn_sync(self._ctx))

    def set_wait_limit(self, timeout_ns: int):
        """Limit of the kernels' bounded device waits (default 2 s)."""
        check(self._ctx, self._L.oomattn_set_wait_limit(self._ctx, int(timeout_ns)))

    def set_test_flags(self, flags: int):
        """Test-only launch flags (_lib.TEST_DROP_DECODE_COPIES, _lib.TEST_DROP_LINEAR_COPIES); 0 in normal use."""
        check(self._ctx, self._L.oomattn_set_test_flags(self._ctx, int(flags)))

    def reset(self):
        """TurboEngine::reset (src/oomllama_turbo.rs:726-728)."""
        check(self._ctx, self._L.oomattn_reset(self._ctx))

    def seq_len(self, layer: int = 0, seq: int = 0) -> int:
        """TurboEngine::seq_len (src/oomllama_turbo.rs:731-733), per layer and sequence."""
        out = ctypes.c_int32()
        check(self._ctx, self._L.oomattn_seq_len(self._ctx, layer, seq, ctypes.byref(out)))
        return out.value

    # ------------------------------------------------------------ cache
    def set_block_table(self, seq: int, pages):
        pages = list(pages)
        check(self._ctx, self._L.oomattn_set_block_table(self._ctx, seq, int_array(pages), len(pages)))

    def set_position_offset(self, seq: int, offset: int):
        check(self._ctx, self._L.oomattn_set_position_offset(self._ctx, seq, offset))

    def set_seq_len(self, layer: int, seq: int, length: int):
        check(self._ctx, self._L.oomattn_set_seq_len(self._ctx, layer, seq, length))

    def kv_pool(self):
        """(k_pool, v_pool) device tensors [n_layers, n_pages+1, n_kv, 16, 128] aliasing the pools."""
        kp, vp = ctypes.c_void_p(), ctypes.c_void_p()
        check(self._ctx, self._L.oomattn_kv_pool(self._ctx, ctypes.byref(kp), ctypes.byref(vp)))
        c = self.config
        shape = (c.n_layers, self._n_pages + 1, c.n_kv_heads, PAGE_SIZE, HEAD_DIM)
        dt = torch.bfloat16 if c.kv_dtype == "bf16" else torch.float32
        return _alias(kp.value, shape, dt, self.device), _alias(vp.value, shape, dt, self.device)

    def kv_write(self, layer: int, seq: int, k: torch.Tensor, v: torch.Tensor):
        """Append already-rotated rows k, v [n, n_kv, 128] (LayerKVCache::append, :41-55)."""
        n = k.shape[0]
        nk = self.config.n_kv_heads * HEAD_DIM
        _dev(k, "k", self.device, numel=n * nk)
        _dev(v, "v", self.device, dtype=k.dtype, numel=n * nk)
        self._bind_stream()
        check(self._ctx, self._L.oomattn_kv_write(self._ctx, layer, seq, _ptr(k), _ptr(v), n, _dtype_code(k)))

    def kv_read(self, layer: int, seq: int):
        """LayerKVCache::get (src/oomllama_turbo.rs:57-63): host tensors [n_kv, L, 128]."""
        L_ = self.seq_len(layer, seq)
        dt = torch.bfloat16 if self.config.kv_dtype == "bf16" else torch.float32
        k = torch.empty(self.config.n_kv_heads, L_, HEAD_DIM, dtype=dt)
        v = torch.empty_like(k)
        self._bind_stream()
        check(self._ctx, self._L.oomattn_kv_read(self._ctx, layer, seq, _ptr(k), _ptr(v)))
        return k, v

    # ------------------------------------------------------------ K-A
    def rope_append(self, layer: int, seq_ids, q, k, v, bq=None, bk=None, bv=None, q_out_dtype=torch.float32):
        """Bias + RoPE + append for projected rows; q [T, Hq*128], k/v [T, Hkv*128]
        with T = len(seq_ids) * n_new.  Returns the rotated q [T, Hq, 128]."""
        seq_ids = list(seq_ids)
        T = q.shape[0]
        if T % len(seq_ids):
            raise ValueError("token count is not a multiple of the number of sequences")
        n_new = T // len(seq_ids)
        c = self.config
        _dev(q, "q", self.device, numel=T * c.n_heads * HEAD_DIM)
        _dev(k, "k", self.device, dtype=q.dtype, numel=T * c.n_kv_heads * HEAD_DIM)
        _dev(v, "v", self.device, dtype=q.dtype, numel=T * c.n_kv_heads * HEAD_DIM)
        for b, n in ((bq, c.n_heads), (bk, c.n_kv_heads), (bv, c.n_kv_heads)):
            if b is not None:
                _dev(b, "bias", self.device, dtype=torch.float32, numel=n * HEAD_DIM)
        q_out = torch.empty(T, c.n_heads, HEAD_DIM, dtype=q_out_dtype, device=q.device)
        self._bind_stream()
        check(self._ctx, self._L.oomattn_rope_append(
            self._ctx, layer, len(seq_ids), int_array(seq_ids), n_new, _ptr(q), _ptr(k), _ptr(v), _dtype_code(q),
            _ptr(bq), _ptr(bk), _ptr(bv), _ptr(q_out), _DT[q_out_dtype]))
        return q_out

    def rope_q(self, positions, q, bq=None, q_out_dtype=torch.float32, out=None):
        """RoPE of q rows [R, Hq*128] at explicit positions, nothing appended (the q half of
        TurboEngine::apply_rope, src/oomllama_turbo.rs:737-786).  Returns [R, Hq, 128]."""
        positions = list(positions)
        R = len(positions)
        c = self.config
        _dev(q, "q", self.device, numel=R * c.n_heads * HEAD_DIM)
        if bq is not None:
            _dev(bq, "bq", self.device, dtype=torch.float32, numel=c.n_heads * HEAD_DIM)
        if out is None:
            out = torch.empty(R, c.n_heads, HEAD_DIM, dtype=q_out_dtype, device=q.device)
        self._bind_stream()
        check(self._ctx, self._L.oomattn_rope_q(self._ctx, R, int_array(positions), _ptr(q), _dtype_code(q), _ptr(bq),
                                                _ptr(out), _DT[out.dtype]))
        return out

    def qkv_rope_append(self, layer: int, seq_ids, x, wq, wk, wv, bq=None, bk=None, bv=None,
                        q_out_dtype=torch.float32):
        """QKV projection + bias + RoPE + append (src/oomllama_turbo.rs:638-681).
        x [T, hidden] f32; weights [out, hidden] f32 or bf16."""
        seq_ids = list(seq_ids)
        c = self.config
        T = x.shape[0]
        n_new = T // len(seq_ids)
        H = c.hidden_size
        _dev(x, "x", self.device, dtype=torch.float32, numel=T * H)
        _dev(wq, "wq", self.device, numel=c.n_heads * HEAD_DIM * H)
        _dev(wk, "wk", self.device, dtype=wq.dtype, numel=c.n_kv_heads * HEAD_DIM * H)
        _dev(wv, "wv", self.device, dtype=wq.dtype, numel=c.n_kv_heads * HEAD_DIM * H)
        q_out = torch.empty(T, c.n_heads, HEAD_DIM, dtype=q_out_dtype, device=x.device)
        self._bind_stream()
        check(self._ctx, self._L.oomattn_qkv_rope_append(
            self._ctx, layer, len(seq_ids), int_array(seq_ids), n_new, _ptr(x), _ptr(wq), _ptr(wk), _ptr(wv),
            _dtype_code(wq), _ptr(bq), _ptr(bk), _ptr(bv), _ptr(q_out), _DT[q_out_dtype]))
        return q_out

    # ------------------------------------------------------------ K-B / K-C
    def decode(self, layer: int, seq_ids, q, lens=None, with_lse: bool = False, out=None, lse=None):
        """One query row per entry of seq_ids over the paged cache.
        q [rows, Hq, 128] f32 (rotated) -> out [rows, Hq, 128] f32 (, lse [rows, Hq])."""
        seq_ids = list(seq_ids)
        c = self.config
        rows = len(seq_ids)
        _dev(q, "q", self.device, dtype=torch.float32, numel=rows * c.n_heads * HEAD_DIM)
        if out is None:
            out = torch.empty(rows, c.n_heads, HEAD_DIM, dtype=torch.float32, device=q.device)
        if with_lse and lse is None:
            lse = torch.empty(rows, c.n_heads, dtype=torch.float32, device=q.device)
        self._bind_stream()
        check(self._ctx, self._L.oomattn_decode(
            self._ctx, layer, rows, int_array(seq_ids), None if lens is None else int_array(lens), _ptr(q),
            _ptr(out), _ptr(lse) if with_lse else None))
        return (out, lse) if with_lse else out

    def decode_packed(self, layer: int, seq_ids, q, lens=None, out=None):
        """decode() with (O, lse) packed per (row, q head) for one collective:
        -> [rows, Hq, PACKED_STRIDE] f32, O in [..., :128], natural-log lse in [..., 128]."""
        seq_ids = list(seq_ids)
        c = self.config
        rows = len(seq_ids)
        _dev(q, "q", self.device, dtype=torch.float32, numel=rows * c.n_heads * HEAD_DIM)
        if out is None:
            out = torch.empty(rows, c.n_heads, _lib.PACKED_STRIDE, dtype=torch.float32, device=q.device)
        else:
            _dev(out, "out", self.device, dtype=torch.float32, numel=rows * c.n_heads * _lib.PACKED_STRIDE)
        self._bind_stream()
        check(self._ctx, self._L.oomattn_decode_packed(
            self._ctx, layer, rows, int_array(seq_ids), None if lens is None else int_array(lens), _ptr(q),
            _ptr(out)))
        return out

    def merge_packed(self, packed: torch.Tensor, n_parts: int, out=None, lse=None):
        """LSE merge of packed partials [P, R, PACKED_STRIDE] -> (out [R, 128], lse [R])."""
        R = packed.numel() // (n_parts * _lib.PACKED_STRIDE)
        _dev(packed, "packed", self.device, dtype=torch.float32, numel=n_parts * R * _lib.PACKED_STRIDE)
        out = torch.empty(R, HEAD_DIM, dtype=torch.float32, device=packed.device) if out is None else out
        _dev(out, "out", self.device, dtype=torch.float32, numel=R * HEAD_DIM)
        self._bind_stream()
        check(self._ctx, self._L.oomattn_merge_packed(self._ctx, n_parts, R, _ptr(packed), _ptr(out), _ptr(lse)))
        return out, lse

    def prefill(self, layer: int, seq: int, q, out_dtype=torch.float32, with_lse: bool = False, out=None,
                blocks=None):
        """Causal attention of the n_new newest tokens of `seq` (bf16 cache).
        q [n_new, Hq, 128] bf16 (rotated) -> out [n_new, Hq, 128].  `blocks`: optional list of
        (lo, hi) ranges of 256-row query blocks to compute (the others' rows are not written)."""
        c = self.config
        n_new = q.shape[0]
        _dev(q, "q", self.device, dtype=torch.bfloat16, numel=n_new * c.n_heads * HEAD_DIM)
        if out is None:
            out = torch.empty(n_new, c.n_heads, HEAD_DIM, dtype=out_dtype, device=q.device)
        lse = torch.empty(n_new, c.n_heads, dtype=torch.float32, device=q.device) if with_lse else None
        self._bind_stream()
        if blocks is None:
            check(self._ctx, self._L.oomattn_prefill(self._ctx, layer, seq, n_new, _ptr(q), _ptr(out),
                                                     _DT[out.dtype], _ptr(lse)))
        else:
            flat = [int(x) for lo_hi in blocks for x in lo_hi]
            check(self._ctx, self._L.oomattn_prefill_blocks(self._ctx, layer, seq, n_new, _ptr(q), _ptr(out),
                                                            _DT[out.dtype], _ptr(lse), len(blocks),
                                                            int_array(flat)))
        return (out, lse) if with_lse else out

    def merge_partials(self, parts: torch.Tensor, lses: torch.Tensor):
        """LSE merge of split-context partials: parts [P, R, 128], lses [P, R] -> (out [R, 128], lse [R])."""
        P, R = lses.shape
        _dev(parts, "parts", self.device, dtype=torch.float32, numel=P * R * HEAD_DIM)
        _dev(lses, "lses", self.device, dtype=torch.float32)
        out = torch.empty(R, HEAD_DIM, dtype=torch.float32, device=parts.device)
        lse = torch.empty(R, dtype=torch.float32, device=parts.device)
        self._bind_stream()
        check(self._ctx, self._L.oomattn_merge_partials(self._ctx, P, R, _ptr(parts), _ptr(lses), _ptr(out),
                                                        _ptr(lse)))
        return out, lse

    # ------------------------------------------------------------ the layer step
    def attention_forward_with_bias(self, layer_idx: int, x, wq, wk, wv, wo, bq=None, bk=None, bv=None):
        """TurboEngine::attention_forward_with_bias (src/oomllama_turbo.rs:618-723).
        x [B, S, hidden] f32, weights [out, in] f32 -> [B, S, o_out] f32."""
        c = self.config
        B, S, H = x.shape
        if H != c.hidden_size:
            raise ValueError(f"hidden size {H} != config {c.hidden_size}")
        o_out = wo.shape[0]
        _dev(x, "x", self.device, dtype=torch.float32)
        for name, w, n in (("wq", wq, c.n_heads), ("wk", wk, c.n_kv_heads), ("wv", wv, c.n_kv_heads)):
            _dev(w, name, self.device, dtype=torch.float32, numel=n * HEAD_DIM * H)
        _dev(wo, "wo", self.device, dtype=torch.float32, numel=o_out * c.n_heads * HEAD_DIM)
        for name, b, n in (("bq", bq, c.n_heads), ("bk", bk, c.n_kv_heads), ("bv", bv, c.n_kv_heads)):
            if b is not None:
                _dev(b, name, self.device, dtype=torch.float32, numel=n * HEAD_DIM)
        out = torch.empty(B, S, o_out, dtype=torch.float32, device=x.device)
        self._bind_stream()
        check(self._ctx, self._L.oomattn_attention_forward_with_bias(
            self._ctx, layer_idx, B, S, _ptr(x), _ptr(wq), _ptr(wk), _ptr(wv), _ptr(wo), o_out, _ptr(bq), _ptr(bk),
            _ptr(bv), _ptr(out)))
        return out


    def linear(self, x: torch.Tensor, w: torch.Tensor, bias=None, out=None):
        """x @ W^T (+ bias) for f32 activations and f32 or bf16 weights [out, in] (candle's matmul with the
        transposed weight, src/oomllama_turbo.rs:643-645, :715-720): x [T, in] -> [T, out] f32."""
        if x.dim() != 2 or w.dim() != 2 or x.shape[1] != w.shape[1]:
            raise ValueError(f"x {tuple(x.shape)} and w {tuple(w.shape)} do not match")
        _dev(x, "x", self.device, dtype=torch.float32)
        _dev(w, "w", self.device)
        T, (rows, cols) = x.shape[0], w.shape
        if bias is not None:
            _dev(bias, "bias", self.device, dtype=torch.float32, numel=rows)
        out = (torch.empty(T, rows, dtype=torch.float32, device=x.device) if out is None
               else _dev(out, "out", self.device, dtype=torch.float32, numel=T * rows))
        self._bind_stream()
        check(self._ctx, self._L.oomattn_linear(self._ctx, _ptr(x), _ptr(w), _dtype_code(w), T, rows, cols,
                                                _ptr(bias), _ptr(out)))
        return out

    # ------------------------------------------------------------ Q8 weights (K-E)
    def q8_linear(self, w: "Q8Matrix", x: torch.Tensor, bias=None, out=None):
        """x @ W^T (+ bias) for a resident Q8 matrix: x [T, cols] f32 -> [T, rows] f32.
        Replaces dequantize-to-f32-then-matmul (src/quant.rs:413-468, src/oomllama.rs:425-439,
        src/oom_inference.rs:168-180) without materialising W."""
        if x.dim() != 2 or x.shape[1] != w.cols:
            raise ValueError(f"x must be [T, {w.cols}], got {tuple(x.shape)}")
        _dev(x, "x", self.device, dtype=torch.float32)
        if bias is not None:
            _dev(bias, "bias", self.device, dtype=torch.float32, numel=w.rows)
        T = x.shape[0]
        if out is None:
            out = torch.empty(T, w.rows, dtype=torch.float32, device=x.device)
        else:
            _dev(out, "out", self.device, dtype=torch.float32, numel=T * w.rows)
        self._bind_stream()
        check(self._ctx, self._L.oomattn_q8_linear(self._ctx, ctypes.byref(w.c_struct()), _ptr(x), T, _ptr(bias),
                                                   _ptr(out)))
        return out


    # ------------------------------------------------------------ the layer steps around attention
    def rmsnorm(self, x: torch.Tensor, weight: torch.Tensor, eps: float, out=None):
        """GhostRMSNorm::forward (src/oomllama.rs:200-211): x [T, H] f32 -> [T, H]."""
        T, H = x.shape
        _dev(x, "x", self.device, dtype=torch.float32)
        _dev(weight, "weight", self.device, dtype=torch.float32, numel=H)
        out = torch.empty_like(x) if out is None else _dev(out, "out", self.device, dtype=torch.float32, numel=T * H)
        self._bind_stream()
        check(self._ctx, self._L.oomattn_rmsnorm(self._ctx, _ptr(x), _ptr(weight), float(eps), T, H, _ptr(out)))
        return out

    def q8_mlp(self, gate: "Q8Matrix", up: "Q8Matrix", down: "Q8Matrix", x: torch.Tensor, residual=None, out=None):
        """GhostMlp::forward (src/oomllama.rs:230-242) plus the residual add: down(silu(gate x) * up x) (+ residual)."""
        T, H = x.shape
        _dev(x, "x", self.device, dtype=torch.float32)
        if residual is not None:
            _dev(residual, "residual", self.device, dtype=torch.float32, numel=T * down.rows)
        out = torch.empty(T, down.rows, dtype=torch.float32, device=x.device) if out is None else out
        self._bind_stream()
        check(self._ctx, self._L.oomattn_q8_mlp(self._ctx, ctypes.byref(gate.c_struct()), ctypes.byref(up.c_struct()),
                                                ctypes.byref(down.c_struct()), _ptr(x), T, _ptr(residual), _ptr(out)))
        return out

    def decoder_layer_q8(self, layer: int, seq_ids, x: torch.Tensor, w: "Q8DecoderLayer", out=None):
        """GhostDecoderLayer::forward_turbo (src/oomllama.rs:387-402) for one new token per sequence:
        x [B, hidden] f32 -> [B, hidden]; appends each sequence's token to the cache of `layer`."""
        B, H = x.shape
        _dev(x, "x", self.device, dtype=torch.float32)
        out = torch.empty_like(x) if out is None else _dev(out, "out", self.device, dtype=torch.float32, numel=B * H)
        self._bind_stream()
        ids = int_array(seq_ids)
        check(self._ctx, self._L.oomattn_decoder_layer_q8(self._ctx, layer, B, ids, _ptr(x),
                                                          ctypes.byref(w.c_struct()), _ptr(out)))
        return out

    def q8_repack(self, blocks: torch.Tensor, n_values: int, rows: int = None, cols: int = None):
        """Device-side repack of one Q8 tensor's .oom block stream (uint8 device tensor, any offset) into a
        resident Q8Matrix [rows][cols] (src/gguf2oom.rs:782-829 layout; the result equals q8_unpack's)."""
        _dev(blocks, "blocks", self.device, dtype=torch.uint8)
        nb = (n_values + 255) // 256
        q = torch.empty(n_values, dtype=torch.uint8, device=self.device)
        scale = torch.empty(nb, dtype=torch.float32, device=self.device)
        mn = torch.empty(nb, dtype=torch.float32, device=self.device)
        self._bind_stream()
        check(self._ctx, self._L.oomattn_q8_repack(self._ctx, _ptr(blocks), blocks.numel(), n_values, _ptr(q),
                                                   _ptr(scale), _ptr(mn)))
        return Q8Matrix(q, scale, mn, rows if rows is not None else 1, cols if cols is not None else n_values)

    def embed_q8(self, emb: "Q8Matrix", token_ids: torch.Tensor, out=None):
        """embed_w.embedding(tokens) (src/oomllama.rs:508-515) on a resident Q8 table: int32 ids [T] ->
        f32 [T, hidden]."""
        T = token_ids.numel()
        _dev(token_ids, "token_ids", self.device, dtype=torch.int32)
        out = (torch.empty(T, emb.cols, dtype=torch.float32, device=self.device) if out is None
               else _dev(out, "out", self.device, dtype=torch.float32, numel=T * emb.cols))
        self._bind_stream()
        check(self._ctx, self._L.oomattn_embed_q8(self._ctx, ctypes.byref(emb.c_struct()), _ptr(token_ids), T,
                                                  _ptr(out)))
        return out

    def argmax(self, logits: torch.Tensor, out=None):
        """The greedy pick of the generation loop (src/oomllama.rs:1000-1003): f32 [R, n] -> int32 [R]."""
        R, n = logits.shape
        _dev(logits, "logits", self.device, dtype=torch.float32)
        out = (torch.empty(R, dtype=torch.int32, device=self.device) if out is None
               else _dev(out, "out", self.device, dtype=torch.int32, numel=R))
        self._bind_stream()
        check(self._ctx, self._L.oomattn_argmax(self._ctx, _ptr(logits), R, n, _ptr(out)))
        return out

    def decode_step_q8(self, model: "Q8Model", seq_ids, tokens: torch.Tensor, next_tokens=None, logits=None):
        """OomLlamaModel::forward_turbo (src/oomllama.rs:504-553) for one new token per sequence plus the greedy
        pick: int32 tokens [B] -> int32 next [B] (may be `tokens` itself).  `logits` [B, vocab] f32 receives the
        LM head output when given.  Every layer's cache grows by one token per sequence."""
        B = tokens.numel()
        _dev(tokens, "tokens", self.device, dtype=torch.int32)
        nxt = (torch.empty(B, dtype=torch.int32, device=self.device) if next_tokens is None
               else _dev(next_tokens, "next_tokens", self.device, dtype=torch.int32, numel=B))
        if logits is not None:
            _dev(logits, "logits", self.device, dtype=torch.float32, numel=B * model.lm_head.rows)
        self._bind_stream()
        ids = int_array(seq_ids)
        check(self._ctx, self._L.oomattn_decode_step_q8(self._ctx, ctypes.byref(model.c_struct()), B, ids,
                                                        _ptr(tokens), _ptr(nxt),
                                                        None if logits is None else _ptr(logits)))
        return nxt

    def prefill_step_q8(self, model: "Q8Model", seq_ids, tokens: torch.Tensor, next_tokens=None, logits=None):
        """The prompt through the whole model (OomLlamaModel::forward_turbo over every prompt token,
        src/oomllama.rs:504-553, 969-970): int32 tokens [B, n_new] -> int32 next [B], the greedy pick after each
        sequence's last prompt token.  Every layer's cache grows by n_new tokens per sequence (bf16 cache)."""
        B, n_new = tokens.shape
        _dev(tokens, "tokens", self.device, dtype=torch.int32)
        nxt = (torch.empty(B, dtype=torch.int32, device=self.device) if next_tokens is None
               else _dev(next_tokens, "next_tokens", self.device, dtype=torch.int32, numel=B))
        if logits is not None:
            _dev(logits, "logits", self.device, dtype=torch.float32, numel=B * model.lm_head.rows)
        self._bind_stream()
        check(self._ctx, self._L.oomattn_prefill_step_q8(self._ctx, ctypes.byref(model.c_struct()), B,
                                                         int_array(seq_ids), n_new, _ptr(tokens), _ptr(nxt),
                                                         None if logits is None else _ptr(logits)))
        return nxt


def q8_unpack(stream, n_values: int):
    """Unpack one .oom Q8 tensor's block stream ([f32 scale][f32 min][u32 len][bytes] per 256 values,
    src/gguf2oom.rs:823-826) into host arrays (q uint8 [n_values], scale, min f32 [n_blocks])."""
    import numpy as np
    buf = np.frombuffer(bytes(stream) if not isinstance(stream, np.ndarray) else stream.tobytes(), dtype=np.uint8)
    nb = (n_values + 255) // 256
    q = np.empty(max(1, n_values), np.uint8)
    scale = np.empty(max(1, nb), np.float32)
    mn = np.empty(max(1, nb), np.float32)
    err = ctypes.create_string_buffer(256)
    rc = _lib.load().oomattn_q8_unpack(buf.ctypes.data_as(ctypes.c_void_p), buf.size, n_values,
                                       q.ctypes.data_as(ctypes.c_void_p), scale.ctypes.data_as(ctypes.c_void_p),
                                       mn.ctypes.data_as(ctypes.c_void_p), err, 256)
    if rc != _lib.OK:
        raise _lib.OomAttnError(rc, err.value.decode(errors="replace"))
    return q[:n_values], scale[:nb], mn[:nb]


def oom_scan(image):
    """OomLoader::load's metadata scan (src/quant.rs:320-367) of an .oom file image (bytes, or a uint8 numpy
    array / memory map): {name: OomTensor} in file order."""
    import numpy as np
    buf = image if isinstance(image, np.ndarray) else np.frombuffer(image, dtype=np.uint8)
    L = _lib.load()
    err = ctypes.create_string_buffer(256)
    n = ctypes.c_int32(0)
    rc = L.oomattn_oom_scan(buf.ctypes.data_as(ctypes.c_void_p), buf.size, None, 0, ctypes.byref(n), err, 256)
    if rc != _lib.OK:
        raise _lib.OomAttnError(rc, err.value.decode(errors="replace"))
    metas = (_lib.OomTensor * max(1, n.value))()
    rc = L.oomattn_oom_scan(buf.ctypes.data_as(ctypes.c_void_p), buf.size, metas, n.value, ctypes.byref(n), err, 256)
    if rc != _lib.OK:
        raise _lib.OomAttnError(rc, err.value.decode(errors="replace"))
    out = {}
    for m in metas[:n.value]:
        name = bytes(buf[m.name_offset:m.name_offset + m.name_len]).decode("utf-8")
        out[name] = m
    return out


class OomFile:
    """An .oom file for GPU-resident inference: the metadata scan of OomLoader::load (src/quant.rs:320-367) and,
    per tensor, one upload of its block stream followed by the device repack into a resident Q8Matrix -- the
    weights are never dequantised to f32 (src/oomllama.rs:425-439 dequantises and uploads on every call)."""

    def __init__(self, path_or_image):
        import os
        import numpy as np
        if isinstance(path_or_image, (str, os.PathLike)):
            self.image = np.memmap(path_or_image, dtype=np.uint8, mode="r")
        elif isinstance(path_or_image, (bytes, bytearray)):
            self.image = np.frombuffer(path_or_image, dtype=np.uint8)
        else:
            self.image = path_or_image
        self.tensors = oom_scan(self.image)

    def blocks(self, name: str):
        m = self.tensors[name]
        return self.image[m.data_offset:m.data_offset + m.data_bytes]

    def q8_matrix(self, engine: "TurboEngine", name: str, rows: int, cols: int) -> "Q8Matrix":
        """Upload the tensor's blocks (padded to a 4-byte multiple) and repack them on the device."""
        m = self.tensors[name]
        if m.quant_type != 8:
            raise ValueError(f"{name}: quant type {m.quant_type}, not Q8")
        if m.total_values != rows * cols:
            raise ValueError(f"{name}: {m.total_values} values, not {rows} x {cols}")
        import numpy as np
        raw = self.blocks(name)
        dev = torch.empty((raw.size + 3) // 4 * 4, dtype=torch.uint8, device=engine.device)
        dev[:raw.size].copy_(torch.from_numpy(np.array(raw)))  # a writable host copy of the (read-only) image
        return engine.q8_repack(dev[:raw.size], rows * cols, rows, cols)

    def f32_tensor(self, name: str, device=None) -> torch.Tensor:
        """A raw f32 tensor (norms, biases): one block whose data are the values (src/gguf2oom.rs:835-861)."""
        import numpy as np
        m = self.tensors[name]
        if m.quant_type != 0:
            raise ValueError(f"{name}: quant type {m.quant_type}, not f32")
        raw = self.image[m.data_offset + 12:m.data_offset + 12 + 4 * m.total_values]
        t = torch.from_numpy(np.frombuffer(raw.tobytes(), dtype=np.float32).copy())
        return t if device is None else t.to(device)


@dataclass
class Q8Matrix:
    """A Q8 matrix [rows][cols] ([out][in]) resident on the device: q uint8 [rows*cols], scale and min f32 per
    256-value block of the row-major flattening (src/quant.rs:201-224)."""
    q: torch.Tensor
    scale: torch.Tensor
    min: torch.Tensor
    rows: int
    cols: int

    @staticmethod
    def from_oom_stream(stream, rows: int, cols: int, device: int = 0) -> "Q8Matrix":
        """Unpack a .oom Q8 block stream on the host and upload it once."""
        q, scale, mn = q8_unpack(stream, rows * cols)
        dev = f"cuda:{device}"
        return Q8Matrix(torch.from_numpy(q.copy()).to(dev), torch.from_numpy(scale.copy()).to(dev),
                        torch.from_numpy(mn.copy()).to(dev), rows, cols)

    def c_struct(self) -> _lib.Q8Matrix:
        return _lib.Q8Matrix(self.q.data_ptr(), self.scale.data_ptr(), self.min.data_ptr(), self.rows, self.cols)


def _alias(ptr: int, shape, dtype, device: int) -> torch.Tensor:
    """A torch tensor viewing library-owned device memory (no copy, no ownership)."""
    numel = 1
    for s in shape:
        numel *= s
    esize = torch.tensor([], dtype=dtype).element_size()

    class _Holder:
        __cuda_array_interface__ = {
            "shape": (numel * esize,), "typestr": "|u1", "data": (ptr, False), "version": 3, "strides": None,
        }

    with torch.cuda.device(device):
        raw = torch.as_tensor(_Holder(), device=f"cuda:{device}")
    return raw.view(dtype).view(*shape)


@dataclass
class Q8DecoderLayer:
    """One decoder layer's resident weights (GhostDecoderLayer, src/oomllama.rs:366-402): Q8 projections and MLP,
    f32 attention biases (or None) and RMSNorm weights."""
    q: Q8Matrix
    k: Q8Matrix
    v: Q8Matrix
    o: Q8Matrix
    gate: Q8Matrix
    up: Q8Matrix
    down: Q8Matrix
    input_norm: torch.Tensor
    post_norm: torch.Tensor
    eps: float
    bq: torch.Tensor = None
    bk: torch.Tensor = None
    bv: torch.Tensor = None

    def c_struct(self) -> _lib.Q8Layer:
        p = lambda t: None if t is None else t.data_ptr()  # noqa: E731
        return _lib.Q8Layer(self.q.c_struct(), self.k.c_struct(), self.v.c_struct(), self.o.c_struct(),
                            self.gate.c_struct(), self.up.c_struct(), self.down.c_struct(), p(self.bq), p(self.bk),
                            p(self.bv), p(self.input_norm), p(self.post_norm), self.eps)


@dataclass
class Q8Model:
    """A whole model's resident weights (OomLlamaModel, src/oomllama.rs:462-500): decoder layers, the Q8
    embedding table and LM head [vocab][hidden], and the final RMSNorm weight."""
    layers: list
    embed: Q8Matrix
    lm_head: Q8Matrix
    final_norm: torch.Tensor
    eps: float

    @classmethod
    def from_oom(cls, oom: "OomFile", engine: "TurboEngine", n_layers: int, inter: int, vocab: int,
                 eps: float = 1e-6) -> "Q8Model":
        """A model's resident weights from an .oom file, by the converter's tensor names
        (map_tensor_name, src/gguf2oom.rs:936-979): Q8 projections, embedding and LM head; f32 norms and
        biases (src/gguf2oom.rs:1027-1037).  Shapes come from the engine's configuration.  A file without
        lm_head.weight (tied embeddings) uses the embedding table as the LM head."""
        c = engine.config
        H, nq, nkv = c.hidden_size, c.n_heads * HEAD_DIM, c.n_kv_heads * HEAD_DIM
        dev = engine.device
        f32 = lambda name: oom.f32_tensor(name, dev) if name in oom.tensors else None  # noqa: E731
        layers = []
        for i in range(n_layers):
            p = f"model.layers.{i}."
            m = lambda n, r, k: oom.q8_matrix(engine, p + n, r, k)  # noqa: E731
            layers.append(Q8DecoderLayer(
                q=m("self_attn.q_proj.weight", nq, H), k=m("self_attn.k_proj.weight", nkv, H),
                v=m("self_attn.v_proj.weight", nkv, H), o=m("self_attn.o_proj.weight", H, nq),
                gate=m("mlp.gate_proj.weight", inter, H), up=m("mlp.up_proj.weight", inter, H),
                down=m("mlp.down_proj.weight", H, inter), input_norm=f32(p + "input_layernorm.weight"),
                post_norm=f32(p + "post_attention_layernorm.weight"), eps=eps, bq=f32(p + "self_attn.q_proj.bias"),
                bk=f32(p + "self_attn.k_proj.bias"), bv=f32(p + "self_attn.v_proj.bias")))
        embed = oom.q8_matrix(engine, "model.embed_tokens.weight", vocab, H)
        head = oom.q8_matrix(engine, "lm_head.weight", vocab, H) if "lm_head.weight" in oom.tensors else embed
        return cls(layers=layers, embed=embed, lm_head=head, final_norm=f32("model.norm.weight"), eps=eps)

    def c_struct(self) -> _lib.Q8Model:
        arr = (_lib.Q8Layer * len(self.layers))(*[l.c_struct() for l in self.layers])
        m = _lib.Q8Model(len(self.layers), ctypes.cast(arr, ctypes.POINTER(_lib.Q8Layer)), self.embed.c_struct(),
                         self.lm_head.c_struct(), self.final_norm.data_ptr(), self.eps)
        m._keep = arr  # the layer array lives as long as the struct
        return m

"""numpy front-end of the C oracle (oracle/attn_ref.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, by ``__graft_entry__.smoke()`` and
by the CPU-baseline leg of ``bench.py``.  The product package never imports it.

Parity status: UNPINNED -- the Rust reference cannot be built or run here and
its tests hold no golden vectors for this path; see the header of attn_ref.c.
Every function cites the reference code it restates (paths are relative to the
jaspertvdm/oomllama project root).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "liboomattn_oracle.so")
_lib = None

ROPE_SPLIT_HALF = 0
ROPE_INTERLEAVED = 1

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(dtype=np.int64, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")


def build(force: bool = False) -> str:
    """Compile attn_ref.c with the committed Makefile (no-op when up to date)."""
    src = os.path.join(_HERE, "attn_ref.c")
    if force or not os.path.exists(_SO) or os.path.getmtime(_SO) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _SO


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_SO):
        build()
    L = ctypes.CDLL(_SO)
    c_int, c_float, c_void = ctypes.c_int, ctypes.c_float, None
    L.oracle_rope_table.argtypes = [c_float, c_int, c_int, c_int, _f32p, _f32p]
    L.oracle_rope_apply.argtypes = [_f32p, c_int, c_int, _f32p, _f32p, c_int]
    L.oracle_matvec_bias.argtypes = [_f32p, _f32p, ctypes.c_void_p, c_int, c_int, _f32p]
    L.oracle_attention_head.argtypes = [_f32p, _f32p, _f32p, c_int, c_int, c_float, _f32p, _f32p]
    L.oracle_attention_head.restype = c_float
    L.oracle_gqa_attention.argtypes = [_f32p, _f32p, _f32p, c_int, c_int, c_int, c_int, c_int, c_float, c_int,
                                       _f32p, ctypes.c_void_p]
    L.oracle_gqa_attention_rows.argtypes = [_f32p, _f32p, _f32p, c_int, c_int, c_int, c_int, c_int, c_float,
                                            c_int, c_int, _i32p, _i32p, _f32p]
    L.oracle_decode_batch.argtypes = [_f32p, _f32p, _f32p, _i64p, _i32p, c_int, c_int, c_int, c_int, c_float,
                                      c_int, _f32p]
    L.oracle_merge_partials.argtypes = [_f32p, _f32p, c_int, c_int, c_int, _f32p, ctypes.c_void_p]
    L.oracle_layer_attention.argtypes = [_f32p, c_int, c_int, c_int, _f32p, _f32p, _f32p, ctypes.c_void_p,
                                         ctypes.c_void_p, ctypes.c_void_p, c_int, c_int, c_int, c_int, _f32p,
                                         _f32p, c_int, _f32p, _f32p, c_int, c_float, _f32p]
    L.oracle_round_bf16.argtypes = [_f32p, ctypes.c_int64]
    L.oracle_f32_to_bf16.argtypes = [c_float]
    L.oracle_f32_to_bf16.restype = ctypes.c_uint16
    L.oracle_bf16_to_f32.argtypes = [ctypes.c_uint16]
    L.oracle_bf16_to_f32.restype = c_float
    L.oracle_omp_max_threads.restype = c_int
    _u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
    L.oracle_q8_stream_bytes.argtypes = [ctypes.c_int64]
    L.oracle_q8_stream_bytes.restype = ctypes.c_int64
    L.oracle_q8_quantize.argtypes = [_f32p, ctypes.c_int64, _u8p]
    L.oracle_q8_dequantize.argtypes = [_u8p, ctypes.c_int64, ctypes.c_int64, _f32p]
    L.oracle_q8_dequantize.restype = c_int
    L.oracle_linear.argtypes = [_f32p, c_int, _f32p, ctypes.c_void_p, c_int, c_int, _f32p]
    L.oracle_rmsnorm.argtypes = [_f32p, _f32p, c_float, c_int, c_int, _f32p]
    L.oracle_swiglu.argtypes = [_f32p, _f32p, ctypes.c_int64, _f32p]
    _lib = L
    return L


def _c(a, dt=np.float32):
    return np.ascontiguousarray(a, dtype=dt)


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def rope_table(theta: float, head_dim: int, n_pos: int, pos0: int = 0):
    """cos, sin tables [n_pos, head_dim/2] (oomllama_turbo.rs:753-761, :376-396)."""
    half = head_dim // 2
    c = np.empty((n_pos, half), np.float32)
    s = np.empty((n_pos, half), np.float32)
    lib().oracle_rope_table(float(theta), head_dim, pos0, n_pos, c, s)
    return c, s


def rope_apply(x, cos_row, sin_row, variant: int):
    """Rotate x [n_heads, d] (one token) -- apply_rope (interleaved,
    oomllama_turbo.rs:402-438) or split-half (:443-467, :773-783)."""
    x = _c(x).copy()
    nh, d = x.shape
    lib().oracle_rope_apply(x, nh, d, _c(cos_row), _c(sin_row), variant)
    return x


def rope_tokens(x, positions, cos_t, sin_t, variant: int):
    """Rotate x [T, n_heads, d], token t at positions[t]."""
    x = _c(x).copy()
    T, nh, d = x.shape
    L = lib()
    for t in range(T):
        row = x[t]
        L.oracle_rope_apply(row, nh, d, _c(cos_t[positions[t]]), _c(sin_t[positions[t]]), variant)
        x[t] = row
    return x


def matvec_bias(x, w, b=None):
    """y = x @ W^T + b for one row x (oom_inference.rs:168-180; bias :648-656)."""
    w = _c(w)
    out_f, in_f = w.shape
    y = np.empty(out_f, np.float32)
    bb = None if b is None else _c(b)
    lib().oracle_matvec_bias(_c(x), w, _ptr(bb), out_f, in_f, y)
    return y


def attention_head(q, k, v, scale=None):
    """oom_inference.rs:240-272: one head over k, v [L, d]; returns (out, lse)."""
    k = _c(k)
    L_, d = k.shape
    scale = 1.0 / np.sqrt(np.float32(d)) if scale is None else scale
    out = np.empty(d, np.float32)
    ws = np.empty(max(L_, 1), np.float32)
    lse = lib().oracle_attention_head(_c(q), k, _c(v), L_, d, np.float32(scale), ws, out)
    return out, lse


def gqa_attention(q, k, v, causal=True, scale=None, with_lse=False):
    """flash_attention_forward semantics (oomllama_turbo.rs:304-369).
    q [n_q, Hq, d]; k, v [Hkv, L, d]; returns out [n_q, Hq, d] (and lse [n_q, Hq])."""
    q, k, v = _c(q), _c(k), _c(v)
    n_q, hq, d = q.shape
    hkv, L_, _ = k.shape
    scale = float(1.0 / np.sqrt(np.float32(d))) if scale is None else scale
    out = np.empty((n_q, hq, d), np.float32)
    lse = np.empty((n_q, hq), np.float32) if with_lse else None
    lib().oracle_gqa_attention(q, k, v, n_q, L_, hq, hkv, d, np.float32(scale), int(causal), out, _ptr(lse))
    return (out, lse) if with_lse else out


def gqa_attention_rows(q, k, v, rows, heads, causal=True, scale=None):
    """gqa_attention for sampled (row, head) pairs only; returns [n_pairs, d]."""
    q, k, v = _c(q), _c(k), _c(v)
    n_q, hq, d = q.shape
    hkv, L_, _ = k.shape
    scale = float(1.0 / np.sqrt(np.float32(d))) if scale is None else scale
    rows, heads = _c(rows, np.int32), _c(heads, np.int32)
    out = np.empty((len(rows), d), np.float32)
    lib().oracle_gqa_attention_rows(q, k, v, n_q, L_, hq, hkv, d, np.float32(scale), int(causal), len(rows),
                                    rows, heads, out)
    return out


def decode_batch(q, k_list, v_list, n_threads=1, scale=None):
    """Batched one-token decode (oom_inference.rs:240-272 per (seq, head)).
    q [B, Hq, d]; k_list[b], v_list[b]: [Hkv, L_b, d]."""
    q = _c(q)
    B, hq, d = q.shape
    hkv = k_list[0].shape[0]
    Ls = np.array([k.shape[1] for k in k_list], np.int32)
    offs = np.zeros(B, np.int64)
    offs[1:] = np.cumsum([k.size for k in k_list])[:-1]
    K = np.concatenate([_c(k).ravel() for k in k_list])
    V = np.concatenate([_c(v).ravel() for v in v_list])
    scale = float(1.0 / np.sqrt(np.float32(d))) if scale is None else scale
    out = np.empty_like(q)
    lib().oracle_decode_batch(q, K, V, offs, Ls, B, hq, hkv, d, np.float32(scale), int(n_threads), out)
    return out


def merge_partials(parts, lses):
    """LSE merge of split-context partials: parts [P, R, d], lses [P, R]."""
    parts, lses = _c(parts), _c(lses)
    P, R, d = parts.shape
    out = np.empty((R, d), np.float32)
    lse = np.empty(R, np.float32)
    lib().oracle_merge_partials(parts, lses, P, R, d, out, _ptr(lse))
    return out, lse


def layer_attention(x, wq, wk, wv, bq, bk, bv, n_heads, n_kv, kc, vc, cos_t, sin_t, variant, kv_bf16=False):
    """TurboEngine::attention_forward_with_bias (oomllama_turbo.rs:618-723)
    up to the o_proj.  x [B, S, H]; kc, vc [B, Hkv, P, d] cache before the
    append.  Returns (out [B, S, Hq*d], kc_new, vc_new [B, Hkv, P+S, d])."""
    x = _c(x)
    B, S, H = x.shape
    _, _, P, d = kc.shape
    L_ = P + S
    kn = np.zeros((B, n_kv, L_, d), np.float32)
    vn = np.zeros((B, n_kv, L_, d), np.float32)
    kn[:, :, :P] = kc
    vn[:, :, :P] = vc
    out = np.empty((B, S, n_heads * d), np.float32)
    bq_, bk_, bv_ = [None if b is None else _c(b) for b in (bq, bk, bv)]
    scale = np.float32(1.0 / np.sqrt(np.float32(d)))
    lib().oracle_layer_attention(x, B, S, H, _c(wq), _c(wk), _c(wv), _ptr(bq_), _ptr(bk_), _ptr(bv_), n_heads,
                                 n_kv, d, P, kn, vn, int(kv_bf16), _c(cos_t), _c(sin_t), variant, scale, out)
    return out, kn, vn


def round_bf16(x):
    """Round f32 values to bf16 precision (RNE), returned as f32."""
    x = _c(x).copy()
    lib().oracle_round_bf16(x.reshape(-1), x.size)
    return x


def f32_to_bf16_bits(x):
    """f32 -> bf16 bit patterns (uint16), round to nearest even."""
    x = _c(x)
    u = x.view(np.uint32).astype(np.uint64)
    nan = ((u & 0x7F800000) == 0x7F800000) & ((u & 0x007FFFFF) != 0)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_bits_to_f32(h):
    """bf16 bit patterns -> f32 by a 16-bit shift (safetensors2oom.rs:32-39)."""
    return (np.asarray(h, np.uint16).astype(np.uint32) << 16).view(np.float32)


def q8_quantize(values) -> np.ndarray:
    """The .oom Q8 block stream of a flat f32 tensor (src/gguf2oom.rs:719-770)."""
    v = _c(values).ravel()
    out = np.empty(int(lib().oracle_q8_stream_bytes(v.size)), np.uint8)
    lib().oracle_q8_quantize(v, v.size, out)
    return out


def q8_dequantize(stream, n: int) -> np.ndarray:
    """Dequantise n values of a Q8 block stream (src/quant.rs:431-463 with :201-224)."""
    s = np.ascontiguousarray(stream, dtype=np.uint8)
    out = np.empty(max(1, n), np.float32)
    if lib().oracle_q8_dequantize(s, s.size, n, out) != 0:
        raise ValueError("malformed Q8 block stream")
    return out[:n]


def oom_image(tensors) -> bytes:
    """An .oom file image as the reference's writer produces it (src/gguf2oom.rs:708-716 header, :782-829 Q8
    tensors via q8_quantize, :835-861 raw f32 tensors): tensors = [(name, "q8" | "f32", values)]."""
    import struct
    out = bytearray(b"OOML" + struct.pack("<II", 1, len(tensors)))
    for name, kind, values in tensors:
        v = _c(values).ravel()
        nm = name.encode()
        out += struct.pack("<I", len(nm)) + nm
        if kind == "q8":
            out += struct.pack("<BII", 8, (v.size + 255) // 256, v.size) + q8_quantize(v).tobytes()
        else:
            out += struct.pack("<BII", 0, 1, v.size) + struct.pack("<ffI", 0.0, 0.0, 4 * v.size) + v.tobytes()
    return bytes(out)


def oom_scan(image):
    """OomLoader::load's metadata scan (src/quant.rs:320-367): [(name, quant_type, num_blocks, total_values,
    data_offset, data_bytes)] in file order.  The reference's loop stops at a truncated header or block; here
    that raises ValueError, matching the library's stricter scan."""
    b = bytes(image)
    if len(b) < 12 or b[:4] != b"OOML":
        raise ValueError("not an .oom file")
    count = int.from_bytes(b[8:12], "little")
    off, out = 12, []
    for _ in range(count):
        if off + 4 > len(b):
            raise ValueError("truncated header")
        nl = int.from_bytes(b[off:off + 4], "little")
        if off + 4 + nl + 9 > len(b):
            raise ValueError("truncated header")
        name = b[off + 4:off + 4 + nl].decode()
        off += 4 + nl
        qt = b[off]
        nb = int.from_bytes(b[off + 1:off + 5], "little")
        n = int.from_bytes(b[off + 5:off + 9], "little")
        off += 9
        start = off
        for _ in range(nb):  # skip the blocks by their length fields
            if off + 12 > len(b):
                raise ValueError("truncated block")
            ln = int.from_bytes(b[off + 8:off + 12], "little")
            if off + 12 + ln > len(b):
                raise ValueError("truncated block")
            off += 12 + ln
        out.append((name, qt, nb, n, start, off - start))
    return out


def linear(x, w, b=None):
    """x [T, cols] @ w[rows, cols]^T (+ b): the reference's matvec per token (oom_inference.rs:168-180)."""
    x, w = _c(x), _c(w)
    T, cols = x.shape
    rows = w.shape[0]
    y = np.empty((T, rows), np.float32)
    bb = None if b is None else _c(b)
    lib().oracle_linear(x, T, w, _ptr(bb), rows, cols, y)
    return y


def rmsnorm(x, w, eps):
    """GhostRMSNorm::forward (src/oomllama.rs:200-211): x [T, H]."""
    x = _c(x)
    T, H = x.shape
    out = np.empty_like(x)
    lib().oracle_rmsnorm(x, _c(w), np.float32(eps), T, H, out)
    return out


def swiglu(gate, up):
    """gate * sigmoid(gate) * up (src/oomllama.rs:235-238)."""
    g, u = _c(gate), _c(up)
    out = np.empty_like(g)
    lib().oracle_swiglu(g.ravel(), u.ravel(), g.size, out.reshape(-1))
    return out


def embedding(stream, vocab: int, hidden: int, ids) -> np.ndarray:
    """embed_w.embedding(tokens) of OomLlamaModel::forward_turbo (src/oomllama.rs:508-515) on a Q8 table
    [vocab][hidden] given as its block stream: the dequantised rows ids."""
    table = q8_dequantize(stream, vocab * hidden).reshape(vocab, hidden)
    return table[np.asarray(ids, np.int64)].copy()


def argmax(logits) -> np.ndarray:
    """The generation loop's greedy pick (src/oomllama.rs:973-976, :1000-1003), candle-core 0.9.1's argmax over
    the last axis: a scan from element 0 that moves only to a strictly larger value.  Equivalent vectorised form:
    NaN never compares larger, so NaNs become -inf and numpy's first-maximum argmax applies, except that a NaN in
    element 0 is never left."""
    x = np.array(logits, np.float32, ndmin=2)
    first_nan = np.isnan(x[:, 0])
    idx = np.argmax(np.where(np.isnan(x), -np.inf, x), axis=1).astype(np.int32)
    idx[first_nan] = 0
    return idx


def argmax_scan(row) -> int:
    """argmax as the literal strict-greater scan from element 0 (small rows; checks the vectorised form)."""
    best, bi = row[0], 0
    for i in range(1, len(row)):
        if row[i] > best:
            best, bi = row[i], i
    return bi


def decoder_layer_decode(x, w, kc, vc, lens, n_heads, n_kv, cos_t, sin_t, variant, kv_bf16=False):
    """GhostDecoderLayer::forward_turbo (src/oomllama.rs:387-402) for one new token per sequence:
    h = x + o(attention(rope(qkv(rmsnorm(x))))), out = h + mlp(rmsnorm(h)).  x [B, H]; w a dict of dequantised
    matrices q, k, v, o, gate, up, down, biases bq, bk, bv (or None), norms n1, n2 and eps; kc[b], vc[b]
    [lens[b], n_kv, d] the cached (rotated) keys and values, extended in place by the new token (rounded to
    bf16 when kv_bf16).  Returns out [B, H]."""
    x = _c(x)
    B = x.shape[0]
    d = w["q"].shape[0] // n_heads
    store = round_bf16 if kv_bf16 else (lambda a: a)
    xn = rmsnorm(x, w["n1"], w["eps"])
    q = linear(xn, w["q"], w.get("bq")).reshape(B, n_heads, d)
    k = linear(xn, w["k"], w.get("bk")).reshape(B, n_kv, d)
    v = linear(xn, w["v"], w.get("bv")).reshape(B, n_kv, d)
    att = np.empty((B, n_heads * d), np.float32)
    for b in range(B):
        L = lens[b]
        qr = rope_apply(q[b], cos_t[L], sin_t[L], variant)
        kr = rope_apply(k[b], cos_t[L], sin_t[L], variant)
        kc[b] = store(np.concatenate([kc[b][:L], kr[None]], 0))
        vc[b] = store(np.concatenate([vc[b][:L], v[b][None]], 0))
        K = kc[b].transpose(1, 0, 2).copy()
        V = vc[b].transpose(1, 0, 2).copy()
        att[b] = gqa_attention(qr[None], K, V, causal=False)[0].reshape(-1)
    h = linear(att, w["o"]) + x
    hn = rmsnorm(h, w["n2"], w["eps"])
    return linear(swiglu(linear(hn, w["gate"]), linear(hn, w["up"])), w["down"]) + h


def model_decode_step(tokens, embed, layers, final_norm, lm_head, eps, caches, lens, n_heads, n_kv, cos_t, sin_t,
                      variant, kv_bf16=False):
    """OomLlamaModel::forward_turbo (src/oomllama.rs:504-553) for one new token per sequence, then the greedy
    pick (:1000-1003).  embed, lm_head [vocab, H] dequantised; layers a list of decoder_layer_decode weight dicts;
    caches[l] = (kc, vc) lists per sequence, extended in place, and lens advanced by one.  Returns
    (next ids [B], logits [B, vocab])."""
    x = embed[np.asarray(tokens, np.int64)].astype(np.float32)
    for l, w in enumerate(layers):
        x = decoder_layer_decode(x, w, caches[l][0], caches[l][1], lens, n_heads, n_kv, cos_t, sin_t, variant,
                                 kv_bf16)
    for b in range(len(lens)):
        lens[b] += 1
    logits = linear(rmsnorm(x, final_norm, eps), lm_head)
    return argmax(logits), logits


def omp_max_threads() -> int:
    return int(lib().oracle_omp_max_threads())


def set_threads(n: int) -> int:
    """Use n host threads in the OpenMP loops; returns the new maximum."""
    L = lib()
    L.oracle_set_threads.argtypes = [ctypes.c_int]
    L.oracle_set_threads(int(n))
    return omp_max_threads()


def host_cores() -> int:
    """Cores this process may run on."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1

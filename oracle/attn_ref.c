/*
 * CPU oracle for OomLlama's grouped-query attention step.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker the parity tests and
 * the CPU baseline leg of the benchmark use.  The product library never links
 * or calls it.
 *
 * Parity status: UNPINNED.  The reference (Rust + candle 0.9.1) cannot be
 * built or run here (no Rust toolchain, candle is not vendored, and the crate
 * names a module file that does not exist, src/lib.rs:62).  The reference's own
 * tests hold no golden vectors for attention or RoPE
 * (src/oomllama_turbo.rs:815-831 only checks an empty cache and a pin
 * strategy; src/oom_inference.rs:430-436 only checks that softmax sums to 1).
 * This restatement is therefore pinned against known-answer identities and an
 * independent float64 implementation (tests/golden), not against reference
 * outputs.
 *
 * Arithmetic contract (what "the reference's algorithm" means here):
 *  - every scalar op is IEEE binary32 with round-to-nearest-even and NO
 *    fused multiply-add (build with -ffp-contract=off), matching the reference's
 *    separately rounded f32 tensor ops;
 *  - sums run in the reference's loop order (oom_inference.rs:251-270);
 *  - powf/cosf/sinf/expf are the host libm's, as Rust's f32 methods call the
 *    platform libm on Linux.
 *
 * The reference's intended semantics are used where its turbo path is buggy:
 * RoPE position of a new token = that layer's own cache length + s (the
 * reference reads layer 0's length, oomllama_turbo.rs:671 with :101-103), the
 * GQA expansion uses the KV length (oomllama_turbo.rs:324 uses q's length),
 * and the causal mask is aligned to the end of the KV sequence
 * (oomllama_turbo.rs:348-358 assumes q_len == kv_len).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <stdlib.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ROPE_SPLIT_HALF 0
#define ROPE_INTERLEAVED 1

/* bf16 <-> f32.  bf16 -> f32 is a 16-bit left shift
 * (src/safetensors2oom.rs:32-39).  f32 -> bf16 rounds to nearest even, the
 * storage rounding for a bf16 KV cache; NaN stays NaN. */
float oracle_bf16_to_f32(uint16_t h) {
    uint32_t u = ((uint32_t)h) << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

uint16_t oracle_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) return (uint16_t)((u >> 16) | 0x40);
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    return (uint16_t)(u >> 16);
}

void oracle_round_bf16(float* x, int64_t n) {
    for (int64_t i = 0; i < n; ++i) x[i] = oracle_bf16_to_f32(oracle_f32_to_bf16(x[i]));
}

/* RoPE table rows [n_pos][head_dim/2]:
 *   inv_freq_i = 1 / theta^(2i/d)      (f32 powf, oomllama_turbo.rs:756, :380)
 *   angle      = (f32)pos * inv_freq_i (oomllama_turbo.rs:754-757; the
 *                outer-product matmul at :389 is the same single product)
 *   cos/sin    = f32 cosf/sinf          (oomllama_turbo.rs:759-760, :392-393)
 */
void oracle_rope_table(float theta, int head_dim, int pos0, int n_pos, float* cos_t, float* sin_t) {
    int half = head_dim / 2;
    float* inv = (float*)malloc(sizeof(float) * (size_t)half);
    for (int i = 0; i < half; ++i) {
        float e = (2.0f * (float)i) / (float)head_dim;
        inv[i] = 1.0f / powf(theta, e);
    }
    for (int p = 0; p < n_pos; ++p) {
        float pos = (float)(pos0 + p);
        for (int i = 0; i < half; ++i) {
            float a = pos * inv[i];
            cos_t[(size_t)p * half + i] = cosf(a);
            sin_t[(size_t)p * half + i] = sinf(a);
        }
    }
    free(inv);
}

/* Rotate one token's heads in place.  x: [n_heads][head_dim]; cos/sin: the
 * table row of this token's position [head_dim/2].
 *  SPLIT_HALF: pairs (x[i], x[i+d/2])  -- apply_rope_llama
 *              (oomllama_turbo.rs:443-467), TurboEngine::apply_rope's
 *              x*cos + rotate_half(x)*sin (:773-783, identical rounding) and
 *              oom_inference.rs:212-233.
 *  INTERLEAVED: pairs (x[2i], x[2i+1]) -- apply_rope (oomllama_turbo.rs:402-438).
 * Both: x0' = x0*cos - x1*sin ; x1' = x0*sin + x1*cos, each product rounded. */
void oracle_rope_apply(float* x, int n_heads, int head_dim, const float* cos_r, const float* sin_r, int variant) {
    int half = head_dim / 2;
    for (int h = 0; h < n_heads; ++h) {
        float* xh = x + (size_t)h * head_dim;
        for (int i = 0; i < half; ++i) {
            int i0 = variant == ROPE_INTERLEAVED ? 2 * i : i;
            int i1 = variant == ROPE_INTERLEAVED ? 2 * i + 1 : i + half;
            float x0 = xh[i0], x1 = xh[i1];
            float c = cos_r[i], s = sin_r[i];
            float a = x0 * c, b = x1 * s;
            float e = x0 * s, f = x1 * c;
            xh[i0] = a - b;
            xh[i1] = e + f;
        }
    }
}

/* y = x @ W^T + b, one row of x (oom_inference.rs:168-180 loop order; the
 * bias is added after the product as in oomllama_turbo.rs:648-656).
 * W: [out][in] row-major (HF/GGUF layout, oomllama_turbo.rs:637).  b may be NULL. */
void oracle_matvec_bias(const float* x, const float* w, const float* b, int out_f, int in_f, float* y) {
    for (int i = 0; i < out_f; ++i) {
        const float* row = w + (size_t)i * in_f;
        float sum = 0.0f;
        for (int j = 0; j < in_f; ++j) sum += x[j] * row[j];
        y[i] = b ? sum + b[i] : sum;
    }
}

/* Scalar single-head attention over the first L rows of a [*, d] cache
 * (oom_inference.rs:240-272 with softmax :152-164).
 * Writes out[d]; returns the natural-log LSE of the scaled scores
 * (max + log(sum)), used by split-context merge checks. */
float oracle_attention_head(const float* q, const float* k, const float* v, int L, int d, float scale, float* scores_ws, float* out) {
    for (int t = 0; t < L; ++t) {
        const float* kt = k + (size_t)t * d;
        float dot = 0.0f;
        for (int i = 0; i < d; ++i) dot += q[i] * kt[i];
        scores_ws[t] = dot * scale;
    }
    float mx = -INFINITY;
    for (int t = 0; t < L; ++t) mx = fmaxf(mx, scores_ws[t]);
    float sum = 0.0f;
    for (int t = 0; t < L; ++t) {
        scores_ws[t] = expf(scores_ws[t] - mx);
        sum += scores_ws[t];
    }
    for (int t = 0; t < L; ++t) scores_ws[t] /= sum;
    for (int i = 0; i < d; ++i) out[i] = 0.0f;
    for (int t = 0; t < L; ++t) {
        const float* vt = v + (size_t)t * d;
        float p = scores_ws[t];
        for (int i = 0; i < d; ++i) out[i] += p * vt[i];
    }
    return L > 0 ? mx + logf(sum) : -INFINITY;
}

/* GQA attention for one sequence (flash_attention_forward semantics,
 * oomllama_turbo.rs:304-369, with the KV length used for the expansion):
 *   q:   [n_q][n_heads][d]   queries of the n_q newest tokens
 *   k,v: [n_kv][L][d]        the layer cache after the append (LayerKVCache
 *                            layout [n_kv, seq, d], oomllama_turbo.rs:27-30)
 *   out: [n_q][n_heads][d]   lse: [n_q][n_heads] (may be NULL)
 * q head h reads kv head h / (n_heads/n_kv) (repeat_interleave grouping,
 * oomllama_turbo.rs:313-316).  Query i sits at absolute position
 * L - n_q + i and, when causal, sees keys 0..L-n_q+i (the additive -1e9 mask
 * of :348-359 underflows exp to exactly 0 in f32, so skipping is identical).
 * Non-causal queries see all L keys. */
void oracle_gqa_attention(const float* q, const float* k, const float* v, int n_q, int L, int n_heads, int n_kv,
                          int d, float scale, int causal, float* out, float* lse) {
    int group = n_heads / n_kv;
    float* ws = (float*)malloc(sizeof(float) * (size_t)(L > 0 ? L : 1));
    for (int i = 0; i < n_q; ++i) {
        int visible = causal ? (L - n_q + i + 1) : L;
        for (int h = 0; h < n_heads; ++h) {
            int g = h / group;
            const float* qh = q + ((size_t)i * n_heads + h) * d;
            const float* kg = k + (size_t)g * L * d;
            const float* vg = v + (size_t)g * L * d;
            float r = oracle_attention_head(qh, kg, vg, visible, d, scale, ws, out + ((size_t)i * n_heads + h) * d);
            if (lse) lse[(size_t)i * n_heads + h] = r;
        }
    }
    free(ws);
}

/* Same as oracle_gqa_attention for a set of (query row, head) pairs only:
 * rows[j], heads[j] pick the pair; out: [n_pairs][d].  Used to check large
 * prefill shapes on a sample of rows. */
void oracle_gqa_attention_rows(const float* q, const float* k, const float* v, int n_q, int L, int n_heads, int n_kv,
                               int d, float scale, int causal, int n_pairs, const int* rows, const int* heads,
                               float* out) {
    int group = n_heads / n_kv;
#pragma omp parallel
    {
        float* ws = (float*)malloc(sizeof(float) * (size_t)(L > 0 ? L : 1));
#pragma omp for schedule(dynamic, 1)
        for (int j = 0; j < n_pairs; ++j) {
            int i = rows[j], h = heads[j], g = h / group;
            int visible = causal ? (L - n_q + i + 1) : L;
            oracle_attention_head(q + ((size_t)i * n_heads + h) * d, k + (size_t)g * L * d, v + (size_t)g * L * d,
                                  visible, d, scale, ws, out + (size_t)j * d);
        }
        free(ws);
    }
}

/* Batched single-token decode, the timed CPU baseline: for each sequence b
 * and q head h, oom_inference.rs:240-272 over that sequence's L_b cached
 * tokens.  k,v of sequence b at kv_off[b] elements: [n_kv][L_b][d].
 * q,out: [B][n_heads][d].  n_threads <= 1 runs the reference's single-thread
 * loop; otherwise OpenMP shares (b, h) pairs across host threads. */
void oracle_decode_batch(const float* q, const float* k, const float* v, const int64_t* kv_off, const int* L, int B,
                         int n_heads, int n_kv, int d, float scale, int n_threads, float* out) {
    int group = n_heads / n_kv;
    int maxL = 1;
    for (int b = 0; b < B; ++b) maxL = L[b] > maxL ? L[b] : maxL;
#ifdef _OPENMP
    int nt = n_threads > 1 ? n_threads : 1;
#pragma omp parallel num_threads(nt)
#endif
    {
        float* ws = (float*)malloc(sizeof(float) * (size_t)maxL);
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
        for (int bh = 0; bh < B * n_heads; ++bh) {
            int b = bh / n_heads, h = bh % n_heads, g = h / group;
            const float* kb = k + kv_off[b] + (size_t)g * L[b] * d;
            const float* vb = v + kv_off[b] + (size_t)g * L[b] * d;
            oracle_attention_head(q + (size_t)bh * d, kb, vb, L[b], d, scale, ws, out + (size_t)bh * d);
        }
        free(ws);
    }
}

/* Merge split-context partials (normalised O_j with natural-log LSE_j) into
 * one result: M = max lse_j; w_j = exp(lse_j - M); O = sum w_j O_j / sum w_j;
 * lse = M + log(sum w_j).  parts: [n_parts][n_rows][d], lses: [n_parts][n_rows].
 * A part with lse = -inf (no keys) contributes nothing. */
void oracle_merge_partials(const float* parts, const float* lses, int n_parts, int n_rows, int d, float* out,
                           float* lse_out) {
    for (int r = 0; r < n_rows; ++r) {
        float M = -INFINITY;
        for (int j = 0; j < n_parts; ++j) M = fmaxf(M, lses[(size_t)j * n_rows + r]);
        float wsum = 0.0f;
        for (int i = 0; i < d; ++i) out[(size_t)r * d + i] = 0.0f;
        if (M == -INFINITY) {
            if (lse_out) lse_out[r] = -INFINITY;
            continue;
        }
        for (int j = 0; j < n_parts; ++j) {
            float l = lses[(size_t)j * n_rows + r];
            if (l == -INFINITY) continue;
            float w = expf(l - M);
            wsum += w;
            const float* o = parts + ((size_t)j * n_rows + r) * d;
            for (int i = 0; i < d; ++i) out[(size_t)r * d + i] += w * o[i];
        }
        for (int i = 0; i < d; ++i) out[(size_t)r * d + i] /= wsum;
        if (lse_out) lse_out[r] = M + logf(wsum);
    }
}

/* Full layer attention step for one batch of B sequences sharing one cache
 * length P (TurboEngine::attention_forward_with_bias,
 * oomllama_turbo.rs:618-723, without the o_proj, which stays a plain GEMM):
 *   x:     [B][S][H]
 *   wq:    [n_heads*d][H], wk/wv: [n_kv*d][H]; bq/bk/bv may be NULL
 *   kc,vc: [B][n_kv][P+S][d] in/out; rows 0..P-1 hold the cache, rows
 *          P..P+S-1 receive this step's rotated K and V (LayerKVCache::append,
 *          :41-55), rounded to bf16 when kv_bf16
 *   cos_t/sin_t: table rows for positions 0..P+S-1
 *   out:   [B][S][n_heads*d] attention output before o_proj (:711-713)
 * Position of token s is P + s (the layer's own cache length). */
void oracle_layer_attention(const float* x, int B, int S, int H, const float* wq, const float* wk, const float* wv,
                            const float* bq, const float* bk, const float* bv, int n_heads, int n_kv, int d, int P,
                            float* kc, float* vc, int kv_bf16, const float* cos_t, const float* sin_t, int variant,
                            float scale, float* out) {
    int qo = n_heads * d, ko = n_kv * d, L = P + S, half = d / 2;
    float* q = (float*)malloc(sizeof(float) * (size_t)S * qo);
    float* kt = (float*)malloc(sizeof(float) * (size_t)ko);
    float* vt = (float*)malloc(sizeof(float) * (size_t)ko);
    for (int b = 0; b < B; ++b) {
        float* kb = kc + (size_t)b * n_kv * L * d;
        float* vb = vc + (size_t)b * n_kv * L * d;
        for (int s = 0; s < S; ++s) {
            const float* xr = x + ((size_t)b * S + s) * H;
            oracle_matvec_bias(xr, wq, bq, qo, H, q + (size_t)s * qo);
            oracle_matvec_bias(xr, wk, bk, ko, H, kt);
            oracle_matvec_bias(xr, wv, bv, ko, H, vt);
            const float* cr = cos_t + (size_t)(P + s) * half;
            const float* sr = sin_t + (size_t)(P + s) * half;
            oracle_rope_apply(q + (size_t)s * qo, n_heads, d, cr, sr, variant);
            oracle_rope_apply(kt, n_kv, d, cr, sr, variant);
            if (kv_bf16) {
                oracle_round_bf16(kt, ko);
                oracle_round_bf16(vt, ko);
            }
            for (int g = 0; g < n_kv; ++g) {
                memcpy(kb + ((size_t)g * L + P + s) * d, kt + (size_t)g * d, sizeof(float) * d);
                memcpy(vb + ((size_t)g * L + P + s) * d, vt + (size_t)g * d, sizeof(float) * d);
            }
        }
        oracle_gqa_attention(q, kb, vb, S, L, n_heads, n_kv, d, scale, 1, out + (size_t)b * S * qo, NULL);
    }
    free(q);
    free(kt);
    free(vt);
}

/* Host threads used by the OpenMP loops (launchers such as torchrun preset
 * OMP_NUM_THREADS=1 per process). */
/* ------------------------------------------------------------------ Q8 weights
 * The .oom Q8 format.  The writer (src/gguf2oom.rs:719-770, add_tensor_q8)
 * cuts a tensor's values into blocks of 256 (the last may be shorter); per
 * block it takes min and max (f32 compares from f32::MAX / f32::MIN), scale =
 * range / 255 (0 when |range| < 1e-9), q = round((v - min) / scale) with
 * Rust's round-half-away-from-zero and saturating `as u8` (NaN -> 0), and
 * writes [f32 scale][f32 min][u32 len][len bytes] little endian.  The reader
 * (OomLoader::dequantize_tensor_into, src/quant.rs:431-463, with
 * BlockQ8View::dequantize_fast, src/quant.rs:201-224) gives
 * min + (f32)q * scale, separately rounded. */
int64_t oracle_q8_stream_bytes(int64_t n) { return ((n + 255) / 256) * 12 + n; }

void oracle_q8_quantize(const float* v, int64_t n, uint8_t* out) {
    int64_t off = 0;
    for (int64_t start = 0; start < n; start += 256) {
        const int64_t end = start + 256 < n ? start + 256 : n;
        float mn = 3.40282347e38f, mx = -3.40282347e38f;
        for (int64_t i = start; i < end; ++i) {
            if (v[i] < mn) mn = v[i];
            if (v[i] > mx) mx = v[i];
        }
        const float range = mx - mn;
        const float scale = fabsf(range) < 1e-9f ? 0.0f : range / 255.0f;
        const uint32_t len = (uint32_t)(end - start);
        memcpy(out + off, &scale, 4);
        memcpy(out + off + 4, &mn, 4);
        memcpy(out + off + 8, &len, 4);
        off += 12;
        for (int64_t i = start; i < end; ++i) {
            uint8_t q = 0;
            if (scale != 0.0f) {
                const float r = roundf((v[i] - mn) / scale);
                q = isnan(r) ? 0 : r <= 0.0f ? 0 : r >= 255.0f ? 255 : (uint8_t)r;
            }
            out[off++] = q;
        }
    }
}

/* Returns 0, or -1 for a malformed stream (the reader would read past it). */
int oracle_q8_dequantize(const uint8_t* stream, int64_t stream_bytes, int64_t n, float* out) {
    int64_t off = 0, pos = 0;
    while (pos < n) {
        if (off + 12 > stream_bytes) return -1;
        float scale, mn;
        uint32_t len;
        memcpy(&scale, stream + off, 4);
        memcpy(&mn, stream + off + 4, 4);
        memcpy(&len, stream + off + 8, 4);
        off += 12;
        const int64_t num = n - pos < 256 ? n - pos : 256;
        if ((int64_t)len < num || off + (int64_t)len > stream_bytes) return -1;
        for (int64_t i = 0; i < num; ++i) out[pos + i] = mn + (float)stream[off + i] * scale;
        off += len;
        pos += num;
    }
    return 0;
}

/* y[t][r] = sum_c x[t][c] * W[r][c] (+ b[r]): oom_inference.rs:168-180 per token,
 * OpenMP over (token, row) pairs. */
void oracle_linear(const float* x, int T, const float* w, const float* b, int rows, int cols, float* y) {
#pragma omp parallel for collapse(2) schedule(static)
    for (int t = 0; t < T; ++t)
        for (int r = 0; r < rows; ++r) {
            float sum = 0.0f;
            const float* wr = w + (size_t)r * cols;
            const float* xt = x + (size_t)t * cols;
            for (int c = 0; c < cols; ++c) sum += xt[c] * wr[c];
            y[(size_t)t * rows + r] = b ? sum + b[r] : sum;
        }
}

/* ------------------------------------------------------------------ RMSNorm, SwiGLU
 * GhostRMSNorm::forward (src/oomllama.rs:200-211) as candle's ops: sqr,
 * mean over the last dim (sum / H, summed in index order here), + eps, sqrt,
 * x / that, * w; f32 throughout. */
void oracle_rmsnorm(const float* x, const float* w, float eps, int T, int H, float* out) {
    for (int t = 0; t < T; ++t) {
        const float* xr = x + (size_t)t * H;
        float s = 0.0f;
        for (int i = 0; i < H; ++i) s += xr[i] * xr[i];
        const float denom = sqrtf(s / (float)H + eps);
        for (int i = 0; i < H; ++i) out[(size_t)t * H + i] = xr[i] / denom * w[i];
    }
}

/* GhostMlp::forward's gated activation (src/oomllama.rs:235-238):
 * gate * sigmoid(gate) * up, sigmoid(x) = 1 / (1 + exp(-x)). */
void oracle_swiglu(const float* gate, const float* up, int64_t n, float* out) {
    for (int64_t i = 0; i < n; ++i) {
        const float s = 1.0f / (1.0f + expf(-gate[i]));
        out[i] = gate[i] * s * up[i];
    }
}

void oracle_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

int oracle_omp_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

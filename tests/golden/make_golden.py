"""Generates tests/golden/golden.npz: known-answer vectors for the attention
step, computed by an implementation independent of the C oracle (torch,
float64) from the reference's formulas:

  rope_*       RoPE tables and rotations (src/oomllama_turbo.rs:376-467, 753-783)
  head_*       scalar single-head attention (src/oom_inference.rs:240-272)
  gqa_*        causal GQA attention, 7:1 grouping (src/oomllama_turbo.rs:304-369)
  layer_*      QKV + bias + RoPE + append + attention (src/oomllama_turbo.rs:618-713)
  merge_*      log-sum-exp merge of split-context partials

The reference itself cannot run here (Rust toolchain absent), so these vectors
pin the oracle to the reference's mathematics, not to reference outputs.
Run from the repository root:  python tests/golden/make_golden.py
"""
import os

import numpy as np
import torch

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.npz")
D = 128


def rope_tables(theta, positions):
    i = torch.arange(D // 2, dtype=torch.float64)
    inv = 1.0 / theta ** (2.0 * i / D)
    ang = torch.tensor(positions, dtype=torch.float64)[:, None] * inv[None, :]
    return torch.cos(ang), torch.sin(ang)


def rope(x, c, s, interleaved):
    # x [T, H, D]; c, s [T, D/2]
    x = x.clone()
    if interleaved:
        x0, x1 = x[..., 0::2].clone(), x[..., 1::2].clone()
    else:
        x0, x1 = x[..., : D // 2].clone(), x[..., D // 2:].clone()
    c, s = c[:, None, :], s[:, None, :]
    y0, y1 = x0 * c - x1 * s, x0 * s + x1 * c
    if interleaved:
        x[..., 0::2], x[..., 1::2] = y0, y1
    else:
        x[..., : D // 2], x[..., D // 2:] = y0, y1
    return x


def attention(q, k, v, causal):
    # q [n_q, Hq, D]; k, v [Hkv, L, D]
    n_q, hq, _ = q.shape
    hkv, L, _ = k.shape
    grp = hq // hkv
    kk = k.repeat_interleave(grp, dim=0)
    vv = v.repeat_interleave(grp, dim=0)
    sc = torch.einsum("qhd,hld->hql", q, kk) / np.sqrt(D)
    if causal:
        qi = torch.arange(n_q)[:, None] + (L - n_q)
        kj = torch.arange(L)[None, :]
        sc = sc.masked_fill(kj > qi, float("-inf"))
    lse = torch.logsumexp(sc, dim=-1)
    p = torch.softmax(sc, dim=-1)
    return torch.einsum("hql,hld->qhd", p, vv), lse.transpose(0, 1)


def main():
    g = torch.Generator().manual_seed(1234)
    r = {}
    # RoPE, both variants, both thetas, positions where f32 angles are still accurate
    pos = [0, 1, 2, 7, 100, 511, 1000, 4095]
    x = torch.randn(len(pos), 3, D, generator=g, dtype=torch.float64)
    r["rope_x"] = x.float().numpy()
    r["rope_pos"] = np.array(pos, np.int32)
    for theta, tag in ((1e6, "qwen"), (5e5, "llama")):
        c, s = rope_tables(theta, pos)
        r[f"rope_cos_{tag}"] = c.numpy()
        r[f"rope_sin_{tag}"] = s.numpy()
        xf = x.float().double()
        r[f"rope_inter_{tag}"] = rope(xf, c, s, True).numpy()
        r[f"rope_split_{tag}"] = rope(xf, c, s, False).numpy()
    # single head (oom_inference::attention_head)
    L = 37
    q = torch.randn(D, generator=g, dtype=torch.float64)
    k = torch.randn(L, D, generator=g, dtype=torch.float64)
    v = torch.randn(L, D, generator=g, dtype=torch.float64)
    qf, kf, vf = q.float().double(), k.float().double(), v.float().double()
    sc = kf @ qf / np.sqrt(D)
    r["head_q"], r["head_k"], r["head_v"] = q.float().numpy(), k.float().numpy(), v.float().numpy()
    r["head_out"] = (torch.softmax(sc, 0) @ vf).numpy()
    r["head_lse"] = np.array(torch.logsumexp(sc, 0).item())
    # causal GQA 14q / 2kv over a cache of 50 with 9 new queries
    n_q, L, hq, hkv = 9, 50, 14, 2
    q = torch.randn(n_q, hq, D, generator=g, dtype=torch.float64).float().double()
    k = torch.randn(hkv, L, D, generator=g, dtype=torch.float64).float().double()
    v = torch.randn(hkv, L, D, generator=g, dtype=torch.float64).float().double()
    out, lse = attention(q, k, v, True)
    r["gqa_q"], r["gqa_k"], r["gqa_v"] = q.float().numpy(), k.float().numpy(), v.float().numpy()
    r["gqa_out"], r["gqa_lse"] = out.numpy(), lse.numpy()
    # layer step: hidden 64, 4q/2kv heads, cache of 21, 3 new tokens, batch 2, interleaved theta 1e6
    B, S, H, P, hq, hkv = 2, 3, 64, 21, 4, 2
    x = torch.randn(B, S, H, generator=g, dtype=torch.float64).float().double()
    wq = (0.02 * torch.randn(hq * D, H, generator=g, dtype=torch.float64)).float().double()
    wk = (0.02 * torch.randn(hkv * D, H, generator=g, dtype=torch.float64)).float().double()
    wv = (0.02 * torch.randn(hkv * D, H, generator=g, dtype=torch.float64)).float().double()
    bq = (0.1 * torch.randn(hq * D, generator=g, dtype=torch.float64)).float().double()
    bk = (0.1 * torch.randn(hkv * D, generator=g, dtype=torch.float64)).float().double()
    bv = (0.1 * torch.randn(hkv * D, generator=g, dtype=torch.float64)).float().double()
    kc = torch.randn(B, hkv, P, D, generator=g, dtype=torch.float64).float().double()
    vc = torch.randn(B, hkv, P, D, generator=g, dtype=torch.float64).float().double()
    c, s = rope_tables(1e6, list(range(P, P + S)))
    outs = []
    for b in range(B):
        qp = (x[b] @ wq.T + bq).view(S, hq, D)
        kp = (x[b] @ wk.T + bk).view(S, hkv, D)
        vp = (x[b] @ wv.T + bv).view(S, hkv, D)
        qp, kp = rope(qp, c, s, True), rope(kp, c, s, True)
        kf = torch.cat([kc[b], kp.transpose(0, 1)], dim=1)
        vf = torch.cat([vc[b], vp.transpose(0, 1)], dim=1)
        o, _ = attention(qp, kf, vf, True)
        outs.append(o.reshape(S, hq * D))
    for name, t in (("x", x), ("wq", wq), ("wk", wk), ("wv", wv), ("bq", bq), ("bk", bk), ("bv", bv), ("kc", kc),
                    ("vc", vc)):
        r[f"layer_{name}"] = t.float().numpy()
    r["layer_out"] = torch.stack(outs).numpy()
    # merge of 3 partials over 5 rows; one partial empty on row 2
    parts = torch.randn(3, 5, D, generator=g, dtype=torch.float64).float().double()
    lses = (3 * torch.randn(3, 5, generator=g, dtype=torch.float64)).float().double()
    lses[1, 2] = float("-inf")
    w = torch.softmax(lses, dim=0)
    r["merge_parts"], r["merge_lses"] = parts.float().numpy(), lses.float().numpy()
    r["merge_out"] = torch.einsum("pr,prd->rd", w, parts).numpy()
    r["merge_lse"] = torch.logsumexp(lses, dim=0).numpy()
    np.savez_compressed(OUT, **r)
    print(OUT, os.path.getsize(OUT), "bytes")


if __name__ == "__main__":
    main()

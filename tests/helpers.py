"""Shared helpers for the GPU parity tests: build an engine with shuffled
pages, fill caches, and compare against the oracle."""
import numpy as np
import torch

from oomllama_b200 import TurboConfig, TurboEngine

BF16_ATOL = 2e-3   # bf16 KV tolerance: max-abs <= 2e-3 and norm-relative <= 1e-2
BF16_RTOL = 1e-2
F32_ATOL = 1e-4    # f32 path tolerance


def rel_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def assert_close(out, ref, atol, rtol=None, what=""):
    out = np.asarray(out, np.float64)
    ref = np.asarray(ref, np.float64)
    assert np.isfinite(out).all(), f"{what}: non-finite output"
    mx = float(np.abs(out - ref).max()) if out.size else 0.0
    assert mx <= atol, f"{what}: max-abs {mx:.3e} > {atol:.1e}"
    if rtol is not None:
        r = rel_err(out, ref)
        assert r <= rtol, f"{what}: norm-relative {r:.3e} > {rtol:.1e}"


def make_engine(n_heads, n_kv, lens_cap, kv_dtype="bf16", variant="interleaved", theta=1e6, hidden=0,
                shuffle_seed=0, n_layers=1, max_seq_len=None):
    """Engine whose sequences own shuffled pool pages, enough for lens_cap[s] tokens each."""
    B = len(lens_cap)
    msl = max_seq_len or max(16, max(lens_cap))
    pages = [-(-L // 16) for L in lens_cap]
    cfg = TurboConfig(n_layers=n_layers, hidden_size=hidden, n_heads=n_heads, n_kv_heads=n_kv, max_seq_len=msl,
                      max_seqs=B, n_pages=max(1, sum(pages)), kv_dtype=kv_dtype, rope_variant=variant,
                      rope_theta=theta)
    eng = TurboEngine(cfg, device=0, assign_pages=False)
    perm = np.random.default_rng(shuffle_seed).permutation(max(1, sum(pages)))
    o = 0
    for s in range(B):
        eng.set_block_table(s, perm[o:o + pages[s]].tolist())
        o += pages[s]
    return eng


def randn(shape, seed, dtype=torch.float32, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (scale * torch.randn(*shape, generator=g)).to(dtype)


def as_f32_np(t):
    return t.float().cpu().numpy()

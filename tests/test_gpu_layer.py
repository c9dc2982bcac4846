"""The whole layer step through the C ABI: TurboEngine.attention_forward_with_bias
(oomllama_turbo.rs:618-723) vs the oracle's restatement plus an f64 o_proj.
Covers decode (S=1), a short chunk (S=5, decode rows with causal lengths),
RoPE positions from each layer's own length, and the reset lifecycle."""
import numpy as np
import pytest
import torch

from helpers import F32_ATOL, BF16_ATOL, BF16_RTOL, assert_close, randn

pytestmark = pytest.mark.gpu


def _oracle_layer(oracle, x, wq, wk, wv, wo, bq, bk, bv, kc, vc, n_heads, n_kv, theta, kv_bf16):
    B, S, H = x.shape
    P = kc.shape[2]
    c, s = oracle.rope_table(theta, 128, P + S)
    att, kn, vn = oracle.layer_attention(x, wq, wk, wv, bq, bk, bv, n_heads, n_kv, kc, vc, c, s,
                                         oracle.ROPE_INTERLEAVED, kv_bf16=kv_bf16)
    out = (att.astype(np.float64) @ wo.astype(np.float64).T).astype(np.float32)
    return out, kn, vn


@pytest.mark.parametrize("S,kv", [(1, "f32"), (5, "f32"), (1, "bf16"), (5, "bf16")])
def test_attention_forward_with_bias(oracle, S, kv):
    from oomllama_b200 import TurboConfig, TurboEngine
    B, H, n_heads, n_kv, P = 2, 512, 8, 2, 40
    cfg = TurboConfig(n_layers=2, hidden_size=H, n_heads=n_heads, n_kv_heads=n_kv, max_seq_len=256, max_seqs=B,
                      kv_dtype=kv, rope_variant="interleaved", rope_theta=1e6)
    eng = TurboEngine(cfg)
    dt = torch.bfloat16 if kv == "bf16" else torch.float32
    kc = randn((B, n_kv, P, 128), 1, dt)
    vc = randn((B, n_kv, P, 128), 2, dt)
    for b in range(B):
        # layer 1 holds the prefix; layer 0 stays empty so positions must come from layer 1's own length
        eng.kv_write(1, b, kc[b].transpose(0, 1).contiguous().cuda(), vc[b].transpose(0, 1).contiguous().cuda())
    x = randn((B, S, H), 3)
    wq, wk, wv = randn((n_heads * 128, H), 4, scale=0.02), randn((n_kv * 128, H), 5, scale=0.02), \
        randn((n_kv * 128, H), 6, scale=0.02)
    wo = randn((H, n_heads * 128), 7, scale=0.02)
    bq, bk, bv = randn((n_heads * 128,), 8, scale=0.1), randn((n_kv * 128,), 9, scale=0.1), \
        randn((n_kv * 128,), 10, scale=0.1)
    out = eng.attention_forward_with_bias(1, x.cuda(), wq.cuda(), wk.cuda(), wv.cuda(), wo.cuda(), bq.cuda(),
                                          bk.cuda(), bv.cuda())
    eng.sync()
    ref, kn, vn = _oracle_layer(oracle, x.numpy(), wq.numpy(), wk.numpy(), wv.numpy(), wo.numpy(), bq.numpy(),
                                bk.numpy(), bv.numpy(), kc.float().numpy(), vc.float().numpy(), n_heads, n_kv, 1e6,
                                kv == "bf16")
    tol = (F32_ATOL, None) if kv == "f32" else (BF16_ATOL, BF16_RTOL)
    assert_close(out.cpu().numpy(), ref, tol[0], tol[1], what=f"layer S={S} {kv}")
    assert eng.seq_len(1, 0) == P + S and eng.seq_len(0, 0) == 0
    kr, vr = eng.kv_read(1, 1)
    np.testing.assert_allclose(kr.float().numpy(), kn[1], atol=5e-5 if kv == "f32" else 2e-2)
    eng.reset()
    assert eng.seq_len(1, 0) == 0
    eng.close()


def test_prefill_path_of_layer_step(oracle):
    # S > 16 on a bf16 cache runs the tcgen05 prefill inside the layer step
    from oomllama_b200 import TurboConfig, TurboEngine
    B, S, H, n_heads, n_kv = 1, 200, 256, 14, 2
    cfg = TurboConfig(n_layers=1, hidden_size=H, n_heads=n_heads, n_kv_heads=n_kv, max_seq_len=256, max_seqs=B,
                      kv_dtype="bf16", rope_variant="interleaved", rope_theta=1e6)
    eng = TurboEngine(cfg)
    x = randn((B, S, H), 11)
    wq, wk, wv = randn((n_heads * 128, H), 12, scale=0.05), randn((n_kv * 128, H), 13, scale=0.05), \
        randn((n_kv * 128, H), 14, scale=0.05)
    wo = randn((H, n_heads * 128), 15, scale=0.02)
    out = eng.attention_forward_with_bias(0, x.cuda(), wq.cuda(), wk.cuda(), wv.cuda(), wo.cuda())
    eng.sync()
    # reference with the prefill's storage contract: q rounded to bf16 after RoPE, K/V bf16
    c, s = oracle.rope_table(1e6, 128, S)
    xq = np.stack([oracle.matvec_bias(x[0, t].numpy(), wq.numpy()) for t in range(S)]).reshape(S, n_heads, 128)
    xk = np.stack([oracle.matvec_bias(x[0, t].numpy(), wk.numpy()) for t in range(S)]).reshape(S, n_kv, 128)
    xv = np.stack([oracle.matvec_bias(x[0, t].numpy(), wv.numpy()) for t in range(S)]).reshape(S, n_kv, 128)
    q = oracle.round_bf16(oracle.rope_tokens(xq, np.arange(S), c, s, oracle.ROPE_INTERLEAVED))
    k = oracle.round_bf16(oracle.rope_tokens(xk, np.arange(S), c, s, oracle.ROPE_INTERLEAVED))
    v = oracle.round_bf16(xv)
    att = oracle.gqa_attention(q, k.transpose(1, 0, 2).copy(), v.transpose(1, 0, 2).copy(), causal=True)
    ref = (att.reshape(S, -1).astype(np.float64) @ wo.numpy().astype(np.float64).T).astype(np.float32)
    assert_close(out[0].cpu().numpy(), ref, BF16_ATOL, BF16_RTOL, what="layer prefill path")
    eng.close()

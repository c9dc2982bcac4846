"""K-A parity: bias + RoPE + paged append (bit-exact vs the oracle's f32
arithmetic, oomllama_turbo.rs:402-467 / :737-786) and the fused QKV GEMV
(f32 tolerance; the GEMV sums in a different order than the scalar loop of
oom_inference.rs:168-180)."""
import numpy as np
import pytest
import torch

from helpers import as_f32_np, make_engine, randn

pytestmark = pytest.mark.gpu


def _rotate_ref(oracle, x, positions, theta, variant):
    c, s = oracle.rope_table(theta, 128, int(max(positions)) + 1)
    return oracle.rope_tokens(x, positions, c, s, variant)


@pytest.mark.parametrize("variant,theta", [("interleaved", 1e6), ("split_half", 5e5)])
@pytest.mark.parametrize("in_dtype", [torch.float32, torch.bfloat16])
def test_rope_append_bit_exact(oracle, variant, theta, in_dtype):
    n_heads, n_kv = 28, 4
    prefix = [0, 100, 32760]
    n_new = 5
    lens = [p + n_new for p in prefix]
    kvdt = "bf16" if in_dtype == torch.bfloat16 else "f32"
    eng = make_engine(n_heads, n_kv, lens, kv_dtype=kvdt, variant=variant, theta=theta, max_seq_len=32768)
    for s, p in enumerate(prefix):
        eng.set_seq_len(0, s, p)
    T = len(prefix) * n_new
    q = randn((T, n_heads * 128), 1, in_dtype)
    k = randn((T, n_kv * 128), 2, in_dtype)
    v = randn((T, n_kv * 128), 3, in_dtype)
    bq = randn((n_heads * 128,), 4, scale=0.1)
    bk = randn((n_kv * 128,), 5, scale=0.1)
    bv = randn((n_kv * 128,), 6, scale=0.1)
    q_out = eng.rope_append(0, [0, 1, 2], q.cuda(), k.cuda(), v.cuda(), bq.cuda(), bk.cuda(), bv.cuda())
    eng.sync()
    vi = oracle.ROPE_INTERLEAVED if variant == "interleaved" else oracle.ROPE_SPLIT_HALF
    pos = np.concatenate([np.arange(p, p + n_new) for p in prefix])
    qb = (as_f32_np(q) + bq.numpy()[None]).astype(np.float32).reshape(T, n_heads, 128)
    kb = (as_f32_np(k) + bk.numpy()[None]).astype(np.float32).reshape(T, n_kv, 128)
    vb = (as_f32_np(v) + bv.numpy()[None]).astype(np.float32).reshape(T, n_kv, 128)
    q_ref = _rotate_ref(oracle, qb, pos, theta, vi)
    k_ref = _rotate_ref(oracle, kb, pos, theta, vi)
    np.testing.assert_array_equal(q_out.cpu().numpy(), q_ref)
    for s, p in enumerate(prefix):
        assert eng.seq_len(0, s) == p + n_new
        kc, vc = eng.kv_read(0, s)
        kr, vr = k_ref[s * n_new:(s + 1) * n_new], vb[s * n_new:(s + 1) * n_new]
        if kvdt == "bf16":
            kr, vr = oracle.round_bf16(kr), oracle.round_bf16(vr)
        np.testing.assert_array_equal(as_f32_np(kc[:, p:]).transpose(1, 0, 2), kr)
        np.testing.assert_array_equal(as_f32_np(vc[:, p:]).transpose(1, 0, 2), vr)
    eng.close()


def test_rope_append_bf16_q_out(oracle):
    eng = make_engine(28, 4, [64], kv_dtype="bf16")
    q = randn((64, 28 * 128), 7, torch.bfloat16)
    k = randn((64, 4 * 128), 8, torch.bfloat16)
    v = randn((64, 4 * 128), 9, torch.bfloat16)
    q_out = eng.rope_append(0, [0], q.cuda(), k.cuda(), v.cuda(), q_out_dtype=torch.bfloat16)
    eng.sync()
    q_ref = _rotate_ref(oracle, as_f32_np(q).reshape(64, 28, 128), np.arange(64), 1e6, oracle.ROPE_INTERLEAVED)
    np.testing.assert_array_equal(as_f32_np(q_out), oracle.round_bf16(q_ref))
    eng.close()


@pytest.mark.parametrize("T", [1, 3, 8])
@pytest.mark.parametrize("variant", ["interleaved", "split_half"])
def test_qkv_gemv_rope_append(oracle, T, variant):
    H, n_heads, n_kv = 3584, 28, 4
    eng = make_engine(n_heads, n_kv, [600] * T, kv_dtype="f32", variant=variant, hidden=H)
    for s in range(T):
        eng.set_seq_len(0, s, 512 + s)
    x = randn((T, H), 20)
    wq = randn((n_heads * 128, H), 21, scale=0.02)
    wk = randn((n_kv * 128, H), 22, scale=0.02)
    wv = randn((n_kv * 128, H), 23, scale=0.02)
    bq = randn((n_heads * 128,), 24, scale=0.1)
    bk = randn((n_kv * 128,), 25, scale=0.1)
    bv = randn((n_kv * 128,), 26, scale=0.1)
    q_out = eng.qkv_rope_append(0, list(range(T)), x.cuda(), wq.cuda(), wk.cuda(), wv.cuda(), bq.cuda(), bk.cuda(),
                                bv.cuda())
    eng.sync()
    vi = oracle.ROPE_INTERLEAVED if variant == "interleaved" else oracle.ROPE_SPLIT_HALF
    c, s_ = oracle.rope_table(1e6, 128, 600)
    for t in range(T):
        xq = oracle.matvec_bias(x[t].numpy(), wq.numpy(), bq.numpy()).reshape(n_heads, 128)
        xk = oracle.matvec_bias(x[t].numpy(), wk.numpy(), bk.numpy()).reshape(n_kv, 128)
        xv = oracle.matvec_bias(x[t].numpy(), wv.numpy(), bv.numpy()).reshape(n_kv, 128)
        pos = 512 + t
        qr = oracle.rope_apply(xq, c[pos], s_[pos], vi)
        kr = oracle.rope_apply(xk, c[pos], s_[pos], vi)
        np.testing.assert_allclose(q_out[t].cpu().numpy(), qr, atol=2e-5, rtol=1e-5)
        kc, vc = eng.kv_read(0, t)
        np.testing.assert_allclose(kc[:, pos].numpy(), kr, atol=2e-5, rtol=1e-5)
        np.testing.assert_allclose(vc[:, pos].numpy(), xv, atol=2e-5, rtol=1e-5)
    eng.close()


@pytest.mark.parametrize("T", [12, 40])
def test_qkv_bf16_weights(oracle, T):
    # 12 tokens: fused GEMV with bf16 weights (f32 x); 40 tokens: the tensor-core linear (x split into
    # bf16 hi + lo, so x keeps about 16 significant bits) + the K-A epilogue kernel
    H, n_heads, n_kv = 512, 8, 2
    eng = make_engine(n_heads, n_kv, [64], kv_dtype="bf16", hidden=H)
    x = randn((T, H), 30)
    wq = randn((n_heads * 128, H), 31, torch.bfloat16, scale=0.05)
    wk = randn((n_kv * 128, H), 32, torch.bfloat16, scale=0.05)
    wv = randn((n_kv * 128, H), 33, torch.bfloat16, scale=0.05)
    q_out = eng.qkv_rope_append(0, [0], x.cuda(), wq.cuda(), wk.cuda(), wv.cuda())
    eng.sync()
    c, s_ = oracle.rope_table(1e6, 128, 64)
    xq = (x.double() @ wq.double().T).float().numpy().reshape(T, n_heads, 128)
    qr = oracle.rope_tokens(xq, np.arange(T), c, s_, oracle.ROPE_INTERLEAVED)
    np.testing.assert_allclose(q_out.cpu().numpy(), qr, atol=1e-4, rtol=1e-4)
    eng.close()


def test_append_beyond_assigned_pages_rejected():
    from oomllama_b200._lib import OomAttnError
    eng = make_engine(28, 4, [16], kv_dtype="bf16")
    k = torch.zeros(17, 4 * 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(OomAttnError) as e:
        eng.kv_write(0, 0, k, k)
    assert e.value.code == 3
    assert eng.seq_len(0, 0) == 0
    eng.close()

"""The library's own linear kernels against float64 references, through the C ABI:
  * oomattn_linear (candle's x @ W^T, src/oomllama_turbo.rs:643-645, :715-720): the f32 GEMV for up to
    16 tokens and, above that, the tcgen05 tensor-core linear with bf16 hi/lo splits of x and W
    (f32 path tolerance: max-abs <= 1e-4 at unit-scale activations and N(0, 0.02) weights);
  * oomattn_q8_linear above 64 tokens: the tensor-core form with fp16 q values and the per-block
    promotion (BlockQ8View::dequantize_fast, src/quant.rs:201-224) against the oracle's
    dequantise-then-matvec, and against the 16-token-pass form on the same rows;
  * oomattn_q8_mlp above 64 tokens (gated activation formed in the split, residual added by TMA)."""
import numpy as np
import pytest
import torch

from helpers import F32_ATOL, assert_close, make_engine

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def eng():
    e = make_engine(8, 1, [16])
    yield e
    e.close()


def _f64_linear(x, w, b=None):
    y = x.astype(np.float64) @ w.astype(np.float64).T
    return y if b is None else y + b


@pytest.mark.parametrize("T,rows,cols", [(1, 512, 3584), (7, 3584, 512), (16, 260, 136), (17, 512, 3584),
                                         (300, 520, 136), (129, 3584, 3584), (1000, 1024, 3584)])
def test_linear_f32(eng, T, rows, cols):
    rng = np.random.default_rng(T + rows)
    x = rng.standard_normal((T, cols)).astype(np.float32)
    w = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    b = (rng.standard_normal(rows) * 0.1).astype(np.float32)
    y = eng.linear(torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda(), torch.from_numpy(b).cuda())
    eng.sync()
    assert_close(y.cpu().numpy(), _f64_linear(x, w, b), F32_ATOL, what=f"linear f32 T={T} {rows}x{cols}")


def test_linear_bf16_weights(eng):
    rng = np.random.default_rng(3)
    T, rows, cols = 200, 768, 1024
    x = rng.standard_normal((T, cols)).astype(np.float32)
    w = torch.from_numpy((rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)).to(torch.bfloat16)
    y = eng.linear(torch.from_numpy(x).cuda(), w.cuda())
    eng.sync()
    assert_close(y.cpu().numpy(), _f64_linear(x, w.float().numpy()), F32_ATOL, what="linear bf16 W")


def test_linear_rejects_bad_shapes(eng):
    from oomllama_b200._lib import OomAttnError
    x = torch.zeros(40, 130, device="cuda")
    with pytest.raises(OomAttnError):
        eng.linear(x, torch.zeros(64, 130, device="cuda"))  # cols % 8 != 0 on the tensor-core path


def _q8(oracle, rows, cols, seed, scale=0.02):
    from oomllama_b200 import Q8Matrix
    w = (np.random.default_rng(seed).standard_normal((rows, cols)) * scale).astype(np.float32)
    stream = oracle.q8_quantize(w)
    return Q8Matrix.from_oom_stream(stream, rows, cols, device=0), \
        oracle.q8_dequantize(stream, rows * cols).reshape(rows, cols)


@pytest.mark.parametrize("T,rows,cols", [(65, 512, 3584), (300, 1040, 512), (2048, 3584, 3584)])
def test_q8_linear_tensor_core_form(oracle, eng, T, rows, cols):
    wq, wd = _q8(oracle, rows, cols, seed=T)
    rng = np.random.default_rng(T + 1)
    x = rng.standard_normal((T, cols)).astype(np.float32)
    b = (rng.standard_normal(rows) * 0.1).astype(np.float32)
    xd, bd = torch.from_numpy(x).cuda(), torch.from_numpy(b).cuda()
    y = eng.q8_linear(wq, xd, bd)
    y16 = eng.q8_linear(wq, xd[:16].contiguous(), bd)  # the same rows through the 16-token passes
    eng.sync()
    y = y.cpu().numpy()
    assert_close(y, _f64_linear(x, wd, b), F32_ATOL, what=f"q8 tensor-core linear T={T} {rows}x{cols}")
    assert_close(y[:16], y16.cpu().numpy(), 2e-5, what="q8 tensor-core form vs 16-token passes")


def test_q8_mlp_tensor_core_form(oracle, eng):
    T, H, inter = 100, 512, 1024
    gq, gd = _q8(oracle, inter, H, 11)
    uq, ud = _q8(oracle, inter, H, 12)
    dq, dd = _q8(oracle, H, inter, 13)
    rng = np.random.default_rng(14)
    x = rng.standard_normal((T, H)).astype(np.float32)
    res = rng.standard_normal((T, H)).astype(np.float32)
    y = eng.q8_mlp(gq, uq, dq, torch.from_numpy(x).cuda(), residual=torch.from_numpy(res).cuda())
    eng.sync()
    ref = oracle.linear(oracle.swiglu(oracle.linear(x, gd), oracle.linear(x, ud)), dd) + res
    assert_close(y.cpu().numpy(), ref, F32_ATOL, what="q8 mlp T=100")


@pytest.mark.parametrize("T,rows,cols", [(16, 8192, 4096), (9, 8192, 4096), (12, 512, 65536)])
def test_q8_linear_tensor_core_decode_form(oracle, eng, T, rows, cols):
    # 9-16 tokens on a matrix of at least 32 M weights: the integer tensor-core pass (weight bytes as
    # stored x base-128 digits of x, tcgen05 kind::i8); the persistent grid's equal unit ranges cut
    # row tiles between CTAs (512 x 65536: each of the 4 row tiles among ~37 CTAs), whose partial
    # sums the last CTA to arrive adds in order; the bias in the epilogue; repeatable bit for bit
    wq, wd = _q8(oracle, rows, cols, seed=T + rows)
    rng = np.random.default_rng(T + 7)
    x = rng.standard_normal((T, cols)).astype(np.float32)
    b = (rng.standard_normal(rows) * 0.1).astype(np.float32)
    y1 = eng.q8_linear(wq, torch.from_numpy(x).cuda(), torch.from_numpy(b).cuda())
    y2 = eng.q8_linear(wq, torch.from_numpy(x).cuda(), torch.from_numpy(b).cuda())
    eng.sync()
    ref = _f64_linear(x, wd, b)
    assert_close(y1.cpu().numpy(), ref, F32_ATOL * max(1.0, float(np.abs(ref).max()) / 4),
                 what=f"q8 tensor-core pass T={T} {rows}x{cols}")
    assert torch.equal(y1, y2), "the split merge is not repeatable"


def _gpu_q8(rows, cols, g):
    from oomllama_b200 import Q8Matrix
    nb = rows * cols // 256
    return Q8Matrix(torch.randint(0, 256, (rows * cols,), dtype=torch.uint8, device="cuda", generator=g),
                    torch.rand(nb, device="cuda", generator=g) * 2e-4, -torch.rand(nb, device="cuda", generator=g) * 0.02,
                    rows, cols)


def _f64_q8(w):
    q = w.q.view(w.rows, w.cols).double()
    s = w.scale.double().repeat_interleave(256).view(w.rows, w.cols)
    m = w.min.double().repeat_interleave(256).view(w.rows, w.cols)
    return m + q * s


def test_q8_mlp_integer_form_with_gated_input(eng):
    # 16 tokens through gate/up (9472 x 3584 each, one launch) and down (3584 x 9472) on the integer
    # tensor-core form, the gated activation formed in down's digit split and the residual added in
    # its epilogue; against float64 on the device, and against the 16-token-pass form on 8 tokens
    g = torch.Generator(device="cuda").manual_seed(5)
    H, inter, T = 3584, 9472, 16
    gate, up, down = _gpu_q8(inter, H, g), _gpu_q8(inter, H, g), _gpu_q8(H, inter, g)
    x = torch.randn(T, H, device="cuda", generator=g)
    res = torch.randn(T, H, device="cuda", generator=g)
    y16 = eng.q8_mlp(gate, up, down, x, residual=res)
    y8 = torch.cat([eng.q8_mlp(gate, up, down, x[:8].contiguous(), residual=res[:8].contiguous()),
                    eng.q8_mlp(gate, up, down, x[8:].contiguous(), residual=res[8:].contiguous())])
    eng.sync()
    xd = x.double()
    hg, hu = xd @ _f64_q8(gate).T, xd @ _f64_q8(up).T
    ref = (hg * torch.sigmoid(hg) * hu) @ _f64_q8(down).T + res.double()
    tol = F32_ATOL * max(1.0, float(ref.abs().max()))
    assert_close(y16.cpu().numpy(), ref.cpu().numpy(), tol, what="q8 mlp, integer form")
    assert_close(y16.cpu().numpy(), y8.cpu().numpy(), tol, what="integer form vs 16-token passes")


def test_decoder_layer_integer_form_with_normalised_input(oracle):
    # one decoder layer's step for 16 sequences whose gate/up (2 x 8192 x 2048) run on the integer
    # tensor-core form with the RMSNorm folded into their digit split, against the same layer run as
    # two 8-sequence steps (the register form) on an identical second context
    from oomllama_b200 import Q8DecoderLayer, TurboConfig, TurboEngine
    H, hq, hkv, inter, B, ctx = 2048, 16, 2, 8192, 16, 300
    g = torch.Generator(device="cuda").manual_seed(9)
    w = Q8DecoderLayer(q=_gpu_q8(hq * 128, H, g), k=_gpu_q8(hkv * 128, H, g), v=_gpu_q8(hkv * 128, H, g),
                       o=_gpu_q8(H, hq * 128, g), gate=_gpu_q8(inter, H, g), up=_gpu_q8(inter, H, g),
                       down=_gpu_q8(H, inter, g), input_norm=1 + 0.1 * torch.randn(H, device="cuda", generator=g),
                       post_norm=1 + 0.1 * torch.randn(H, device="cuda", generator=g), eps=1e-6)
    x = torch.randn(B, H, device="cuda", generator=g)
    kv_k = torch.randn(B, ctx, hkv, 128, device="cuda", generator=g)
    kv_v = torch.randn(B, ctx, hkv, 128, device="cuda", generator=g)
    outs = []
    for split in (False, True):
        eng = TurboEngine(TurboConfig(n_layers=1, hidden_size=H, n_heads=hq, n_kv_heads=hkv, max_seq_len=ctx + 16,
                                      max_seqs=B, kv_dtype="f32", rope_variant="interleaved", rope_theta=1e6))
        for b in range(B):
            eng.kv_write(0, b, kv_k[b].contiguous(), kv_v[b].contiguous())
        if split:
            o = torch.cat([eng.decoder_layer_q8(0, range(8), x[:8].contiguous(), w),
                           eng.decoder_layer_q8(0, range(8, 16), x[8:].contiguous(), w)])
        else:
            o = eng.decoder_layer_q8(0, range(B), x, w)
        eng.sync()
        outs.append(o.cpu().numpy())
        eng.close()
    tol = F32_ATOL * max(1.0, float(np.abs(outs[1]).max()))
    assert_close(outs[0], outs[1], tol, what="decoder layer, integer form vs register form")

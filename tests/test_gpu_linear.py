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
    # 9-16 tokens on a matrix of at least 32 M weights: the tcgen05 pass (weights converted into TMEM,
    # x hi/lo as a 32-row B operand); 512 x 65536 has 4 row tiles, so its columns split into ranges
    # whose partial sums the last CTA of a row tile adds in order; bias and residual in the epilogue
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

"""K-E parity: the Q8 linear op (oomattn_q8_linear) against the oracle's
dequantise-then-matvec (src/quant.rs:201-224, src/oom_inference.rs:168-180),
on weights quantised by the oracle's restatement of the .oom writer
(src/gguf2oom.rs:719-770) and loaded through the library's stream unpacker.
f32 path tolerance: max-abs <= 1e-4."""
import os

import numpy as np
import pytest
import torch

from helpers import F32_ATOL, assert_close, make_engine

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden_q8.npz")


def _matrix(oracle, rows, cols, seed, scale=0.02):
    from oomllama_b200 import Q8Matrix
    w = (np.random.default_rng(seed).standard_normal((rows, cols)) * scale).astype(np.float32)
    stream = oracle.q8_quantize(w)
    wq = Q8Matrix.from_oom_stream(stream, rows, cols, device=0)
    wd = oracle.q8_dequantize(stream, rows * cols).reshape(rows, cols)
    return wq, wd


def _case(oracle, eng, rows, cols, T, seed, bias=True):
    wq, wd = _matrix(oracle, rows, cols, seed)
    rng = np.random.default_rng(seed + 1)
    x = rng.standard_normal((T, cols)).astype(np.float32)
    b = (rng.standard_normal(rows) * 0.1).astype(np.float32) if bias else None
    y = eng.q8_linear(wq, torch.from_numpy(x).cuda(), None if b is None else torch.from_numpy(b).cuda())
    eng.sync()
    ref = oracle.linear(x, wd, b)
    return y.cpu().numpy(), ref


@pytest.fixture(scope="module")
def eng():
    e = make_engine(8, 1, [16])
    yield e
    e.close()


def test_q8_linear_golden(eng):
    # the committed golden matrix: blocks straddle rows (cols = 320), a constant block, a NaN weight
    from oomllama_b200 import Q8Matrix
    g = np.load(GOLDEN)
    rows, cols = g["w"].shape
    wq = Q8Matrix.from_oom_stream(g["stream"], rows, cols, device=0)
    y = eng.q8_linear(wq, torch.from_numpy(g["x"]).cuda(), torch.from_numpy(g["b"]).cuda())
    eng.sync()
    assert_close(y.cpu().numpy(), g["y"], F32_ATOL, what="q8 golden")


@pytest.mark.parametrize("rows,cols,T", [(16, 64, 1), (64, 256, 3), (128, 320, 8), (48, 704, 9), (96, 512, 17),
                                         (32, 128, 70), (9488, 128, 13)])
def test_q8_linear_small(oracle, eng, rows, cols, T):
    # 9488 rows: a tall matrix (two row tiles per warp) whose last 32-row block is half outside it
    out, ref = _case(oracle, eng, rows, cols, T, seed=rows * 1000 + cols + T)
    assert_close(out, ref, F32_ATOL, what=f"q8 {rows}x{cols} T={T}")


@pytest.mark.parametrize("rows,cols,T", [(3584, 3584, 1), (512, 3584, 4), (3584, 18944, 2), (18944, 3584, 16),
                                         (3584, 18944, 11), (9488, 3584, 13)])
def test_q8_linear_qwen7b_shapes(oracle, eng, rows, cols, T):
    # Qwen2.5-7B projections: q/o 3584x3584, k/v 512x3584, down 3584x18944, gate/up 18944x3584.
    # 9..16 tokens on >= 32 M weights stage x in shared memory: down at T=11 runs 20 column
    # ranges merged in order; 9488 rows leave the last 512-row group partly outside the matrix
    out, ref = _case(oracle, eng, rows, cols, T, seed=rows + cols + T, bias=(rows != 18944))
    assert_close(out, ref, F32_ATOL, what=f"q8 {rows}x{cols} T={T}")


@pytest.mark.parametrize("rows,cols,T", [(512, 3584, 3), (3584, 18944, 11)])
def test_q8_linear_repeatable(oracle, eng, rows, cols, T):
    # split-K partials (and, for the 16-token form with x in shared memory, the
    # 10 column ranges of 3584x18944) are merged in split order by the last
    # CTA: identical bits on every call
    wq, _ = _matrix(oracle, rows, cols, seed=3)
    x = torch.randn(T, cols, generator=torch.Generator().manual_seed(4)).cuda()
    y1 = eng.q8_linear(wq, x).clone()
    y2 = eng.q8_linear(wq, x)
    eng.sync()
    assert torch.equal(y1, y2)


def test_q8_linear_rejects_odd_shapes(oracle, eng):
    from oomllama_b200 import Q8Matrix
    from oomllama_b200._lib import OomAttnError
    w = (np.random.default_rng(0).standard_normal((24, 64)) * 0.02).astype(np.float32)
    wq = Q8Matrix.from_oom_stream(oracle.q8_quantize(w), 24, 64, device=0)
    with pytest.raises(OomAttnError) as e:
        eng.q8_linear(wq, torch.zeros(1, 64, device="cuda"))
    assert e.value.code == 8


def test_q8_linear_reports_activation_outside_fp16(oracle, eng):
    # x enters the tensor cores as an fp16 hi / lo pair
    from oomllama_b200._lib import OomAttnError
    wq, _ = _matrix(oracle, 16, 64, seed=9)
    x = torch.zeros(1, 64, device="cuda")
    x[0, 5] = 70000.0
    eng.q8_linear(wq, x)
    with pytest.raises(OomAttnError) as e:
        eng.sync()
    assert e.value.code == 9
    eng.sync()

"""The bounded device waits end a kernel with a reported error instead of hanging it.

A test-only launch flag makes the bf16 decode's copy producer issue nothing, so every consumer's
mbarrier wait runs out its limit (set to 1 ms here): the kernel records the timeout bit and returns,
oomattn_sync reports OOMATTN_ERR_TIMEOUT, and the same context then decodes correctly.  Nothing
faults or hangs: the waits are the kernel's own bounded ones.  The reference has no device waits
(its only failure handling is a CPU fallback, src/oomllama.rs:702-719).  A second flag does the same
for the Q8 tensor-core pass."""
import numpy as np
import pytest
import torch

from helpers import BF16_ATOL, BF16_RTOL, as_f32_np, assert_close, make_engine, randn

pytestmark = pytest.mark.gpu


def test_decode_wait_runs_out_then_context_recovers(oracle):
    from oomllama_b200._lib import TEST_DROP_DECODE_COPIES, OomAttnError
    lens = [700, 33, 5000]
    eng = make_engine(28, 4, lens, kv_dtype="bf16", shuffle_seed=1)
    ks, vs = [], []
    for s, L in enumerate(lens):
        k, v = randn((L, 4, 128), 10 + s, torch.bfloat16), randn((L, 4, 128), 20 + s, torch.bfloat16)
        eng.kv_write(0, s, k.cuda(), v.cuda())
        ks.append(as_f32_np(k).transpose(1, 0, 2).copy())
        vs.append(as_f32_np(v).transpose(1, 0, 2).copy())
    q = randn((3, 28, 128), 30).cuda()
    eng.sync()
    eng.set_wait_limit(1_000_000)  # 1 ms
    eng.set_test_flags(TEST_DROP_DECODE_COPIES)
    eng.decode(0, [0, 1, 2], q)
    with pytest.raises(OomAttnError) as e:
        eng.sync()
    assert e.value.code == 6, str(e.value)  # OOMATTN_ERR_TIMEOUT
    eng.sync()  # the status word was cleared by the report
    eng.set_test_flags(0)
    eng.set_wait_limit(2_000_000_000)
    for _ in range(2):  # the split counters were left at zero: repeated decodes are correct
        out = eng.decode(0, [0, 1, 2], q).cpu().numpy()
        eng.sync()
        for s in range(3):
            ref = oracle.gqa_attention(as_f32_np(q[s:s + 1].cpu()), ks[s], vs[s], causal=False)[0]
            assert_close(out[s], ref, BF16_ATOL, BF16_RTOL, what=f"row {s} after the timeout")
    eng.close()


def test_q8_tensor_core_wait_runs_out_then_context_recovers():
    # the same for the Q8 tensor-core pass (16 tokens over 8192 x 4096): with its producer silent,
    # the MMA issuer's and promoters' waits run out, no cut tile is counted, and the next pass on the
    # same context is correct (against float64) and repeatable
    from oomllama_b200 import Q8Matrix
    from oomllama_b200._lib import TEST_DROP_LINEAR_COPIES, OomAttnError
    eng = make_engine(8, 1, [16])
    g = torch.Generator(device="cuda").manual_seed(3)
    rows, cols, T = 8192, 4096, 16
    nb = rows * cols // 256
    w = Q8Matrix(torch.randint(0, 256, (rows * cols,), dtype=torch.uint8, device="cuda", generator=g),
                 torch.rand(nb, device="cuda", generator=g) * 2e-4,
                 -torch.rand(nb, device="cuda", generator=g) * 0.02, rows, cols)
    x = torch.randn(T, cols, device="cuda", generator=g)
    eng.sync()
    eng.set_wait_limit(1_000_000)  # 1 ms
    eng.set_test_flags(TEST_DROP_LINEAR_COPIES)
    eng.q8_linear(w, x)
    with pytest.raises(OomAttnError) as e:
        eng.sync()
    assert e.value.code == 6, str(e.value)  # OOMATTN_ERR_TIMEOUT
    eng.set_test_flags(0)
    eng.set_wait_limit(2_000_000_000)
    y1 = eng.q8_linear(w, x)
    y2 = eng.q8_linear(w, x)
    eng.sync()
    q = w.q.view(rows, cols).double()
    wd = w.min.double().repeat_interleave(256).view(rows, cols) + q * w.scale.double().repeat_interleave(256).view(rows, cols)
    ref = (x.double() @ wd.T).cpu().numpy()
    assert_close(y1.cpu().numpy(), ref, 1e-4 * max(1.0, float(np.abs(ref).max())), what="q8 pass after the timeout")
    assert torch.equal(y1, y2)
    eng.close()


def test_test_flags_and_wait_limit_validated():
    from oomllama_b200._lib import OomAttnError
    eng = make_engine(8, 1, [16])
    with pytest.raises(OomAttnError):
        eng.set_test_flags(1 << 5)
    with pytest.raises(OomAttnError):
        eng.set_wait_limit(0)
    eng.close()

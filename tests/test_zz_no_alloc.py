"""The decode entry point for callers that cannot allocate device memory.

Some hosts cannot call cudaMalloc on the decode path -- their device memory is
owned by another allocator, or an allocation inside the token loop could stall
or fail.  oomattn_decode_static_scratch decodes over caller-owned paged K/V
memory with its split-KV scratch in a fixed array inside the library.  This
file checks, through the C ABI, that it matches oomattn_decode (the
context-based entry point) on two calls in a row, and that it rejects requests
beyond its fixed capacity.  It is named to be collected last.
"""
import ctypes

import numpy as np
import pytest
import torch

from helpers import make_engine, randn

pytestmark = pytest.mark.gpu

ATOL = 1e-5   # same kernels and inputs; only the split count may differ
RTOL = 1e-5


def _call(lib, dev, kv_dtype, kp, vp, n_pool_pages, bt, mpps, hq, hkv, seqs, lens, q, out, lse):
    err = ctypes.create_string_buffer(256)
    arr = lambda v: (ctypes.c_int32 * len(v))(*v)
    code = lib.oomattn_decode_static_scratch(
        dev, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), kv_dtype, ctypes.c_void_p(kp.data_ptr()),
        ctypes.c_void_p(vp.data_ptr()), n_pool_pages, ctypes.cast(ctypes.c_void_p(bt.data_ptr()),
                                                                  ctypes.POINTER(ctypes.c_int32)),
        mpps, hq, hkv, ctypes.c_float(0.0), len(seqs), arr(seqs), arr(lens), ctypes.c_void_p(q.data_ptr()),
        ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(lse.data_ptr()) if lse is not None else None, err, 256)
    return code, err.value.decode()


@pytest.mark.parametrize("kv_dtype", ["bf16", "f32"])
def test_static_scratch_decode_matches_context_decode(kv_dtype):
    from oomllama_b200 import _lib
    lib = _lib.load()
    hq, hkv = 28, 4
    lens = [1, 17, 530, 4100, 2048, 9000]
    eng = make_engine(hq, hkv, lens, kv_dtype=kv_dtype, shuffle_seed=7)
    dt = torch.bfloat16 if kv_dtype == "bf16" else torch.float32
    for s, L in enumerate(lens):
        eng.kv_write(0, s, randn((L, hkv, 128), 100 + s, dt).cuda(), randn((L, hkv, 128), 200 + s, dt).cuda())
    q = randn((len(lens), hq, 128), 5).cuda()
    ref, ref_lse = eng.decode(0, list(range(len(lens))), q, with_lse=True)
    eng.sync()
    # the same pages as make_engine assigned, as a caller-owned device block table
    pages = [-(-L // 16) for L in lens]
    perm = np.random.default_rng(7).permutation(sum(pages))
    mpps = max(pages)
    bt = np.zeros((len(lens), mpps), np.int32)
    o = 0
    for s, n in enumerate(pages):
        bt[s, :n] = perm[o:o + n]
        o += n
    bt_d = torch.from_numpy(bt).cuda()
    kp, vp = eng.kv_pool()
    n_pool_pages = kp.shape[1]
    code_dt = _lib.DTYPE_BF16 if kv_dtype == "bf16" else _lib.DTYPE_F32
    for _ in range(2):  # two calls in a row share (and must re-clear) the static scratch
        out = torch.full_like(q, float("nan"))
        lse = torch.full((len(lens), hq), float("nan"), device="cuda")
        code, msg = _call(lib, 0, code_dt, kp[0], vp[0], n_pool_pages, bt_d, mpps, hq, hkv, list(range(len(lens))),
                          lens, q, out, lse)
        assert code == 0, msg
        torch.cuda.synchronize()
        np.testing.assert_allclose(out.cpu().numpy(), ref.cpu().numpy(), atol=ATOL, rtol=RTOL)
        np.testing.assert_allclose(lse.cpu().numpy(), ref_lse.cpu().numpy(), atol=ATOL, rtol=RTOL)
    eng.close()


def test_static_scratch_rejects_requests_beyond_capacity():
    from oomllama_b200 import _lib
    lib = _lib.load()
    kp = torch.zeros(2, 1, 16, 128, dtype=torch.bfloat16, device="cuda")
    bt = torch.zeros(200, 1, dtype=torch.int32, device="cuda")
    q = torch.zeros(200, 8, 128, device="cuda")
    out = torch.empty_like(q)
    code, msg = _call(lib, 0, _lib.DTYPE_BF16, kp, kp, 2, bt, 1, 8, 1, list(range(200)), [16] * 200, q, out, None)
    assert code == 3 and "n_rows" in msg, msg
    code, msg = _call(lib, 0, _lib.DTYPE_BF16, kp, kp, 2, bt, 1, 8, 1, [0], [17], q, out, None)
    assert code == 3 and "length" in msg

"""The decode entry point for callers that cannot allocate device memory.

Some hosts cannot call cudaMalloc on the decode path -- their device memory is
owned by another allocator, or an allocation inside the token loop could stall
or fail.  oomattn_decode_static_scratch decodes over caller-owned paged K/V
memory with its split-KV scratch in a fixed array inside the library.  This
file checks, through the C ABI, that it matches oomattn_decode (the
context-based entry point) on two calls in a row -- also where the fixed array
caps the split count at 2 and at 1 -- that it matches the oracle, that it
reports a bad page id through oomattn_decode_static_scratch_status, and that it
rejects requests beyond its fixed capacity.  It is named to be collected last.
"""
import ctypes

import numpy as np
import pytest
import torch

from helpers import BF16_ATOL, BF16_RTOL, F32_ATOL, as_f32_np, assert_close, make_engine, randn

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


def _status(lib, dev=0):
    flags = ctypes.c_int32(-1)
    err = ctypes.create_string_buffer(256)
    code = lib.oomattn_decode_static_scratch_status(
        dev, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), ctypes.byref(flags), err, 256)
    return code, flags.value, err.value.decode()


def _pool_case(kv_dtype, hq, hkv, lens, seed):
    """A context whose pool is filled on the device (the caller-owned memory of the static call) and
    a block table of shuffled pages as a device tensor."""
    eng = make_engine(hq, hkv, lens, kv_dtype=kv_dtype, shuffle_seed=seed)
    for s, L in enumerate(lens):
        eng.set_seq_len(0, s, L)
    kp, vp = eng.kv_pool()
    g = torch.Generator(device="cuda").manual_seed(seed)
    kp[:, :-1].normal_(generator=g)
    vp[:, :-1].normal_(generator=g)
    pages = [-(-L // 16) for L in lens]
    perm = np.random.default_rng(seed).permutation(sum(pages))
    mpps = max(pages)
    bt = np.zeros((len(lens), mpps), np.int32)
    o = 0
    for s, n in enumerate(pages):
        bt[s, :n] = perm[o:o + n]
        o += n
    return eng, kp, vp, bt


@pytest.mark.parametrize("kv_dtype,hkv", [("bf16", 6), ("bf16", 9), ("f32", 6), ("f32", 9)])
def test_static_scratch_split_cap_two_and_one(kv_dtype, hkv):
    # 128 rows x 8 q heads per kv head: 6 kv heads give 6144 (row, head) pairs, so the fixed array
    # holds 2 splits each; 9 kv heads give 9216, so every row runs unsplit
    from oomllama_b200 import _lib
    lib = _lib.load()
    hq = hkv * 8
    lens = np.random.default_rng(hkv).integers(600, 3000, size=128).tolist()
    eng, kp, vp, bt = _pool_case(kv_dtype, hq, hkv, lens, seed=hkv)
    q = torch.randn(128, hq, 128, generator=torch.Generator(device="cuda").manual_seed(1), device="cuda")
    ref, ref_lse = eng.decode(0, list(range(128)), q, with_lse=True)
    eng.sync()
    bt_d = torch.from_numpy(bt).cuda()
    code_dt = _lib.DTYPE_BF16 if kv_dtype == "bf16" else _lib.DTYPE_F32
    for _ in range(2):
        out = torch.full_like(q, float("nan"))
        lse = torch.full((128, hq), float("nan"), device="cuda")
        code, msg = _call(lib, 0, code_dt, kp[0], vp[0], kp.shape[1], bt_d, bt.shape[1], hq, hkv, list(range(128)),
                          lens, q, out, lse)
        assert code == 0, msg
        torch.cuda.synchronize()
        np.testing.assert_allclose(out.cpu().numpy(), ref.cpu().numpy(), atol=ATOL, rtol=RTOL)
        np.testing.assert_allclose(lse.cpu().numpy(), ref_lse.cpu().numpy(), atol=ATOL, rtol=RTOL)
    assert _status(lib)[0] == 0
    eng.close()


@pytest.mark.parametrize("kv_dtype", ["bf16", "f32"])
def test_static_scratch_matches_oracle(oracle, kv_dtype):
    from oomllama_b200 import _lib
    lib = _lib.load()
    hq, hkv = 28, 4
    lens = [1, 16, 17, 700, 4100]
    eng, kp, vp, bt = _pool_case(kv_dtype, hq, hkv, lens, seed=11)
    q = torch.randn(len(lens), hq, 128, generator=torch.Generator(device="cuda").manual_seed(2), device="cuda")
    out = torch.empty_like(q)
    code, msg = _call(lib, 0, _lib.DTYPE_BF16 if kv_dtype == "bf16" else _lib.DTYPE_F32, kp[0], vp[0], kp.shape[1],
                      torch.from_numpy(bt).cuda(), bt.shape[1], hq, hkv, list(range(len(lens))), lens, q, out, None)
    assert code == 0, msg
    torch.cuda.synchronize()
    for s, L in enumerate(lens):
        pg = torch.from_numpy(bt[s, :-(-L // 16)].astype(np.int64)).cuda()
        kr = kp[0].index_select(0, pg).permute(1, 0, 2, 3).reshape(hkv, -1, 128)[:, :L]
        vr = vp[0].index_select(0, pg).permute(1, 0, 2, 3).reshape(hkv, -1, 128)[:, :L]
        ref = oracle.gqa_attention(as_f32_np(q[s:s + 1]), as_f32_np(kr), as_f32_np(vr), causal=False)[0]
        tol = (BF16_ATOL, BF16_RTOL) if kv_dtype == "bf16" else (F32_ATOL, None)
        assert_close(out[s].cpu().numpy(), ref, *tol, what=f"static scratch row {s} (len {L})")
    assert _status(lib)[0] == 0
    eng.close()


def test_static_scratch_reports_bad_page_id():
    # a page id past the pool is caught by the kernel's own bounds check: read as the pool's last
    # (zeroed) page and reported through the status call, which then clears it
    from oomllama_b200 import _lib
    lib = _lib.load()
    lens = [40, 20]
    eng, kp, vp, bt = _pool_case("bf16", 8, 1, lens, seed=5)
    bt[0, 1] = kp.shape[1] + 7
    q = torch.randn(2, 8, 128, device="cuda")
    out = torch.empty_like(q)
    code, msg = _call(lib, 0, _lib.DTYPE_BF16, kp[0], vp[0], kp.shape[1], torch.from_numpy(bt).cuda(), bt.shape[1],
                      8, 1, [0, 1], lens, q, out, None)
    assert code == 0, msg
    code, flags, msg = _status(lib)
    assert code == 9 and flags & 2, (code, flags, msg)
    assert torch.isfinite(out).all()
    assert _status(lib) == (0, 0, "")
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

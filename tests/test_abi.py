"""C-ABI checks that need no GPU: the library loads, exports every symbol the
header declares, validates configurations on the host, and builds the RoPE
table bit-identically to the oracle's f32 restatement."""
import ctypes
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    src = open(os.path.join(ROOT, "include", "oomattn.h")).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\*?(oomattn_\w+)\(", src, re.M)))


def test_header_declares_the_boundary():
    syms = header_symbols()
    for s in ("oomattn_create", "oomattn_attention_forward_with_bias", "oomattn_decode", "oomattn_prefill",
              "oomattn_rope_append", "oomattn_qkv_rope_append", "oomattn_merge_partials", "oomattn_reset",
              "oomattn_seq_len"):
        assert s in syms


def test_library_exports_every_header_symbol(lib):
    from oomllama_b200 import _lib
    syms = header_symbols()
    assert sorted(_lib.EXPORTS) == syms
    for s in syms:
        assert hasattr(lib, s), s
    assert b"sm_100a" in lib.oomattn_version()


def test_rope_table_matches_oracle_bitwise(lib, oracle):
    from oomllama_b200 import compute_rope_freqs
    for theta in (1e6, 5e5, 1e4):
        sin, cos = compute_rope_freqs(128, 33000, theta)
        c, s = oracle.rope_table(theta, 128, 33000)
        np.testing.assert_array_equal(cos.numpy(), c)
        np.testing.assert_array_equal(sin.numpy(), s)


def _cfg(**kw):
    from oomllama_b200 import _lib
    base = dict(n_layers=1, hidden_size=3584, n_heads=28, n_kv_heads=4, head_dim=128, max_seq_len=1024, max_seqs=2,
                page_size=16, n_pages=128, kv_dtype=0, rope_variant=1, rope_theta=1e6, softmax_scale=0.0)
    base.update(kw)
    return _lib.Config(**base)


@pytest.mark.parametrize("bad", [dict(head_dim=64), dict(page_size=32), dict(n_heads=28, n_kv_heads=3),
                                 dict(n_heads=36, n_kv_heads=2), dict(n_layers=0), dict(kv_dtype=7),
                                 dict(rope_variant=3), dict(rope_theta=0.0), dict(n_pages=0)])
def test_create_rejects_bad_config_on_host(lib, bad):
    ctx = ctypes.c_void_p()
    code = lib.oomattn_create(ctypes.byref(_cfg(**bad)), 0, None, ctypes.byref(ctx))
    assert code == 2  # OOMATTN_ERR_BAD_CONFIG, before any CUDA call
    assert not ctx.value


def test_null_arguments_rejected(lib):
    assert lib.oomattn_create(None, 0, None, None) == 1
    assert lib.oomattn_destroy(None) == 1
    assert lib.oomattn_sync(None) == 1
    assert lib.oomattn_compute_rope_table(ctypes.c_float(1e6), 128, 0, 4, None, None) == 1
    assert lib.oomattn_compute_rope_table(ctypes.c_float(1e6), 64, 0, 4, ctypes.c_void_p(1), ctypes.c_void_p(1)) == 2

"""ctypes binding of liboomattn.so (declarations in include/oomattn.h).

The library is the only compute path: if it is missing or fails to load, every
entry point raises -- there is no CPU or PyTorch fallback.
"""
from __future__ import annotations

import ctypes
import os

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "liboomattn.so")

OK = 0
STATUS_NAMES = {
    0: "OK", 1: "INVALID_ARG", 2: "BAD_CONFIG", 3: "OUT_OF_RANGE", 4: "CUDA", 5: "NCCL", 6: "TIMEOUT",
    7: "NO_MEMORY", 8: "UNSUPPORTED", 9: "DEVICE_CHECK",
}
DTYPE_F32, DTYPE_BF16 = 0, 1
PACKED_STRIDE = 132                 # floats per (row, q head) of a packed decode output: O[128], lse, pad
TEST_DROP_DECODE_COPIES = 1         # oomattn_set_test_flags: the bf16 decode's producer issues no copies
TEST_DROP_LINEAR_COPIES = 2         # oomattn_set_test_flags: the Q8 tensor-core pass's producer issues no copies
ROPE_SPLIT_HALF, ROPE_INTERLEAVED = 0, 1

# Every exported symbol of include/oomattn.h.
EXPORTS = (
    "oomattn_version", "oomattn_create", "oomattn_destroy", "oomattn_last_error", "oomattn_set_stream",
    "oomattn_sync", "oomattn_reset", "oomattn_seq_len", "oomattn_set_block_table", "oomattn_set_position_offset",
    "oomattn_set_seq_len", "oomattn_kv_pool", "oomattn_kv_write", "oomattn_kv_read", "oomattn_rope_table",
    "oomattn_compute_rope_table", "oomattn_rope_append", "oomattn_qkv_rope_append", "oomattn_decode", "oomattn_merge_partials",
    "oomattn_prefill", "oomattn_attention_forward_with_bias", "oomattn_decode_static_scratch",
    "oomattn_q8_unpack", "oomattn_q8_linear", "oomattn_rmsnorm", "oomattn_q8_mlp", "oomattn_decoder_layer_q8",
    "oomattn_embed_q8", "oomattn_argmax", "oomattn_decode_step_q8", "oomattn_oom_scan", "oomattn_q8_repack",
    "oomattn_set_wait_limit", "oomattn_set_test_flags", "oomattn_rope_q", "oomattn_decode_packed",
    "oomattn_merge_packed", "oomattn_decode_static_scratch_status", "oomattn_prefill_blocks",
    "oomattn_linear", "oomattn_prefill_step_q8",
)


class OomAttnError(RuntimeError):
    """A non-zero oomattn_status (the reference maps candle errors to RuntimeError, src/python.rs:139-141)."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"oomattn {STATUS_NAMES.get(code, code)}: {msg}")
        self.code = code


class Config(ctypes.Structure):
    _fields_ = [
        ("n_layers", ctypes.c_int32), ("hidden_size", ctypes.c_int32), ("n_heads", ctypes.c_int32),
        ("n_kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32), ("max_seq_len", ctypes.c_int32),
        ("max_seqs", ctypes.c_int32), ("page_size", ctypes.c_int32), ("n_pages", ctypes.c_int32),
        ("kv_dtype", ctypes.c_int32), ("rope_variant", ctypes.c_int32), ("rope_theta", ctypes.c_float),
        ("softmax_scale", ctypes.c_float),
    ]


class Q8Matrix(ctypes.Structure):
    """oomattn_q8_matrix: device pointers of a resident Q8 matrix [rows][cols]."""
    _fields_ = [("q", ctypes.c_void_p), ("scale", ctypes.c_void_p), ("min", ctypes.c_void_p),
                ("rows", ctypes.c_int32), ("cols", ctypes.c_int32)]


class Q8Layer(ctypes.Structure):
    """oomattn_q8_layer: one decoder layer's resident Q8 weights, biases and norm weights."""
    _fields_ = [("q", Q8Matrix), ("k", Q8Matrix), ("v", Q8Matrix), ("o", Q8Matrix), ("gate", Q8Matrix),
                ("up", Q8Matrix), ("down", Q8Matrix), ("bq", ctypes.c_void_p), ("bk", ctypes.c_void_p),
                ("bv", ctypes.c_void_p), ("input_norm", ctypes.c_void_p), ("post_norm", ctypes.c_void_p),
                ("eps", ctypes.c_float)]


class OomTensor(ctypes.Structure):
    """oomattn_oom_tensor: one tensor of an .oom file image (OomTensorMeta plus name and block extents)."""
    _fields_ = [("name_offset", ctypes.c_uint64), ("name_len", ctypes.c_uint32), ("quant_type", ctypes.c_uint32),
                ("num_blocks", ctypes.c_uint32), ("total_values", ctypes.c_uint32), ("data_offset", ctypes.c_uint64),
                ("data_bytes", ctypes.c_uint64)]


class Q8Model(ctypes.Structure):
    """oomattn_q8_model: the layers (host array), embedding, LM head and final norm of a Q8 model."""
    _fields_ = [("n_layers", ctypes.c_int32), ("layers", ctypes.POINTER(Q8Layer)), ("embed", Q8Matrix),
                ("lm_head", Q8Matrix), ("final_norm", ctypes.c_void_p), ("eps", ctypes.c_float)]


_lib = None


def load():
    """Load liboomattn.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m oomllama_b200.build`")
    L = ctypes.CDLL(LIB_PATH)
    P, I, F = ctypes.c_void_p, ctypes.c_int32, ctypes.c_float
    IP = ctypes.POINTER(ctypes.c_int32)
    sig = {
        "oomattn_version": ([], ctypes.c_char_p),
        "oomattn_create": ([ctypes.POINTER(Config), ctypes.c_int, P, ctypes.POINTER(P)], ctypes.c_int),
        "oomattn_destroy": ([P], ctypes.c_int),
        "oomattn_last_error": ([P], ctypes.c_char_p),
        "oomattn_set_stream": ([P, P], ctypes.c_int),
        "oomattn_sync": ([P], ctypes.c_int),
        "oomattn_reset": ([P], ctypes.c_int),
        "oomattn_seq_len": ([P, I, I, IP], ctypes.c_int),
        "oomattn_set_block_table": ([P, I, IP, I], ctypes.c_int),
        "oomattn_set_position_offset": ([P, I, I], ctypes.c_int),
        "oomattn_set_seq_len": ([P, I, I, I], ctypes.c_int),
        "oomattn_kv_pool": ([P, ctypes.POINTER(P), ctypes.POINTER(P)], ctypes.c_int),
        "oomattn_kv_write": ([P, I, I, P, P, I, I], ctypes.c_int),
        "oomattn_kv_read": ([P, I, I, P, P], ctypes.c_int),
        "oomattn_rope_table": ([P, I, I, P, P], ctypes.c_int),
        "oomattn_compute_rope_table": ([F, I, I, I, P, P], ctypes.c_int),
        "oomattn_rope_append": ([P, I, I, IP, I, P, P, P, I, P, P, P, P, I], ctypes.c_int),
        "oomattn_qkv_rope_append": ([P, I, I, IP, I, P, P, P, P, I, P, P, P, P, I], ctypes.c_int),
        "oomattn_decode": ([P, I, I, IP, IP, P, P, P], ctypes.c_int),
        "oomattn_merge_partials": ([P, I, I, P, P, P, P], ctypes.c_int),
        "oomattn_prefill": ([P, I, I, I, P, P, I, P], ctypes.c_int),
        "oomattn_attention_forward_with_bias": ([P, I, I, I, P, P, P, P, P, I, P, P, P, P], ctypes.c_int),
        "oomattn_decode_static_scratch": ([ctypes.c_int, P, I, P, P, I, P, I, I, I, F, I, IP, IP, P, P, P,
                                           ctypes.c_char_p, I], ctypes.c_int),
        "oomattn_q8_unpack": ([P, ctypes.c_uint64, ctypes.c_int64, P, P, P, ctypes.c_char_p, I], ctypes.c_int),
        "oomattn_q8_linear": ([P, ctypes.POINTER(Q8Matrix), P, I, P, P], ctypes.c_int),
        "oomattn_rmsnorm": ([P, P, P, F, I, I, P], ctypes.c_int),
        "oomattn_q8_mlp": ([P, ctypes.POINTER(Q8Matrix), ctypes.POINTER(Q8Matrix), ctypes.POINTER(Q8Matrix), P, I, P,
                            P], ctypes.c_int),
        "oomattn_decoder_layer_q8": ([P, I, I, IP, P, ctypes.POINTER(Q8Layer), P], ctypes.c_int),
        "oomattn_embed_q8": ([P, ctypes.POINTER(Q8Matrix), P, I, P], ctypes.c_int),
        "oomattn_argmax": ([P, P, I, I, P], ctypes.c_int),
        "oomattn_decode_step_q8": ([P, ctypes.POINTER(Q8Model), I, IP, P, P, P], ctypes.c_int),
        "oomattn_oom_scan": ([P, ctypes.c_uint64, ctypes.POINTER(OomTensor), I, ctypes.POINTER(ctypes.c_int32),
                              ctypes.c_char_p, I], ctypes.c_int),
        "oomattn_q8_repack": ([P, P, ctypes.c_uint64, ctypes.c_int64, P, P, P], ctypes.c_int),
        "oomattn_set_wait_limit": ([P, ctypes.c_uint64], ctypes.c_int),
        "oomattn_set_test_flags": ([P, I], ctypes.c_int),
        "oomattn_rope_q": ([P, I, IP, P, I, P, P, I], ctypes.c_int),
        "oomattn_decode_packed": ([P, I, I, IP, IP, P, P], ctypes.c_int),
        "oomattn_merge_packed": ([P, I, I, P, P, P], ctypes.c_int),
        "oomattn_decode_static_scratch_status": ([ctypes.c_int, P, IP, ctypes.c_char_p, I], ctypes.c_int),
        "oomattn_prefill_blocks": ([P, I, I, I, P, P, I, P, I, IP], ctypes.c_int),
        "oomattn_linear": ([P, P, P, I, I, I, I, P, P], ctypes.c_int),
        "oomattn_prefill_step_q8": ([P, ctypes.POINTER(Q8Model), I, IP, I, P, P, P], ctypes.c_int),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res
    _lib = L
    return L


def int_array(values):
    vals = [int(v) for v in values]
    return (ctypes.c_int32 * max(1, len(vals)))(*vals)


def check(ctx, code: int):
    if code != OK:
        msg = load().oomattn_last_error(ctx) if ctx else b""
        raise OomAttnError(code, (msg or b"").decode(errors="replace"))

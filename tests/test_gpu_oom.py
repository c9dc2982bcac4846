"""The device repack of .oom Q8 tensors (oomattn_q8_repack) against the host
block walk (oomattn_q8_unpack, src/quant.rs:431-463) and the golden vectors:
bit-exact q, scale and min, from block streams at every byte alignment, and a
damaged length field reported by oomattn_sync."""
import os

import numpy as np
import pytest
import torch

from helpers import F32_ATOL, assert_close, make_engine

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def eng():
    e = make_engine(2, 1, [16])
    yield e
    e.close()


@pytest.fixture(scope="module")
def oom():
    from oomllama_b200 import OomFile
    with open(os.path.join(GOLD, "golden.oom"), "rb") as f:
        return OomFile(f.read())


def _same(w, blocks, n):
    from oomllama_b200 import q8_unpack
    q, sc, mn = q8_unpack(np.asarray(blocks), n)
    assert np.array_equal(w.q.cpu().numpy(), q)
    assert np.array_equal(w.scale.cpu().numpy().view(np.uint32), sc.view(np.uint32))
    assert np.array_equal(w.min.cpu().numpy().view(np.uint32), mn.view(np.uint32))


def test_repack_golden_tensors(eng, oom):
    for name, rows, cols in (("model.layers.0.mlp.up_proj.weight", 48, 320), ("lm_head.weight", 48, 320)):
        w = oom.q8_matrix(eng, name, rows, cols)
        eng.sync()
        _same(w, oom.blocks(name), rows * cols)
    t = oom.tensors["model.layers.0.self_attn.q_proj.bias"]
    w = oom.q8_matrix(eng, "model.layers.0.self_attn.q_proj.bias", 1, t.total_values)  # 300 values: partial block
    eng.sync()
    _same(w, oom.blocks("model.layers.0.self_attn.q_proj.bias"), t.total_values)


def test_repack_from_a_whole_file_upload(eng, oom):
    # one upload of the file image; each tensor's blocks start at their own byte offset (58, 16485, 16836)
    img = torch.from_numpy(np.asarray(oom.image).copy())
    dev = torch.zeros((img.numel() + 3) // 4 * 4, dtype=torch.uint8, device="cuda")
    dev[:img.numel()].copy_(img)
    for name, m in oom.tensors.items():
        if m.quant_type != 8:
            continue
        w = eng.q8_repack(dev[m.data_offset:m.data_offset + m.data_bytes], m.total_values)
        eng.sync()
        _same(w, oom.blocks(name), m.total_values)


@pytest.mark.parametrize("shift", [0, 1, 2, 3])
def test_repack_alignments_and_the_linear(eng, shift):
    from oomllama_b200 import Q8Matrix
    g = np.load(os.path.join(GOLD, "golden_q8.npz"))
    buf = torch.zeros(g["stream"].size + 8, dtype=torch.uint8, device="cuda")
    buf[shift:shift + g["stream"].size].copy_(torch.from_numpy(g["stream"]))
    w = eng.q8_repack(buf[shift:shift + g["stream"].size], g["w"].size, 48, 320)
    eng.sync()
    _same(w, g["stream"], g["w"].size)
    y = eng.q8_linear(Q8Matrix(w.q, w.scale, w.min, 48, 320), torch.from_numpy(g["x"]).cuda(),
                      torch.from_numpy(g["b"]).cuda())
    eng.sync()
    assert_close(y.cpu().numpy(), g["y"], F32_ATOL, what="linear on repacked weights")


def test_repack_reports_a_damaged_length(eng):
    from oomllama_b200._lib import OomAttnError
    g = np.load(os.path.join(GOLD, "golden_q8.npz"))
    s = g["stream"].copy()
    s[268 * 3 + 8:268 * 3 + 12] = np.frombuffer(np.uint32(200).tobytes(), np.uint8)  # block 3 claims 200 values
    eng.q8_repack(torch.from_numpy(s).cuda(), g["w"].size)
    with pytest.raises(OomAttnError) as e:
        eng.sync()
    assert e.value.code == 9
    eng.sync()


def test_repack_rejects_a_wrong_stream_size(eng):
    from oomllama_b200._lib import OomAttnError
    g = np.load(os.path.join(GOLD, "golden_q8.npz"))
    with pytest.raises(OomAttnError) as e:
        eng.q8_repack(torch.from_numpy(g["stream"][:-1]).cuda(), g["w"].size)
    assert e.value.code == 1

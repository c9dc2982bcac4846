"""Generates tests/golden/golden.oom: a small .oom file image laid out as the
reference's writer lays it (src/gguf2oom.rs:708-716 header, :782-829 Q8
tensors, :835-861 raw f32 tensors), assembled with struct.pack from the Q8
block streams of tests/golden/golden_q8.npz (themselves an independent numpy
restatement of the Q8 writer):

  "OOML", u32 version 1, u32 tensor count, then per tensor
  u32 name length, name bytes, u8 quant type (8 Q8, 0 f32), u32 blocks,
  u32 values, and the blocks [f32 scale][f32 min][u32 len][len bytes]
  (a raw f32 tensor is one block: scale 0, min 0, len = 4 * values).

Tensors, in file order:
  model.layers.0.mlp.up_proj.weight   Q8 48 x 320 (blocks straddle rows, a NaN weight)
  model.norm.weight                   f32, 64 values
  model.layers.0.self_attn.q_proj.bias  Q8, 300 values (a partial last block)
  lm_head.weight                      Q8 48 x 320 again (a second copy, after an odd-length name)
Also writes golden_oom_meta.npz with the expected scan table.
Run from the repository root:  python tests/golden/make_golden_oom.py
"""
import os
import struct

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def main():
    g = np.load(os.path.join(HERE, "golden_q8.npz"))
    norm = (1.0 + 0.01 * np.arange(64)).astype(np.float32)
    tensors = [
        ("model.layers.0.mlp.up_proj.weight", 8, g["stream"].tobytes(), g["w"].size, (g["w"].size + 255) // 256),
        ("model.norm.weight", 0, struct.pack("<ffI", 0.0, 0.0, 4 * norm.size) + norm.tobytes(), norm.size, 1),
        ("model.layers.0.self_attn.q_proj.bias", 8, g["stream_tail"].tobytes(), g["tail"].size, 2),
        ("lm_head.weight", 8, g["stream"].tobytes(), g["w"].size, (g["w"].size + 255) // 256),
    ]
    out = bytearray(b"OOML" + struct.pack("<II", 1, len(tensors)))
    meta = {"name_offset": [], "name_len": [], "quant_type": [], "num_blocks": [], "total_values": [],
            "data_offset": [], "data_bytes": []}
    for name, qt, blocks, n, nb in tensors:
        nm = name.encode()
        out += struct.pack("<I", len(nm))
        meta["name_offset"].append(len(out))
        meta["name_len"].append(len(nm))
        out += nm
        out += struct.pack("<BII", qt, nb, n)
        meta["quant_type"].append(qt)
        meta["num_blocks"].append(nb)
        meta["total_values"].append(n)
        meta["data_offset"].append(len(out))
        meta["data_bytes"].append(len(blocks))
        out += blocks
    with open(os.path.join(HERE, "golden.oom"), "wb") as f:
        f.write(bytes(out))
    np.savez(os.path.join(HERE, "golden_oom_meta.npz"), names=np.array([t[0] for t in tensors]), norm=norm,
             **{k: np.array(v, np.int64) for k, v in meta.items()})


if __name__ == "__main__":
    main()

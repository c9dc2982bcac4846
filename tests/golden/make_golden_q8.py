"""Generates tests/golden/golden_q8.npz: known-answer vectors for the .oom Q8
format and the Q8 linear op, computed by a numpy restatement independent of
the C oracle, from the reference's formulas:

  stream       the block stream of add_tensor_q8 (src/gguf2oom.rs:719-770):
               per 256 values [f32 scale][f32 min][u32 len][len bytes q],
               min/max from f32::MAX / f32::MIN (NaN never updates them),
               scale = range / 255 (0 when |range| < 1e-9),
               q = round-half-away((v - min) / scale) saturated to u8 (NaN -> 0)
  deq          min + (f32)q * scale, separately rounded
               (BlockQ8View::dequantize_fast, src/quant.rs:201-224)
  y            x @ W^T + b in float64 on the dequantised W
               (matvec, src/oom_inference.rs:168-180)

The values include a partial last block, a constant block (scale 0), a block
holding a NaN and blocks straddling matrix rows (cols = 320).
Run from the repository root:  python tests/golden/make_golden_q8.py
"""
import os
import struct

import numpy as np

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden_q8.npz")
F32 = np.float32


def quantize(values):
    v = np.asarray(values, F32).ravel()
    out = bytearray()
    for start in range(0, v.size, 256):
        blk = v[start:start + 256]
        mn, mx = F32(3.4028234663852886e38), F32(-3.4028234663852886e38)
        for x in blk:  # sequential compares, as the writer's loop
            if x < mn:
                mn = x
            if x > mx:
                mx = x
        rng = F32(mx - mn)
        scale = F32(0.0) if abs(rng) < F32(1e-9) else F32(rng / F32(255.0))
        q = np.zeros(blk.size, np.uint8)
        if scale != 0:
            r = (blk - mn).astype(F32) / scale  # f32 subtract and divide
            r = r.astype(F32).astype(np.float64)
            rr = np.sign(r) * np.floor(np.abs(r) + 0.5)  # round half away from zero (exact in f64)
            rr = np.where(np.isnan(rr), 0, np.clip(rr, 0, 255))
            q = rr.astype(np.uint8)
        out += struct.pack("<ffI", float(scale), float(mn), blk.size) + q.tobytes()
    return np.frombuffer(bytes(out), np.uint8)


def dequantize(stream, n):
    s = bytes(stream)
    off, pos, out = 0, 0, np.empty(n, F32)
    while pos < n:
        scale, mn, length = struct.unpack_from("<ffI", s, off)
        off += 12
        num = min(256, n - pos)
        q = np.frombuffer(s, np.uint8, num, off).astype(F32)
        out[pos:pos + num] = (F32(mn) + (q * F32(scale)).astype(F32)).astype(F32)
        off += length
        pos += num
    return out


def main():
    rng = np.random.default_rng(20240806)
    rows, cols = 48, 320                       # 15360 values: 60 blocks, many straddle rows
    w = (rng.standard_normal((rows, cols)) * 0.02).astype(F32)
    w[1, :] = F32(0.125)                       # row 1 is constant: block 1 (values 256..511) keeps scale > 0
    w.ravel()[512:768] = F32(-0.5)             # block 2 is constant: scale 0, q 0
    w.ravel()[1000] = np.nan                   # block 3 holds a NaN (q 0, excluded from min / max)
    w.ravel()[1300] = F32(3.0)                 # a large value widens block 5's range
    flat = w.ravel()
    tail = (rng.standard_normal(300) * 0.5).astype(F32)  # a 300-value tensor: partial last block
    stream = quantize(flat)
    stream_tail = quantize(tail)
    deq = dequantize(stream, flat.size)
    deq_tail = dequantize(stream_tail, tail.size)
    wd = deq.reshape(rows, cols).astype(np.float64)
    wd[~np.isfinite(wd)] = 0.0                 # the NaN dequantises to min (finite) in any case
    x = rng.standard_normal((5, cols)).astype(F32)
    b = (rng.standard_normal(rows) * 0.1).astype(F32)
    y = x.astype(np.float64) @ wd.T + b.astype(np.float64)
    np.savez_compressed(OUT, w=w, stream=stream, deq=deq, tail=tail, stream_tail=stream_tail, deq_tail=deq_tail,
                        x=x, b=b, y=y)
    print("wrote", OUT, stream.size, "stream bytes")


if __name__ == "__main__":
    main()

"""ggml block layouts (ggml.nim:23-32): QK = 32 weights per block.

  BlockQ8_0 = fp16 d + 32 x int8           34 bytes   value = d * q
  BlockQ4_0 = fp16 d + 16 bytes (nibbles)  18 bytes   value = d * (nibble - 8),
              low nibbles are lanes 0..15, high nibbles lanes 16..31
"""
import numpy as np

QK = 32
Q8_0_BYTES = 34
Q4_0_BYTES = 18

BlockQ8_0 = np.dtype([("d", "<u2"), ("qs", "i1", (QK,))])
BlockQ4_0 = np.dtype([("d", "<u2"), ("qs", "u1", (QK // 2,))])
assert BlockQ8_0.itemsize == Q8_0_BYTES and BlockQ4_0.itemsize == Q4_0_BYTES

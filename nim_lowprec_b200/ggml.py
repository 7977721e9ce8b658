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

# k-quant super-blocks (ggml.nim:108-124), dequantize only
QK_K = 256
Q4_K_BYTES = 144
Q6_K_BYTES = 210
BlockQ4_K = np.dtype([("d", "<u2"), ("dmin", "<u2"), ("scales", "u1", (12,)),
                      ("qs", "u1", (QK_K // 2,))])
BlockQ6_K = np.dtype([("ql", "u1", (QK_K // 2,)), ("qh", "u1", (QK_K // 4,)),
                      ("scales", "i1", (QK_K // 16,)), ("d", "<u2")])
assert BlockQ4_K.itemsize == Q4_K_BYTES and BlockQ6_K.itemsize == Q6_K_BYTES

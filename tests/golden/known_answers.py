"""Known-answer dequantization vectors of the reference's own unit tests.

Each case restates one hand-built block of cllm_inference tests/quant_test.cpp
(the line numbers are given per case) as (type, block bytes, {index: value}).
Bytes not listed are zero; fp16 1.0 is 0x3C00, stored little-endian.
"""

Q4_0, Q5_0, Q8_0, Q4_K, Q5_K, Q6_K = 2, 6, 8, 12, 13, 14


def _block(size, sets):
    b = bytearray(size)
    for off, val in sets:
        b[off] = val
    return bytes(b)


CASES = [
    # quant_test.cpp:58-67  d=1.0, qs[0]=0x9A -> elem0=2, elem16=1, elem1=-8
    ("Q4_0", Q4_0, _block(18, [(0, 0x00), (1, 0x3C), (2, 0x9A)]), 32, {0: 2.0, 16: 1.0, 1: -8.0}),
    # quant_test.cpp:83-92  qh bit0 set, qs[0]=0x21 -> elem0=1, elem16=-14
    ("Q5_0", Q5_0, _block(22, [(1, 0x3C), (2, 0x01), (6, 0x21)]), 32, {0: 1.0, 16: -14.0}),
    # quant_test.cpp:108-117  qs[0]=0xFF -> -1, qs[1]=2
    ("Q8_0", Q8_0, _block(34, [(1, 0x3C), (2, 0xFF), (3, 0x02)]), 32, {0: -1.0, 1: 2.0}),
    # quant_test.cpp:173-186  scales {1,1,1,1,0,0,0,0,1,1,1,1}, qs[0]=0x21
    ("Q4_K", Q4_K, _block(144, [(1, 0x3C)] + [(4 + i, v) for i, v in enumerate([1, 1, 1, 1, 0, 0, 0, 0, 1, 1, 1, 1])]
                          + [(16, 0x21)]), 256, {0: 1.0, 32: 2.0, 1: 0.0}),
    # quant_test.cpp:189-206  same scales, qs[0]=0x21 at offset 48
    ("Q5_K", Q5_K, _block(176, [(1, 0x3C)] + [(4 + i, v) for i, v in enumerate([1, 1, 1, 1, 0, 0, 0, 0, 1, 1, 1, 1])]
                          + [(48, 0x21)]), 256, {0: 1.0, 32: 2.0}),
    # quant_test.cpp:200-205  plus qh[0] bit0 -> elem0 = 17
    ("Q5_K_qh", Q5_K, _block(176, [(1, 0x3C)] + [(4 + i, v) for i, v in enumerate([1, 1, 1, 1, 0, 0, 0, 0, 1, 1, 1, 1])]
                             + [(48, 0x21), (16, 0x01)]), 256, {0: 17.0}),
    # quant_test.cpp:209-218  all 16 scales 1, ql[0]=0x21, d=1.0 at 208 -> elem0=-31, elem64=-30
    ("Q6_K", Q6_K, _block(210, [(192 + i, 1) for i in range(16)] + [(0, 0x21), (209, 0x3C)]), 256,
     {0: -31.0, 64: -30.0}),
]

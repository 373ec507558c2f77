"""Hand-built K-quant edge-case blocks (shared by the oracle and GPU tests and the golden
fixture script): every packed 6-bit scale/min field position (phi4.rs:492-498), every
Q5_K qh bit (phi4.rs:535), every Q6_K quad/half with scales -128 and 127 (phi4.rs:458-475)
and subnormal / zero / signed / non-finite f16 d values."""
import numpy as np

F16_SPECIAL = [0x0000, 0x8000, 0x0001, 0x03FF, 0x0400, 0x3C00, 0xBC00, 0x7BFF, 0x7C00, 0xFC00, 0x7E00]


def _f16(bits):
    return np.array([bits], np.uint16).view(np.uint8)


def q4k_edge() -> np.ndarray:
    blocks = []
    # one block per (scale byte, bit): isolates every bit of the 12-byte packed field
    for byte in range(12):
        for bit in range(8):
            b = np.zeros(144, np.uint8)
            b[0:2] = _f16(0x3C00)   # d = 1
            b[2:4] = _f16(0x3800)   # dmin = 0.5
            b[4 + byte] = 1 << bit
            b[16:144] = (np.arange(128) * 37 % 256).astype(np.uint8)
            blocks.append(b)
    for d in F16_SPECIAL:
        b = np.full(144, 0xFF, np.uint8)
        b[0:2] = _f16(d)
        b[2:4] = _f16(F16_SPECIAL[(F16_SPECIAL.index(d) + 3) % len(F16_SPECIAL)])
        blocks.append(b)
    return np.concatenate(blocks)


def q5k_edge() -> np.ndarray:
    blocks = []
    for byte in range(12):
        for bit in range(8):
            b = np.zeros(176, np.uint8)
            b[0:2] = _f16(0x3C00)
            b[2:4] = _f16(0x3800)
            b[4 + byte] = 1 << bit
            b[16:48] = (np.arange(32) * 11 % 256).astype(np.uint8)
            b[48:176] = (np.arange(128) * 53 % 256).astype(np.uint8)
            blocks.append(b)
    for j in range(32):       # every qh byte, all bits set / single bits
        b = np.zeros(176, np.uint8)
        b[0:2] = _f16(0x3C00)
        b[4:16] = 0xFF
        b[16 + j] = 1 << (j % 8)
        blocks.append(b)
    for d in F16_SPECIAL:
        b = np.full(176, 0xA5, np.uint8)
        b[0:2] = _f16(d)
        b[2:4] = _f16(0x0001)
        blocks.append(b)
    return np.concatenate(blocks)


def q6k_edge() -> np.ndarray:
    blocks = []
    for sc in (-128, 127, -1, 0, 1, -32, 31):
        b = np.zeros(210, np.uint8)
        b[0:128] = (np.arange(128) * 29 % 256).astype(np.uint8)
        b[128:192] = (np.arange(64) * 97 % 256).astype(np.uint8)
        b[192:208] = np.array([sc] * 16, np.int8).view(np.uint8)
        b[208:210] = _f16(0x3C00)
        blocks.append(b)
    for s in range(16):       # each of the 16 scale slots distinct (catches is = g*8 + l/16)
        b = np.zeros(210, np.uint8)
        b[0:128] = 0xFF
        b[128:192] = 0xFF
        sc = np.zeros(16, np.int8)
        sc[s] = -128 if s % 2 else 127
        b[192:208] = sc.view(np.uint8)
        b[208:210] = _f16(0x3C00)
        blocks.append(b)
    for d in F16_SPECIAL:
        b = np.full(210, 0x5A, np.uint8)
        b[192:208] = np.array([-128, 127] * 8, np.int8).view(np.uint8)
        b[208:210] = _f16(d)
        blocks.append(b)
    return np.concatenate(blocks)


EDGE = {12: q4k_edge, 13: q5k_edge, 14: q6k_edge}

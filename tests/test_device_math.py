"""CPU checks of integer/float tricks the CUDA kernels rely on, restated on the host with the kernels' own constants.

* q8_K rounding without the conversion unit (b2q_device.cuh q8_K_bits): for every product p the quantizer can form
  (|p| <= 127 + ulp), the low byte of the bits of fl(min(p, 127) + 1.5 * 2^23) is the byte of min(127, rint(p)).
* IQ4_NL level lookup by byte permutes (gemv_kernels.cuh iq4nl_levels4 and the per-word form in chunk_dot): PTX prmt
  emulated here; every 16-bit group of four nibbles gives the four table levels in nibble order, and the activation
  interleave (iq4nl_interleave) lines each level up with its value's activation, so the dp4a sum is the block dot.
"""

import os
import re

import numpy as np

from oracle import ref

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
KERNELS = os.path.join(ROOT, "comp_b200", "csrc", "gemv_kernels.cuh")


def _prmt(a, b, sel):
    """PTX prmt.b32 default mode: result byte j = byte (sel_j & 7) of the 8-byte value {b, a}; sel_j & 8 replicates
    that byte's sign bit (sel_j = bits 4j..4j+3 of sel, j = 0..3)."""
    src = [(a >> (8 * i)) & 0xFF for i in range(4)] + [(b >> (8 * i)) & 0xFF for i in range(4)]
    out = 0
    for j in range(4):
        nib = (sel >> (4 * j)) & 0xF
        byte = src[nib & 7]
        if nib & 8:
            byte = 0xFF if byte & 0x80 else 0x00
        out |= byte << (8 * j)
    return out


def _table_words():
    text = open(KERNELS).read()
    words = {int(m.group(1)): int(m.group(2), 16) for m in re.finditer(r"kIq4Lv(\d) = 0x([0-9A-Fa-f]+)u", text)}
    return [words[i] for i in range(4)]


def _levels4(nibs, t):
    lo = _prmt(t[0], t[1], nibs & 0x7777)
    hi = _prmt(t[2], t[3], nibs & 0x7777)
    return _prmt(lo, hi, 0x3210 | ((nibs >> 1) & 0x4444))


def _s8(byte):
    return byte - 256 if byte >= 128 else byte


def test_q8_K_rounding_by_magic_add_is_exact():
    f32 = np.float32
    ties = np.arange(-127.5, 128.0, 0.5, dtype=f32)
    near = np.concatenate([np.nextafter(ties, f32(np.inf)), np.nextafter(ties, f32(-np.inf))])
    rng = np.random.default_rng(0)
    rand = rng.uniform(-127.01, 127.01, 2_000_000).astype(f32)
    p = np.concatenate([ties, near, rand, np.array([0.0, -0.0, 127.0, -127.0, 1e-30, -1e-30], f32)])
    bits = (np.minimum(p, f32(127.0)) + f32(12582912.0)).astype(f32).view(np.uint32)
    got = (bits & 0xFF).astype(np.uint8)
    want = np.minimum(np.rint(p), f32(127.0)).astype(np.int32).astype(np.uint8)
    assert np.array_equal(got, want)


def test_iq4_nl_levels_by_byte_permute():
    t = _table_words()
    levels = [_s8((t[v // 4] >> (8 * (v % 4))) & 0xFF) for v in range(16)]
    assert levels == ref.IQ4_NL_LEVELS.tolist()
    for nibs in range(1 << 16):
        got = _levels4(nibs, t)
        for j in range(4):
            assert _s8((got >> (8 * j)) & 0xFF) == levels[(nibs >> (4 * j)) & 0xF]


def test_iq4_nl_interleave_lines_up_levels_and_activations():
    """One 16-byte chunk (32 values) of random nibbles and activations: the dp4a sums over looked-up words and
    interleaved activation words equal the natural-order block dot."""
    t = _table_words()
    rng = np.random.default_rng(1)
    for _ in range(200):
        q = rng.integers(0, 256, 16, dtype=np.uint8)
        x = rng.integers(-128, 128, 32).astype(np.int64)
        vals = np.concatenate([ref.IQ4_NL_LEVELS[q & 15], ref.IQ4_NL_LEVELS[q >> 4]]).astype(np.int64)
        want = int(np.dot(vals, x))
        xb = (x & 0xFF).astype(np.uint32)
        xw0 = [int(xb[4 * k] | xb[4 * k + 1] << 8 | xb[4 * k + 2] << 16 | xb[4 * k + 3] << 24) for k in range(4)]
        xw1 = [int(xb[16 + 4 * k] | xb[17 + 4 * k] << 8 | xb[18 + 4 * k] << 16 | xb[19 + 4 * k] << 24) for k in range(4)]
        s = 0
        for k in range(4):
            wk = int(q[4 * k]) | int(q[4 * k + 1]) << 8 | int(q[4 * k + 2]) << 16 | int(q[4 * k + 3]) << 24
            ia, ib = _prmt(xw0[k], xw1[k], 0x5140), _prmt(xw0[k], xw1[k], 0x7362)  # iq4nl_interleave
            va, vb = _levels4(wk & 0xFFFF, t), _levels4(wk >> 16, t)
            for v, xi in ((va, ia), (vb, ib)):
                s += sum(_s8((v >> (8 * j)) & 0xFF) * _s8((xi >> (8 * j)) & 0xFF) for j in range(4))
        assert s == want

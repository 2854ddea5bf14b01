"""TEST INFRASTRUCTURE ONLY (see oracle/__init__.py): numpy restatement of the reference's math.

Each function cites the reference file:line it restates (paths inside the komp project). Float work is done in the
precision the reference uses (f32 for the quantizers, IEEE round-to-nearest; f64 for KURN's reference dot), so the
results are bit-identical, not approximate.
"""

import numpy as np

# q8_0 weights are an extension beyond the reference (which has Q4_0 and TQ2_0 only): ggml's Q8_0 block of an f16 scale
# and 32 int8 values, against q8_0 activations, with Q4_0's multiply order; pinned to gguf-py's Q8_0 codec.
# iq4_nl weights are a second extension: ggml's IQ4_NL block (f16 scale, 16 bytes of nibbles laid out as Q4_0's) whose
# nibbles index a fixed table of 16 int8 levels instead of nibble - 8; q8_0 activations and Q4_0's multiply order;
# pinned to gguf-py's IQ4_NL codec.
# q4_k weights are a third extension: ggml's Q4_K super-block of 256 values (f16 d and dmin, eight 6-bit sub-block
# scales and mins packed in 12 bytes, 128 bytes of nibbles), value = d * sc_j * q - dmin * m_j for sub-block j of 32
# values, against q8_K activations; pinned to gguf-py's Q4_K codec. Its split planes are this backend's own layout
# (split_q4_k below): nibbles regrouped so each 16-byte chunk holds one sub-block laid out as a Q4_0 block, and the
# scales unpacked to 20 bytes per super-block.
BLOCK = {"q4_0": 32, "tq2_0": 256, "q8_0": 32, "iq4_nl": 32, "q4_k": 256}
ACT = {"q4_0": "q8_0", "tq2_0": "q8_K", "q8_0": "q8_0", "iq4_nl": "q8_0", "q4_k": "q8_K"}
QBYTES = {"q4_0": 16, "tq2_0": 64, "q8_0": 32, "iq4_nl": 16, "q4_k": 128}
NBYTES = {"q4_0": 18, "tq2_0": 66, "q8_0": 34, "iq4_nl": 18, "q4_k": 144}
QOFF = {"q4_0": 2, "tq2_0": 0, "q8_0": 2, "iq4_nl": 2}
SOFF = {"q4_0": 0, "tq2_0": 64, "q8_0": 0, "iq4_nl": 0}
Q4K_SCALE_BYTES = 20  # split scale plane per super-block: f16 d, f16 dmin, (sc_j, m_j) bytes for j = 0..7
# ggml's IQ4_NL levels (kvalues_iq4nl), the codebook of the format
IQ4_NL_LEVELS = np.array([-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113], dtype=np.int8)
TOL = 1e-5  # KURN's relative-error rule for the f32 GEMV output (src/komp/verify.py:28)

F32 = np.float32


# ---------------------------------------------------------------------------------------------------------------
# Rounding (patches/0001-language-extra-kurn.patch:84-101)
# ---------------------------------------------------------------------------------------------------------------


def round_half_away(x):
    """roundf(): nearest integer, halfway cases away from zero (patch:85-90). f32 in, f32 out, exact."""
    x = np.asarray(x, dtype=F32)
    a = np.abs(x)
    f = np.floor(a)
    r = np.where(a - f >= F32(0.5), f + F32(1), f).astype(F32)
    return np.where(x < 0, -r, r).astype(F32)


def round_half_even(x):
    """nearbyint() in round-to-nearest-even mode (patch:94-101). numpy's rint is exactly that."""
    return np.rint(np.asarray(x, dtype=F32)).astype(F32)


# ---------------------------------------------------------------------------------------------------------------
# Activation quantizers
# ---------------------------------------------------------------------------------------------------------------


def quant_q8_0(x):
    """f32 [M][K] -> (xq int8 [M][K], xd f32 [M][K/32]): ggml quantize_row_q8_0_ref as restated by
    ktl.q8_0_quantize (patch:104-114) and stored by kernel quant_q8_0 (src/komp/kernels.py:22-33):
    d = amax / 127 (f32 division), id = 1/d (0 when d == 0), q = roundf(x * id) from the UNROUNDED d,
    stored scale = f32(f16(d))."""
    x = np.ascontiguousarray(x, dtype=F32)
    m, k = x.shape
    if k % 32:
        raise ValueError("K must be a multiple of 32")
    b = x.reshape(m, k // 32, 32)
    amax = np.abs(b).max(axis=-1) if k else np.zeros((m, 0), F32)
    d = (amax / F32(127)).astype(F32)
    nz = d != 0
    idv = np.where(nz, (F32(1) / np.where(nz, d, F32(1))).astype(F32), F32(0)).astype(F32)
    q = round_half_away((b * idv[..., None]).astype(F32))
    return q.astype(np.int8).reshape(m, k), d.astype(np.float16).astype(F32)


def quant_q8_K(x):
    """f32 [M][K] -> (xq int8 [M][K], xd f32 [M][K/256], bsums int16 [M][K/256][16]): ggml quantize_row_q8_K_ref
    as restated by ktl.q8_K_quantize (patch:117-131) with the bsums host.q8_K_blocks adds (src/komp/host.py:43-52).
    mx = the signed value of largest magnitude, lowest index on ties; iscale = -127/mx; q = min(127, rint(iscale*x));
    d = 1/iscale; an all-zero block gives q = 0, d = 0."""
    x = np.ascontiguousarray(x, dtype=F32)
    m, k = x.shape
    if k % 256:
        raise ValueError("K must be a multiple of 256")
    nb = k // 256
    b = x.reshape(m, nb, 256)
    ax = np.abs(b)
    amax = ax.max(axis=-1) if k else np.zeros((m, 0), F32)
    first = np.argmax(ax == amax[..., None], axis=-1) if k else np.zeros((m, 0), np.int64)
    mx = np.take_along_axis(b, first[..., None], axis=-1)[..., 0] if k else np.zeros((m, 0), F32)
    nz = amax != 0
    iscale = (F32(-127) / np.where(nz, mx, F32(1))).astype(F32)
    q = np.minimum(round_half_even((iscale[..., None] * b).astype(F32)), F32(127))
    q = np.where(nz[..., None], q, F32(0))
    d = np.where(nz, (F32(1) / iscale).astype(F32), F32(0)).astype(F32)
    xq = q.astype(np.int8).reshape(m, k)
    bsums = xq.astype(np.int32).reshape(m, nb, 16, 16).sum(axis=-1).astype(np.int16)
    return xq, d, bsums


def quantize(fmt, x):
    """The activation quantizer of weight format `fmt` (src/komp/host.py:63-73): -> (xq, xd)."""
    if ACT[fmt] == "q8_0":
        return quant_q8_0(x)
    xq, xd, _ = quant_q8_K(x)
    return xq, xd


# ---------------------------------------------------------------------------------------------------------------
# Weight decode (patch:16-19, 39-63; verify.py:57-67)
# ---------------------------------------------------------------------------------------------------------------


def decode_q4_0(wq, k):
    """Q4_0 quant plane uint8 [n][k/2] -> int8 values [n][k] = nibble - 8 in natural order: byte i of a block
    holds value i (low nibble) and value i + 16 (high nibble) (patch:16-17, 39-55)."""
    wq = np.asarray(wq, dtype=np.uint8)
    n = wq.shape[0]
    blocks = wq[:, : k // 2].reshape(n, k // 32, 16)
    lo = (blocks & 15).astype(np.int8) - 8
    hi = (blocks >> 4).astype(np.int8) - 8
    return np.concatenate([lo, hi], axis=-1).reshape(n, k)


_TQ2_BYTE = np.array([(v // 128) * 32 + v % 32 for v in range(256)], dtype=np.int64)
_TQ2_SHIFT = np.array([2 * ((v % 128) // 32) for v in range(256)], dtype=np.uint8)


def decode_tq2_0(wq, k):
    """TQ2_0 quant plane uint8 [n][k/4] -> int8 values [n][k] = crumb - 1: value v of a block sits in byte
    (v/128)*32 + v%32 at bits 2*((v%128)/32) (patch:18-19, 58-63; verify.py:62-67). Crumb 3 decodes to +2."""
    wq = np.asarray(wq, dtype=np.uint8)
    n = wq.shape[0]
    blocks = wq[:, : k // 4].reshape(n, k // 256, 64)
    vals = (blocks[:, :, _TQ2_BYTE] >> _TQ2_SHIFT) & 3
    return (vals.astype(np.int8) - 1).reshape(n, k)


def decode_q8_0(wq, k):
    """Q8_0 quant plane uint8 [n][k] -> int8 values [n][k] (ggml block_q8_0.qs, natural order)."""
    wq = np.asarray(wq, dtype=np.uint8)
    return wq[:, :k].view(np.int8).copy()


def decode_iq4_nl(wq, k):
    """IQ4_NL quant plane uint8 [n][k/2] -> int8 values [n][k] = level[nibble], nibbles laid out as Q4_0's (byte i
    of a block: value i in the low nibble, value i + 16 in the high nibble)."""
    wq = np.asarray(wq, dtype=np.uint8)
    n = wq.shape[0]
    blocks = wq[:, : k // 2].reshape(n, k // 32, 16)
    return np.concatenate([IQ4_NL_LEVELS[blocks & 15], IQ4_NL_LEVELS[blocks >> 4]], axis=-1).reshape(n, k)


def decode(fmt, wq, k):
    return {"q4_0": decode_q4_0, "tq2_0": decode_tq2_0, "q8_0": decode_q8_0, "iq4_nl": decode_iq4_nl,
            "q4_k": decode_q4_k_quants}[fmt](wq, k)


# ---------------------------------------------------------------------------------------------------------------
# Q4_K (extension): ggml block_q4_K <-> this backend's split planes
# ---------------------------------------------------------------------------------------------------------------


def q4_k_scale_min(scales):
    """12 packed bytes per super-block [..][12] -> (sc, m) uint8 [..][8]: sub-blocks 0-3 take the low 6 bits of bytes
    0-3 (scales) and 4-7 (mins); sub-blocks 4-7 take the nibbles of bytes 8-11 as their low 4 bits and the top 2 bits
    of bytes 0-3 / 4-7 as their high 2 bits (ggml get_scale_min_k4)."""
    b = np.asarray(scales, dtype=np.uint8)
    d, m, md = b[..., 0:4], b[..., 4:8], b[..., 8:12]
    sc = np.concatenate([d & 0x3F, (md & 0x0F) | ((d >> 2) & 0x30)], axis=-1)
    mn = np.concatenate([m & 0x3F, (md >> 4) | ((m >> 2) & 0x30)], axis=-1)
    return sc.astype(np.uint8), mn.astype(np.uint8)


def q4_k_pack_scale_min(sc, mn):
    """Inverse of q4_k_scale_min: 6-bit (sc, m) [..][8] -> 12 packed bytes [..][12]."""
    sc = np.asarray(sc, dtype=np.uint8)
    mn = np.asarray(mn, dtype=np.uint8)
    d = (sc[..., :4] & 0x3F) | ((sc[..., 4:] >> 4) << 6)
    m = (mn[..., :4] & 0x3F) | ((mn[..., 4:] >> 4) << 6)
    md = (sc[..., 4:] & 0x0F) | ((mn[..., 4:] & 0x0F) << 4)
    return np.concatenate([d, m, md], axis=-1).astype(np.uint8)


def split_q4_k(W, n, k):
    """ggml Q4_K blocks (144 bytes: f16 d, f16 dmin, 12 scale bytes, 128 nibble bytes) -> (WQ uint8 [n][k/2],
    WS int16 [n][k/256 * 10]). WQ: per sub-block j of 32 values one 16-byte chunk laid out as a Q4_0 block (byte i:
    value i in the low nibble, value i + 16 in the high nibble); in the ggml block, byte i of 32-byte group g holds
    value i of sub-block 2g (low nibble) and of sub-block 2g + 1 (high nibble). WS: per super-block 20 bytes: d, dmin
    (f16 bits), then (sc_j, m_j) for j = 0..7."""
    nb = k // 256
    b = np.frombuffer(W, dtype=np.uint8).reshape(n, nb, 144)
    qs = b[:, :, 16:].reshape(n, nb, 4, 32)
    q = np.stack([qs & 0x0F, qs >> 4], axis=3).reshape(n, nb, 8, 32)  # sub-block 2g + h = nibble h of group g
    chunk = (q[..., :16] | (q[..., 16:] << 4)).astype(np.uint8)       # [n][nb][8][16]
    wq = np.ascontiguousarray(chunk.reshape(n, nb * 128))
    sc, mn = q4_k_scale_min(b[:, :, 4:16])
    rec = np.zeros((n, nb, Q4K_SCALE_BYTES), dtype=np.uint8)
    rec[:, :, 0:4] = b[:, :, 0:4]
    rec[:, :, 4::2] = sc
    rec[:, :, 5::2] = mn
    return wq, np.ascontiguousarray(rec.reshape(n, nb * Q4K_SCALE_BYTES)).view(np.int16)


def q4_k_parts(wq, ws, k):
    """Split planes -> (q uint8 [n][k] nibbles in value order, d f32 [n][nb], dmin f32 [n][nb], sc [n][nb][8],
    m [n][nb][8])."""
    wq = np.asarray(wq, dtype=np.uint8)
    n, nb = wq.shape[0], k // 256
    c = wq[:, : k // 2].reshape(n, k // 32, 16)
    q = np.concatenate([c & 15, c >> 4], axis=-1).reshape(n, k)
    rec = np.ascontiguousarray(np.asarray(ws, dtype=np.int16)).view(np.uint8).reshape(n, nb, Q4K_SCALE_BYTES)
    d = rec[:, :, 0:2].copy().view(np.float16)[..., 0].astype(F32)
    dmin = rec[:, :, 2:4].copy().view(np.float16)[..., 0].astype(F32)
    return q, d, dmin, rec[:, :, 4::2], rec[:, :, 5::2]


def decode_q4_k_quants(wq, k):
    """Q4_K split quant plane -> the nibbles (0..15) in value order, int8 [n][k] (the integer part of the dots)."""
    wq = np.asarray(wq, dtype=np.uint8)
    n = wq.shape[0]
    c = wq[:, : k // 2].reshape(n, k // 32, 16)
    return np.concatenate([c & 15, c >> 4], axis=-1).reshape(n, k).astype(np.int8)


def decode_q4_k(wq, ws, k):
    """Q4_K split planes -> f32 weight values [n][k] = (d * sc_j) * q - dmin * m_j in f32, gguf-py's dequantize
    arithmetic (so equal bit for bit)."""
    q, d, dmin, sc, mn = q4_k_parts(wq, ws, k)
    n, nb = d.shape
    ds = (d[..., None] * sc.astype(F32)).astype(F32)        # [n][nb][8]
    dm = (dmin[..., None] * mn.astype(F32)).astype(F32)
    v = (ds[..., None] * q.reshape(n, nb, 8, 32).astype(F32) - dm[..., None]).astype(F32)
    return v.reshape(n, k)


def q4_k_idots(wq, ws, xq, k):
    """Exact integer parts of the Q4_K dot per super-block, int64 [M][N][K/256] each: S = sum_j sc_j * sum_i q_i x_i
    (the block dot the kernels dump) and Mn = sum_j m_j * sum_i x_i (the min term)."""
    q, _, _, sc, mn = q4_k_parts(wq, ws, k)
    n, nb = sc.shape[0], k // 256
    xq = np.asarray(xq).astype(np.int64)
    m = xq.shape[0]
    if n == 0 or m == 0 or nb == 0:
        z = np.zeros((m, n, nb), np.int64)
        return z, z.copy()
    qv = q.reshape(n, nb * 8, 32).astype(np.float64).transpose(1, 0, 2)      # [sb][n][32]
    xv = xq.reshape(m, nb * 8, 32).astype(np.float64).transpose(1, 2, 0)     # [sb][32][m]
    sub = np.rint(np.matmul(qv, xv)).astype(np.int64).transpose(2, 1, 0)     # [m][n][sb]
    sub = sub.reshape(m, n, nb, 8)
    s = (sub * sc[None].astype(np.int64)).sum(-1)
    sx = xq.reshape(m, nb, 8, 32).sum(-1)                                   # [m][nb][8]
    mnt = (sx[:, None] * mn[None].astype(np.int64)).sum(-1)
    return s, mnt


def q4_k_reference(ws, xd, s, mnt, k):
    """f64 reference per output: sequential over super-blocks of dx * (d * S - dmin * Mn) -> f64 [M][N]."""
    n = np.asarray(ws).shape[0]
    _, d, dmin, _, _ = q4_k_parts(np.zeros((n, k // 2), np.uint8), ws, k)
    dx = np.asarray(xd, dtype=np.float32).astype(np.float64)
    m, _, nb = s.shape
    total = np.zeros((m, n), np.float64)
    for b in range(nb):
        total += dx[:, None, b] * (d[None, :, b].astype(np.float64) * s[:, :, b] -
                                   dmin[None, :, b].astype(np.float64) * mnt[:, :, b])
    return total


# ---------------------------------------------------------------------------------------------------------------
# GEMV: exact block dots, KURN's reference dot, relative error (verify.py:94-137)
# ---------------------------------------------------------------------------------------------------------------


def idots(fmt, wq, xq, k):
    """Exact block dots int64 [M][N][K/block] of the decoded weight values with the int8 activations
    (verify.exact_idots, src/komp/verify.py:94-100). Computed as f64 matmuls, exact since |dot| < 2^53."""
    blk = BLOCK[fmt]
    vals = decode(fmt, wq, k).astype(np.float64)
    n = vals.shape[0]
    xq = np.asarray(xq)
    m = xq.shape[0]
    nb = k // blk
    if nb == 0 or n == 0 or m == 0:
        return np.zeros((m, n, nb), dtype=np.int64)
    v = vals.reshape(n, nb, blk).transpose(1, 0, 2)                   # [nb][n][blk]
    q = xq.astype(np.float64).reshape(m, nb, blk).transpose(1, 2, 0)  # [nb][blk][m]
    out = np.matmul(v, q)                                             # [nb][n][m]
    return np.rint(out).astype(np.int64).transpose(2, 1, 0).copy()    # [m][n][nb]


def reference_dot(fmt, ws, xd, s):
    """KURN's kurn.formats.reference_dot for every output, from the int block dots s [M][N][nb]: per output a
    sequential Python-float (f64) sum over blocks of d_w * d_x * s (q4_0) or d_x * d_w * s (tq2_0), the exact
    float operations and order of verify.rebuild_reference (src/komp/verify.py:103-120). -> f64 [M][N]."""
    dw = np.asarray(ws, dtype=np.int16).view(np.float16).astype(np.float64)  # [n][nb]
    xd = np.asarray(xd, dtype=np.float32)
    # q8_0 blocks carry an f16 scale (the stored xd is already f16-exact); q8_K blocks carry the f32 scale
    dx = (xd.astype(np.float16) if ACT[fmt] == "q8_0" else xd).astype(np.float64)  # [m][nb]
    s = np.asarray(s)
    m, n, nb = s.shape
    total = np.zeros((m, n), dtype=np.float64)
    for b in range(nb):
        sb = s[:, :, b].astype(np.float64)
        if fmt != "tq2_0":
            total += (dw[None, :, b] * dx[:, None, b]) * sb
        else:
            total += (dx[:, None, b] * dw[None, :, b]) * sb
    return total


def gemv(fmt, wq, ws, xq, xd, k):
    """-> (reference f64 [M][N], exact block dots int64 [M][N][nb]) for the GEMV of src/komp/kernels.py:48-142
    (q4_k: the block dots are S = sum_j sc_j * dot_j; the reference adds the min term)."""
    if fmt == "q4_k":
        s, mnt = q4_k_idots(wq, ws, xq, k)
        return q4_k_reference(ws, xd, s, mnt, k), s
    s = idots(fmt, wq, xq, k)
    return reference_dot(fmt, ws, xd, s), s


def relerr(y, ref):
    """Normwise relative error max|y - ref| / max|ref| (KURN's `ref.relerr` is not in the reference archive; this
    is the definition used here, applied to every output of a problem at once)."""
    y = np.asarray(y, dtype=np.float64).reshape(-1)
    r = np.asarray(ref, dtype=np.float64).reshape(-1)
    if r.size == 0:
        return 0.0
    scale = np.max(np.abs(r))
    return float(np.max(np.abs(y - r)) / (scale if scale > 0 else 1.0))


def dp4a_ref(a, b, c):
    """PTX dp4a.s32.s32: c + sum of the products of the four signed bytes of a and b, int32 wraparound
    (src/komp/verify.py:37-41). Vectorized over int arrays."""
    a = np.asarray(a, dtype=np.int64) & 0xFFFFFFFF
    b = np.asarray(b, dtype=np.int64) & 0xFFFFFFFF
    r = np.asarray(c, dtype=np.int64).copy()
    for i in range(4):
        sa = ((a >> (8 * i)) & 0xFF).astype(np.int64)
        sb = ((b >> (8 * i)) & 0xFF).astype(np.int64)
        sa = np.where(sa >= 128, sa - 256, sa)
        sb = np.where(sb >= 128, sb - 256, sb)
        r = r + sa * sb
    return ((r + 2**31) % 2**32 - 2**31).astype(np.int64)


# ---------------------------------------------------------------------------------------------------------------
# Seeded synthetic inputs (the distributions BASELINE.json's configs name; KURN's generators are not available)
# ---------------------------------------------------------------------------------------------------------------


def weight_blocks(fmt, rng, n, k, extreme=False):
    """ggml weight blocks (bytes) for n rows of k values.

    random:  q4_0 quant bytes uniform 0..255, d = f16(|N(0, 0.02)|); tq2_0 crumbs uniform {0,1,2},
             d = f16(|N(0, 0.05)|); q8_0 values uniform -127..127, d = f16(|N(0, 0.002)|); iq4_nl nibbles uniform
             0..15, d = f16(|N(0, 0.002)|).
    extreme: q4_0 / iq4_nl nibbles only 0 or 15 (levels -127 and 113 for iq4_nl); tq2_0 crumbs 0, 2 and 3 (3 decodes to +2); q8_0 values -128, -127 and 127;
             scales include 0, f16 subnormals,
             the largest normal f16 below 2^8 and negative scales."""
    blk = BLOCK[fmt]
    nb = k // blk
    if fmt == "q4_k":
        return q4_k_blocks(rng, n, k, extreme)
    out = np.zeros((n, nb, NBYTES[fmt]), dtype=np.uint8)
    if fmt in ("q4_0", "iq4_nl"):
        if extreme:
            nib = rng.choice(np.array([0, 15], dtype=np.uint8), size=(n, nb, 32))
        else:
            nib = rng.integers(0, 16, size=(n, nb, 32), dtype=np.uint8)
        q = (nib[:, :, :16] | (nib[:, :, 16:] << 4)).astype(np.uint8)
        sd = 0.02 if fmt == "q4_0" else 0.002
    elif fmt == "q8_0":
        vals = rng.choice(np.array([-128, -127, 127], dtype=np.int8), size=(n, nb, 32)) if extreme else \
            rng.integers(-127, 128, size=(n, nb, 32)).astype(np.int8)
        q = vals.view(np.uint8)
        sd = 0.002
    else:
        crumbs = rng.choice(np.array([0, 2, 3], dtype=np.uint8), size=(n, nb, 256)) if extreme else \
            rng.integers(0, 3, size=(n, nb, 256), dtype=np.uint8)
        q = np.zeros((n, nb, 64), dtype=np.uint8)
        for v in range(256):
            q[:, :, _TQ2_BYTE[v]] |= (crumbs[:, :, v] << _TQ2_SHIFT[v]).astype(np.uint8)
        sd = 0.05
    d = np.abs(rng.normal(0.0, sd, size=(n, nb))).astype(np.float16)
    if extreme and n * nb:
        flat = d.reshape(-1)
        pick = rng.choice(flat.size, size=min(flat.size, 8), replace=False)
        specials = np.array([0.0, 6e-8, 3e-5, 255.9, -0.75, -1e-3, 1.0, 2.0 ** -14], dtype=np.float16)
        flat[pick] = specials[: pick.size]
    qoff, soff = QOFF[fmt], SOFF[fmt]
    out[:, :, qoff : qoff + QBYTES[fmt]] = q
    out[:, :, soff : soff + 2] = d.view(np.uint8).reshape(n, nb, 2)
    return out.tobytes()


def q4_k_blocks(rng, n, k, extreme=False):
    """ggml Q4_K blocks: nibbles uniform 0..15, 6-bit scales and mins uniform 0..63, d = f16(|N(0, 0.002)|), dmin =
    f16(|N(0, 0.004)|). extreme: nibbles 0 or 15, scales and mins 0 or 63, d and dmin including 0 and f16 extremes."""
    nb = k // 256
    out = np.zeros((n, nb, 144), dtype=np.uint8)
    if extreme:
        q = rng.choice(np.array([0, 15], dtype=np.uint8), size=(n, nb, 8, 32))
        sc = rng.choice(np.array([0, 63], dtype=np.uint8), size=(n, nb, 8))
        mn = rng.choice(np.array([0, 63], dtype=np.uint8), size=(n, nb, 8))
    else:
        q = rng.integers(0, 16, size=(n, nb, 8, 32), dtype=np.uint8)
        sc = rng.integers(0, 64, size=(n, nb, 8), dtype=np.uint8)
        mn = rng.integers(0, 64, size=(n, nb, 8), dtype=np.uint8)
    d = np.abs(rng.normal(0.0, 0.002, size=(n, nb))).astype(np.float16)
    dmin = np.abs(rng.normal(0.0, 0.004, size=(n, nb))).astype(np.float16)
    if extreme and n * nb:
        for arr in (d, dmin):
            flat = arr.reshape(-1)
            pick = rng.choice(flat.size, size=min(flat.size, 4), replace=False)
            flat[pick] = np.array([0.0, 6e-8, 65504.0, 2.0 ** -14], dtype=np.float16)[: pick.size]
    out[:, :, 0:2] = d.view(np.uint8).reshape(n, nb, 2)
    out[:, :, 2:4] = dmin.view(np.uint8).reshape(n, nb, 2)
    out[:, :, 4:16] = q4_k_pack_scale_min(sc, mn)
    g = q.reshape(n, nb, 4, 2, 32)
    out[:, :, 16:] = (g[:, :, :, 0] | (g[:, :, :, 1] << 4)).reshape(n, nb, 128)
    return out.tobytes()


def activations(rng, m, k, extreme=False):
    """f32 [m][k]: N(0, 1). extreme: plus 5% exact zeros, 1% +-1e4 outliers, an all-zero 256-block, a block at
    exact rounding half-points (amax 127 so q8_0's id is 1.0, max -127 so q8_K's iscale is 1.0) and a block whose
    largest magnitude is tied between signs."""
    x = rng.standard_normal((m, k)).astype(F32)
    if extreme and k:
        x[rng.random((m, k)) < 0.05] = 0.0
        out = rng.random((m, k)) < 0.01
        x[out] = np.where(rng.random(out.sum()) < 0.5, -1e4, 1e4).astype(F32)
        blocks = k // 32
        for row in range(m):
            if k >= 256:
                z = rng.integers(0, k // 256)
                x[row, z * 256 : (z + 1) * 256] = 0.0
            if blocks >= 2:
                b = rng.integers(0, blocks)
                half = (rng.integers(-126, 126, size=32) + 0.5).astype(F32)
                half[rng.integers(0, 32)] = -127.0
                x[row, b * 32 : (b + 1) * 32] = half
                b2 = (b + 1) % blocks
                tie = rng.standard_normal(32).astype(F32)
                i, j = rng.choice(32, size=2, replace=False)
                tie[min(i, j)], tie[max(i, j)] = 7.25, -7.25
                x[row, b2 * 32 : (b2 + 1) * 32] = tie
    return x


def quant_config_input(seed=0, m=4, k=14336):
    """f32 [4][14336], N(0,1) with 5% exact zeros, 1% +-1e4 outliers, one all-zero 32-block, one
    all-zero 256-block, and blocks of exact rounding half-points for both quantizers."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((m, k)).astype(F32)
    x[rng.random((m, k)) < 0.05] = 0.0
    out = rng.random((m, k)) < 0.01
    x[out] = np.where(rng.random(out.sum()) < 0.5, -1e4, 1e4).astype(F32)
    x[0, 32:64] = 0.0                       # all-zero q8_0 block (its 256-block is not all zero)
    x[1, 512:768] = 0.0                     # all-zero q8_K block
    half = (np.arange(-16, 16) + 0.5).astype(F32)
    half[5] = 127.0                         # q8_0: amax 127 -> d = 1, id = 1, q = roundf(k + 0.5)
    x[2, 64:96] = half
    blk = (rng.integers(-120, 120, size=256) + 0.5).astype(F32)
    blk[17] = -127.0                        # q8_K: max is -127 -> iscale = 1, q = rint(k + 0.5)
    x[3, 1024:1280] = blk
    tie = rng.standard_normal(256).astype(F32)
    tie[40], tie[200] = -9.5, 9.5           # q8_K tie on |x|: the first (negative) one wins
    x[2, 2048:2304] = tie
    return x


def problem(fmt, n, k, m, seed=0, extreme=False):
    """(ggml weight bytes, f32 activations [m][k]) for one GEMV problem."""
    rng = np.random.default_rng(seed)
    W = weight_blocks(fmt, rng, n, k, extreme)
    x = activations(rng, m, k, extreme)
    return W, x


def split(fmt, W, n, k):
    """ggml blocks -> (WQ uint8 [n][qbytes*k/blk], WS int16 [n][k/blk]) (src/komp/host.py:16-22); q4_k: split_q4_k."""
    if fmt == "q4_k":
        return split_q4_k(W, n, k)
    blk = BLOCK[fmt]
    b = np.frombuffer(W, dtype=np.uint8).reshape(n, k // blk, NBYTES[fmt])
    qoff, soff = QOFF[fmt], SOFF[fmt]
    wq = np.ascontiguousarray(b[:, :, qoff : qoff + QBYTES[fmt]]).reshape(n, -1)
    ws = np.ascontiguousarray(b[:, :, soff : soff + 2]).view(np.int16).reshape(n, k // blk)
    return wq, ws


def random_split(fmt, rng, n, k):
    """Split planes directly (fast path for large synthetic layers): same distributions as weight_blocks."""
    blk = BLOCK[fmt]
    nb = k // blk
    if fmt == "q4_k":
        return split_q4_k(q4_k_blocks(rng, n, k), n, k)
    if fmt in ("q4_0", "iq4_nl"):
        wq = rng.integers(0, 256, size=(n, k // 2), dtype=np.uint8)
        d = np.abs(rng.normal(0.0, 0.02 if fmt == "q4_0" else 0.002, size=(n, nb))).astype(np.float16)
    elif fmt == "q8_0":
        wq = rng.integers(-127, 128, size=(n, k), dtype=np.int8).view(np.uint8)
        d = np.abs(rng.normal(0.0, 0.002, size=(n, nb))).astype(np.float16)
    else:
        # crumbs uniform in {0,1,2}: draw each byte's 4 crumbs from base-3 digits of a uniform 0..80
        t = rng.integers(0, 81, size=(n, k // 4), dtype=np.uint8)
        c0, c1, c2, c3 = t % 3, (t // 3) % 3, (t // 9) % 3, (t // 27) % 3
        wq = (c0 | (c1 << 2) | (c2 << 4) | (c3 << 6)).astype(np.uint8)
        d = np.abs(rng.normal(0.0, 0.05, size=(n, nb))).astype(np.float16)
    return wq, d.view(np.int16)

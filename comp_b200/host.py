"""Host side of the B200 backend: KURN split layouts from ggml blocks, and the CUDA launches.

Drop-in for COMP's `komp.host` (src/komp/host.py): same names, argument meanings and return values. `quantize` and
`gemv` launch this package's sm_100a kernels through the C-ABI library (include/comp_b200.h); they take CUDA
tensors only and raise on anything else -- there is no CPU path.

Tuning arguments of the Triton kernels (`bb`, `block_n`, `nb`, `num_warps`) are accepted and ignored: the CUDA
schedule is planned from (N, K, M) by the library, and results do not depend on them. `mode` selects the variant:
0 = byte-wise unpack, 1 or 2 = packed-word dp4a; all variants give identical int32 block dots and identical Y.
"""

import contextlib

import numpy as np
import torch

from . import _lib

# weights: block values, block bytes, quant offset/bytes in the ggml block, scale offset, int16s of the scale plane
# per block, activation format (q4_0 and tq2_0: the same table as src/komp/host.py:9-12; q8_0, iq4_nl and q4_k are
# extensions beyond the reference: ggml block_q8_0 / block_iq4_nl weights against q8_0 activations, block_q4_K
# super-blocks against q8_K activations, split by split_q4_k into this backend's own planes)
FORMATS = {
    "q4_0": dict(block=32, nbytes=18, qoff=2, qbytes=16, soff=0, sshorts=1, act="q8_0"),
    "tq2_0": dict(block=256, nbytes=66, qoff=0, qbytes=64, soff=64, sshorts=1, act="q8_K"),
    "q8_0": dict(block=32, nbytes=34, qoff=2, qbytes=32, soff=0, sshorts=1, act="q8_0"),
    "iq4_nl": dict(block=32, nbytes=18, qoff=2, qbytes=16, soff=0, sshorts=1, act="q8_0"),
    "q4_k": dict(block=256, nbytes=144, qoff=16, qbytes=128, soff=0, sshorts=10, act="q8_K"),
}
MODES = {"bytes": 0, "dp4a": 2}  # src/komp/host.py:13
ACT_BLOCK = {"q8_0": 32, "q8_K": 256}
FMT_ID = {"q4_0": 0, "tq2_0": 1, "q8_0": 2, "iq4_nl": 3, "q4_k": 4}
GEMV_ENTRY = {"q4_0": "b2q_gemv_q4_0", "tq2_0": "b2q_gemv_tq2_0", "q8_0": "b2q_gemv_q8_0",
              "iq4_nl": "b2q_gemv_iq4_nl", "q4_k": "b2q_gemv_q4_k"}


def _fmt(fmt):
    if fmt not in FORMATS:
        raise ValueError(f"unknown weight format {fmt!r}: expected one of {sorted(FORMATS)}")
    return FORMATS[fmt]


# ---------------------------------------------------------------------------------------------------------------
# Layout helpers (numpy, host memory). Same semantics as src/komp/host.py:16-56.
# ---------------------------------------------------------------------------------------------------------------


def split(fmt, W, n, k):
    """ggml blocks (bytes, n rows of k values) -> (WQ uint8 [n][quant bytes per row], WS int16 [n][k/block])
    (q4_k: WS int16 [n][k/256 * 10], see split_q4_k)."""
    f = _fmt(fmt)
    if k % f["block"]:
        raise ValueError(f"k={k} is not a multiple of the {fmt} block ({f['block']})")
    nb = k // f["block"]
    raw = np.frombuffer(W, dtype=np.uint8)
    if raw.size != n * nb * f["nbytes"]:
        raise ValueError(f"{raw.size} bytes do not hold {n} x {nb} {fmt} blocks of {f['nbytes']} bytes")
    blocks = raw.reshape(n, nb, f["nbytes"])
    if fmt == "q4_k":
        return split_q4_k(blocks)
    wq = blocks[:, :, f["qoff"] : f["qoff"] + f["qbytes"]].reshape(n, nb * f["qbytes"]).copy()
    ws = blocks[:, :, f["soff"] : f["soff"] + 2].copy().view(np.int16).reshape(n, nb)
    return wq, ws


def split_q4_k(blocks):
    """ggml block_q4_K uint8 [n][nb][144] (f16 d, f16 dmin, 12 bytes of packed 6-bit scales and mins, 128 nibble
    bytes) -> this backend's planes (WQ uint8 [n][nb*128], WS int16 [n][nb*10]):
      WQ: per 32-value sub-block j one 16-byte chunk laid out like a Q4_0 block, byte i holding value i (low nibble)
          and value i + 16 (high nibble); in the ggml block byte i of the 32-byte group g holds value i of sub-block
          2g (low nibble) and of sub-block 2g + 1 (high nibble);
      WS: per super-block 20 bytes: d, dmin (f16 bits), then the unpacked bytes sc_0, m_0, ..., sc_7, m_7 (ggml's
          6-bit fields: j < 4 in the low 6 bits of scale bytes j (sc) and 4 + j (m); j >= 4 in the nibbles of byte
          8 + (j - 4) for the low 4 bits and the top 2 bits of bytes j - 4 (sc) and j (m))."""
    n, nb = blocks.shape[:2]
    qs = blocks[:, :, 16:].reshape(n, nb, 4, 32)
    sub = np.stack([qs & 0x0F, qs >> 4], axis=3).reshape(n, nb, 8, 32)  # sub-block 2g + h: nibble h of group g
    wq = (sub[..., :16] | (sub[..., 16:] << 4)).astype(np.uint8).reshape(n, nb * 128)
    p = blocks[:, :, 4:16]
    lo, mid, top = p[..., 0:4], p[..., 4:8], p[..., 8:12]
    sc = np.concatenate([lo & 0x3F, (top & 0x0F) | ((lo >> 2) & 0x30)], axis=-1)
    mn = np.concatenate([mid & 0x3F, (top >> 4) | ((mid >> 2) & 0x30)], axis=-1)
    rec = np.empty((n, nb, 20), dtype=np.uint8)
    rec[:, :, 0:4] = blocks[:, :, 0:4]
    rec[:, :, 4::2] = sc
    rec[:, :, 5::2] = mn
    return np.ascontiguousarray(wq), np.ascontiguousarray(rec.reshape(n, nb * 20)).view(np.int16)


def split_q4_0(W, n, k):
    return split("q4_0", W, n, k)


def split_device(fmt, blocks, n, k, ldwq=None):
    """split() on the GPU: ggml blocks as a CUDA uint8 tensor (n rows of k values, the bytes as stored in a GGUF
    file) -> (WQ uint8 [n][ldwq], WS int16 [n][k/block]) CUDA tensors, byte-identical to split(). ldwq defaults to the
    quant bytes per row (a multiple of 16 for every K the GEMVs take)."""
    f = _fmt(fmt)
    if k % f["block"]:
        raise ValueError(f"k={k} is not a multiple of the {fmt} block ({f['block']})")
    dev = _need_cuda("split_device", blocks)
    nb = k // f["block"]
    if blocks.dtype != torch.uint8 or blocks.numel() != n * nb * f["nbytes"]:
        raise ValueError(f"split_device: expected {n * nb * f['nbytes']} uint8 bytes of {fmt} blocks, got "
                         f"{blocks.dtype} x {blocks.numel()}")
    blocks = blocks.reshape(-1)
    if not blocks.is_contiguous() or blocks.data_ptr() % 16:
        blocks = blocks.clone()
    qb = nb * f["qbytes"]
    ldwq = qb if ldwq is None else ldwq
    wq = torch.empty((n, ldwq), dtype=torch.uint8, device=dev)
    ws = torch.empty((n, nb * f["sshorts"]), dtype=torch.int16, device=dev)
    with _on(dev):
        _lib.call("b2q_split_blocks", FMT_ID[fmt], blocks.data_ptr(), n, k, wq.data_ptr(), ldwq, ws.data_ptr(),
                  _stream(dev))
    return (wq if ldwq == qb else wq[:, :qb]), ws


def tq2_0_qplane(W, nblk):
    """ggml tq2_0 blocks -> quant plane uint8 [nblk][64] (the f16 scale at byte 64 goes to the scale plane)."""
    return np.frombuffer(W, dtype=np.uint8).reshape(nblk, 66)[:, :64].copy()


def q8_0_blocks(xq, xd):
    """q8_0 split planes (numpy) -> ggml q8_0 blocks (bytes): f16 d, then 32 int8 per block."""
    xq, xd = np.asarray(xq), np.asarray(xd)
    m, k = xq.shape
    nb = k // 32
    out = np.empty((m, nb, 34), dtype=np.uint8)
    out[:, :, 0:2] = np.asarray(xd, dtype=np.float32).astype(np.float16).view(np.uint8).reshape(m, nb, 2)
    out[:, :, 2:34] = xq.astype(np.int8).view(np.uint8).reshape(m, nb, 32)
    return out.tobytes()


def q8_K_bsums(xq):
    """int16 sums of each run of 16 quants: [m][k/256][16] (ggml block_q8_K.bsums)."""
    xq = np.asarray(xq)
    m, k = xq.shape
    return xq.astype(np.int32).reshape(m, k // 256, 16, 16).sum(axis=-1).astype(np.int16)


def q8_K_blocks(xq, xd):
    """q8_K split planes (numpy) -> ggml q8_K blocks (bytes): f32 d, 256 int8, 16 int16 bsums."""
    xq, xd = np.asarray(xq), np.asarray(xd)
    m, k = xq.shape
    nb = k // 256
    out = np.empty((m, nb, 292), dtype=np.uint8)
    out[:, :, 0:4] = np.asarray(xd, dtype=np.float32).view(np.uint8).reshape(m, nb, 4)
    out[:, :, 4:260] = xq.astype(np.int8).view(np.uint8).reshape(m, nb, 256)
    out[:, :, 260:292] = q8_K_bsums(xq).view(np.uint8).reshape(m, nb, 32)
    return out.tobytes()


def act_blocks(fmt, xq, xd):
    return (q8_0_blocks if _fmt(fmt)["act"] == "q8_0" else q8_K_blocks)(xq, xd)


def device():
    """'cuda' when a GPU is visible. Unlike the reference there is no CPU execution: compute calls need CUDA."""
    return "cuda" if torch.cuda.is_available() else "cpu"


# ---------------------------------------------------------------------------------------------------------------
# Launches
# ---------------------------------------------------------------------------------------------------------------


def _need_cuda(name, *tensors):
    for t in tensors:
        if not isinstance(t, torch.Tensor) or t.device.type != "cuda":
            raise RuntimeError(f"comp_b200.{name}: tensors must be CUDA tensors (this backend has no CPU path)")
    dev = tensors[0].device
    for t in tensors[1:]:
        if t.device != dev:
            raise RuntimeError(f"comp_b200.{name}: tensors on different devices ({dev} and {t.device})")
    return dev


def _check(t, name, dtype, shape):
    if t.dtype != dtype:
        raise TypeError(f"{name}: dtype {t.dtype}, expected {dtype}")
    if tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name}: shape {tuple(t.shape)}, expected {tuple(shape)}")


def _rows_aligned(t):
    """Returns a tensor with unit column stride and a 16-byte aligned base (copies only when needed)."""
    if t.stride(-1) != 1 or t.data_ptr() % 16 or (t.dim() == 2 and t.stride(0) % 4):
        t = t.clone(memory_format=torch.contiguous_format)
    return t


def _stream(dev):
    return torch.cuda.current_stream(dev).cuda_stream


def _on(dev):
    """Context making `dev` the current device (a no-op when it already is: the common single-GPU case)."""
    return contextlib.nullcontext() if dev.index == torch.cuda.current_device() else torch.cuda.device(dev)


def quantize(fmt, x, bb=4):
    """f32 [M][K] CUDA tensor -> (XQ int8 [M][K], XD f32 [M][K/block]) with the q8_0 / q8_K quantizer of `fmt`'s
    activation format (src/komp/host.py:63-73). Bytes equal ggml's reference quantizers."""
    del bb  # Triton block-count hint; the CUDA kernel has its own schedule
    act = _fmt(fmt)["act"]
    dev = _need_cuda("quantize", x)
    if x.dtype != torch.float32 or x.dim() != 2:
        raise TypeError(f"quantize: x must be a 2-D float32 tensor, got {x.dtype} {tuple(x.shape)}")
    m, k = x.shape
    blk = ACT_BLOCK[act]
    if k % blk:
        raise ValueError(f"quantize: K={k} is not a multiple of the {act} block ({blk})")
    x = _rows_aligned(x)
    xq = torch.empty((m, k), dtype=torch.int8, device=dev)
    xd = torch.empty((m, k // blk), dtype=torch.float32, device=dev)
    with _on(dev):
        if act == "q8_0":
            _lib.call("b2q_quant_q8_0", x.data_ptr(), x.stride(0), xq.data_ptr(), xd.data_ptr(), m, k, _stream(dev))
        else:
            _lib.call("b2q_quant_q8_K", x.data_ptr(), x.stride(0), xq.data_ptr(), xd.data_ptr(), None, m, k,
                      _stream(dev))
    return xq, xd


def quantize_q8_K_bsums(x):
    """q8_K of f32 [M][K] -> (XQ, XD, bsums int16 [M][K/256][16]): the full ggml block_q8_K content, on the GPU."""
    dev = _need_cuda("quantize_q8_K_bsums", x)
    m, k = x.shape
    if k % 256:
        raise ValueError(f"K={k} is not a multiple of 256")
    x = _rows_aligned(x)
    xq = torch.empty((m, k), dtype=torch.int8, device=dev)
    xd = torch.empty((m, k // 256), dtype=torch.float32, device=dev)
    bs = torch.empty((m, k // 256, 16), dtype=torch.int16, device=dev)
    with _on(dev):
        _lib.call("b2q_quant_q8_K", x.data_ptr(), x.stride(0), xq.data_ptr(), xd.data_ptr(), bs.data_ptr(), m, k,
                  _stream(dev))
    return xq, xd, bs


def _check_weights(fmt, wq, ws, n, k):
    f = _fmt(fmt)
    if k % f["block"]:
        raise ValueError(f"gemv: k={k} is not a multiple of the {fmt} block ({f['block']})")
    qbytes = k // f["block"] * f["qbytes"]
    if wq.dtype != torch.uint8 or wq.dim() != 2 or wq.shape[0] != n or wq.shape[1] < qbytes or \
            (wq.numel() and wq.stride(1) != 1):
        raise ValueError(f"gemv: wq must be uint8 [{n}][>= {qbytes}] with unit column stride, got {wq.dtype} "
                         f"{tuple(wq.shape)}")
    _check(ws, "ws", torch.int16, (n, k // f["block"] * f["sshorts"]))
    if ws.numel() and not ws.is_contiguous():
        raise ValueError("gemv: ws must be contiguous")


def gemv(fmt, wq, ws, xq, xd, n, k, block_n=32, nb=4, mode=0, num_warps=4, store_s=False):
    """-> (Y f32 [M][N], S int32 [M][N][blocks] or None) (src/komp/host.py:76-85).

    mode: 0 bytes, 1 dp4a (the reference's interpreter fallback), 2 dp4a; all give identical results."""
    del block_n, nb, num_warps  # Triton schedule hints; the CUDA schedule is planned by the library
    f = _fmt(fmt)
    if mode not in (0, 1, 2):
        raise ValueError(f"gemv: mode {mode} not in (0, 1, 2)")
    dev = _need_cuda("gemv", wq, ws, xq, xd)
    _check_weights(fmt, wq, ws, n, k)
    m = xq.shape[0]
    _check(xq, "xq", torch.int8, (m, k))
    _check(xd, "xd", torch.float32, (m, k // f["block"]))
    xq = _rows_aligned(xq.contiguous())
    xd = xd.contiguous()
    y = torch.empty((m, n), dtype=torch.float32, device=dev)
    s = torch.empty((m, n, k // f["block"]), dtype=torch.int32, device=dev) if store_s else None
    name = GEMV_ENTRY[fmt]
    with _on(dev):
        _lib.call(name, wq.data_ptr(), wq.stride(0), ws.data_ptr(), xq.data_ptr(), xd.data_ptr(), y.data_ptr(),
                  s.data_ptr() if store_s else None, n, k, m, mode, _stream(dev))
    return y, s


def workspace_size(fmt, n, k, m):
    """Bytes of split-K workspace quant_gemv uses for this shape (0: the layer is not split)."""
    return int(_lib.load().b2q_workspace_size(FMT_ID[fmt], n, k, m))


def quant_gemv(fmt, wq, ws, x, n, k, return_act=False, split=True, workspace=None, out=None):
    """Fused quantize + gemv: f32 x [M][K] -> Y f32 [M][N] (and (XQ, XD) when return_act).

    out: optional preallocated contiguous f32 [M][N] CUDA tensor for Y (returned), e.g. to avoid an allocation per
    decode step.

    split=False: Y equals gemv(fmt, wq, ws, *quantize(fmt, x), n, k) exactly (same bytes, same schedule, same f32
    order); one launch up to 4 columns, with more the quantizer and the tensor-core GEMM. split=True (default): with a
    workspace (allocated here unless given; a CUDA byte tensor of at least workspace_size(...) bytes) tall-K layers
    may run the split-K schedule, and from 5 columns (TQ2_0: 3) layers that fill the GPU the fused tensor-core GEMM;
    Y then differs from the split=False result only by f32 rounding of the sum order, and is deterministic."""
    f = _fmt(fmt)
    dev = _need_cuda("quant_gemv", wq, ws, x)
    _check_weights(fmt, wq, ws, n, k)
    if x.dtype != torch.float32 or x.dim() != 2 or x.shape[1] != k:
        raise ValueError(f"quant_gemv: x must be float32 [M][{k}], got {x.dtype} {tuple(x.shape)}")
    m = x.shape[0]
    x = _rows_aligned(x)
    if out is None:
        y = torch.empty((m, n), dtype=torch.float32, device=dev)
    else:
        if out.dtype != torch.float32 or tuple(out.shape) != (m, n) or out.device != dev or not out.is_contiguous():
            raise ValueError(f"quant_gemv: out must be a contiguous float32 [{m}][{n}] tensor on {dev}")
        y = out
    xq = xd = None
    if return_act:
        xq = torch.empty((m, k), dtype=torch.int8, device=dev)
        xd = torch.empty((m, k // f["block"]), dtype=torch.float32, device=dev)
    # the workspace enables split-K (split=True, at most 4 columns) or, with more columns, the scratch for the
    # quantized activations of the tensor-core GEMM
    wsb = workspace_size(fmt, n, k, m) if (split or m > 4) else 0
    if wsb and workspace is None:
        workspace = torch.empty(wsb, dtype=torch.uint8, device=dev)
    with _on(dev):
        _lib.call("b2q_quant_gemv_ws", FMT_ID[fmt], wq.data_ptr(), wq.stride(0), ws.data_ptr(), x.data_ptr(),
                  x.stride(0), xq.data_ptr() if return_act else None, xd.data_ptr() if return_act else None,
                  y.data_ptr(), n, k, m, workspace.data_ptr() if wsb else None,
                  workspace.numel() * workspace.element_size() if wsb else 0, _stream(dev))
    return (y, xq, xd) if return_act else y


def pinned_workspace_size(fmt, n, k, m):
    """Bytes of device workspace quant_gemv_pinned needs for this shape (staged activations + GEMV workspace)."""
    return int(_lib.load().b2q_pinned_workspace_size(FMT_ID[fmt], n, k, m))


def quant_gemv_pinned(fmt, wq, ws, x, n, k, out, workspace=None):
    """quant_gemv with the activations and the output in page-locked host memory.

    x: f32 [M][K] CPU tensor in pinned memory (x.pin_memory()); out: contiguous f32 [M][N] pinned CPU tensor that
    receives Y. The copy of x to the GPU and the store of Y to `out` are made by the kernels through the buffers'
    device mappings (no memcpy), on the current stream of the weights' device, asynchronously: synchronize that
    stream before reading `out`. Y equals quant_gemv(fmt, wq, ws, x.cuda(), n, k) bit for bit. workspace: optional CUDA
    byte tensor of at least pinned_workspace_size(fmt, n, k, M) bytes, 256-byte aligned (allocated here when None).
    Returns `out`."""
    _fmt(fmt)
    dev = _need_cuda("quant_gemv_pinned", wq, ws)
    _check_weights(fmt, wq, ws, n, k)
    for t, name in ((x, "x"), (out, "out")):
        if not isinstance(t, torch.Tensor) or t.device.type != "cpu" or not t.is_pinned():
            raise ValueError(f"quant_gemv_pinned: {name} must be a pinned CPU tensor (tensor.pin_memory())")
    if x.dtype != torch.float32 or x.dim() != 2 or x.shape[1] != k or x.stride(1) != 1:
        raise ValueError(f"quant_gemv_pinned: x must be float32 [M][{k}] with unit column stride, got {x.dtype} "
                         f"{tuple(x.shape)}")
    m = x.shape[0]
    if out.dtype != torch.float32 or tuple(out.shape) != (m, n) or not out.is_contiguous():
        raise ValueError(f"quant_gemv_pinned: out must be a contiguous float32 [{m}][{n}] pinned CPU tensor")
    need = pinned_workspace_size(fmt, n, k, m)
    if workspace is None:
        workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=dev)
    with _on(dev):
        _lib.call("b2q_quant_gemv_pinned", FMT_ID[fmt], wq.data_ptr(), wq.stride(0), ws.data_ptr(), x.data_ptr(),
                  x.stride(0), out.data_ptr(), n, k, m, workspace.data_ptr(),
                  workspace.numel() * workspace.element_size(), _stream(dev))
    return out

"""Parity of the CUDA path (through the C-ABI, via comp_b200.host) with the reference and the oracle.

Bars: quantizer bytes and every int32 block dot bit-exact; f32 Y within KURN's relative-error rule (1e-5) of the
exact reference dot, which is itself rebuilt bit-identically from our int32 dots. Mirrors the reference's checks in
src/komp/verify.py (check_dp4a, check_decode, check_gemv) on the reference's own recorded outputs.
"""

import numpy as np
import pytest
import torch

from comp_b200 import _lib, host
from oracle import native, ref

from .conftest import golden_case_ids

pytestmark = pytest.mark.gpu

TOL = 1e-5  # KURN's rule (src/komp/verify.py:28)


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _same_f32(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


# ---------------------------------------------------------------------------------------------------------------
# probes (verify.check_dp4a / check_decode)
# ---------------------------------------------------------------------------------------------------------------


def test_dp4a_probe_matches_reference(cuda, golden):
    a, b, c = (_t(golden[f"dp4a/{k}"], cuda) for k in "abc")
    out = torch.empty_like(a)
    _lib.call("b2q_probe_dp4a", a.data_ptr(), b.data_ptr(), c.data_ptr(), out.data_ptr(), a.numel(),
              torch.cuda.current_stream().cuda_stream)
    assert np.array_equal(out.cpu().numpy(), golden["dp4a/out"])


def test_decode_probes_match_reference(cuda, golden):
    for fmt, vals in (("q4_0", 32), ("tq2_0", 256)):
        wq = _t(golden[f"decode/{fmt}/wq"], cuda)
        out = torch.empty((wq.shape[0], vals), dtype=torch.int32, device=cuda)
        _lib.call(f"b2q_decode_{fmt}", wq.data_ptr(), out.data_ptr(), wq.shape[0],
                  torch.cuda.current_stream().cuda_stream)
        assert np.array_equal(out.cpu().numpy(), golden[f"decode/{fmt}/out"]), fmt


# ---------------------------------------------------------------------------------------------------------------
# quantizers
# ---------------------------------------------------------------------------------------------------------------


@pytest.mark.parametrize("fmt", ["q4_0", "tq2_0"])
def test_quantizer_bytes_match_reference(cuda, golden, fmt):
    x = golden["quant/x"]
    xq, xd = host.quantize(fmt, _t(x, cuda))
    act = ref.ACT[fmt]
    assert np.array_equal(xq.cpu().numpy(), golden[f"quant/{act}/xq"])
    assert _same_f32(xd.cpu().numpy(), golden[f"quant/{act}/xd"])
    # ggml block bytes, as verify.check_gemv compares them (src/komp/verify.py:128-130)
    oq, od = ref.quantize(fmt, x)
    assert host.act_blocks(fmt, xq.cpu().numpy(), xd.cpu().numpy()) == host.act_blocks(fmt, oq, od)


def test_q8_K_bsums_match_oracle(cuda, golden):
    x = golden["quant/x"]
    xq, xd, bs = host.quantize_q8_K_bsums(_t(x, cuda))
    oq, od, obs = ref.quant_q8_K(x)
    assert np.array_equal(xq.cpu().numpy(), oq) and _same_f32(xd.cpu().numpy(), od)
    assert np.array_equal(bs.cpu().numpy(), obs)


def test_quantizer_row_stride_and_tails(cuda):
    rng = np.random.default_rng(5)
    for m, k, ldx in ((3, 96, 100), (1, 32, 32), (5, 512, 520), (2, 0, 4)):
        big = rng.standard_normal((m, ldx)).astype(np.float32) * 3
        xt = _t(big, cuda)[:, :k]
        for fmt in ("q4_0", "tq2_0"):
            if k % ref.BLOCK[fmt] and fmt == "tq2_0":
                continue
            xq, xd = host.quantize(fmt, xt)
            oq, od = ref.quantize(fmt, big[:, :k])
            assert np.array_equal(xq.cpu().numpy(), oq), (fmt, m, k)
            assert _same_f32(xd.cpu().numpy(), od), (fmt, m, k)


# ---------------------------------------------------------------------------------------------------------------
# GEMVs on the reference's recorded problems (verify.PROBLEMS + config-0/1 row slices, random and extreme)
# ---------------------------------------------------------------------------------------------------------------


@pytest.mark.parametrize("cid", golden_case_ids())
def test_gemv_matches_reference(cuda, golden, cid):
    c = next(c for c in golden.cases() if c["id"] == cid)
    g = golden.case(cid)
    fmt, n, k, m = c["fmt"], c["n"], c["k"], c["m"]
    wq, ws = host.split(fmt, g["W"].tobytes(), n, k)
    xq, xd = host.quantize(fmt, _t(g["x"], cuda))
    assert np.array_equal(xq.cpu().numpy(), g["xq"]) and _same_f32(xd.cpu().numpy(), g["xd"])
    r, _ = ref.gemv(fmt, wq, ws, g["xq"], g["xd"], k)
    ys = []
    for mode in (0, 1, 2):
        y, s = host.gemv(fmt, _t(wq, cuda), _t(ws, cuda), xq, xd, n, k, mode=mode, store_s=True)
        s = s.cpu().numpy()
        assert np.array_equal(s, g["s0"]), f"int32 block dots differ (mode {mode})"
        # KURN's reference dot rebuilt from our dots, same float ops and order, is bit-identical
        assert np.array_equal(ref.reference_dot(fmt, ws, g["xd"], s).view(np.uint64), r.view(np.uint64))
        y = y.cpu().numpy()
        assert ref.relerr(y, r) <= TOL, f"mode {mode}: relerr {ref.relerr(y, r):.2e}"
        assert ref.relerr(g["y0"], r) <= TOL  # the reference's own f32 output, for scale
        ys.append(y)
    # every variant gives the same f32 Y, bit for bit (schedule-independent summation order)
    assert _same_f32(ys[0], ys[1]) and _same_f32(ys[1], ys[2])
    # without store_s the same Y
    y, s = host.gemv(fmt, _t(wq, cuda), _t(ws, cuda), xq, xd, n, k, mode=2)
    assert s is None and _same_f32(y.cpu().numpy(), ys[2])
    # fused quantizer prologue: same activations, same Y
    yf, fq, fd = host.quant_gemv(fmt, _t(wq, cuda), _t(ws, cuda), _t(g["x"], cuda), n, k, return_act=True,
                                 split=False)
    assert np.array_equal(fq.cpu().numpy(), g["xq"]) and _same_f32(fd.cpu().numpy(), g["xd"])
    assert _same_f32(yf.cpu().numpy(), ys[2])


# ---------------------------------------------------------------------------------------------------------------
# BASELINE-size problems against the oracle
# ---------------------------------------------------------------------------------------------------------------


def _layer(fmt, n, k, m, seed, dev):
    rng = np.random.default_rng(seed)
    wq, ws = ref.random_split(fmt, rng, n, k)
    x = rng.standard_normal((m, k)).astype(np.float32)
    return wq, ws, x, _t(wq, dev), _t(ws, dev), _t(x, dev)


@pytest.mark.parametrize("fmt,n,k,m", [
    ("q4_0", 4096, 4096, 1),    # config 0
    ("tq2_0", 4096, 4096, 1),   # config 1
    ("tq2_0", 4096, 4096, 3),   # config 1, 3 columns
    ("q4_0", 4100, 4096, 3),    # config 3 row tail
    ("q4_0", 4096, 14336, 2),   # config 3 down (tall K)
    ("q4_0", 300, 28672, 1),    # K = 28672: two chunks per thread
    ("q8_0", 4096, 4096, 1),    # Q8_0 weights (extension beyond the reference)
    ("q8_0", 4100, 14336, 3),   # Q8_0 tall K, row tail, 3 columns
    ("q8_0", 300, 28672, 1),    # Q8_0 K = 28672: two chunks per thread
    ("iq4_nl", 4096, 4096, 1),  # IQ4_NL weights (second extension)
    ("iq4_nl", 4100, 14336, 3), # IQ4_NL tall K, row tail, 3 columns
])
def test_gemv_full_size_matches_oracle(cuda, fmt, n, k, m):
    wq, ws, x, twq, tws, tx = _layer(fmt, n, k, m, 11, cuda)
    xq, xd = host.quantize(fmt, tx)
    oq, od = ref.quantize(fmt, x)
    assert np.array_equal(xq.cpu().numpy(), oq) and _same_f32(xd.cpu().numpy(), od)
    y, s = host.gemv(fmt, twq, tws, xq, xd, n, k, mode=2, store_s=True)
    r, os_ = native.gemv(fmt, wq, ws, oq, od, k, want_s=True)
    assert np.array_equal(s.cpu().numpy(), os_)
    assert ref.relerr(y.cpu().numpy(), r) <= TOL


@pytest.mark.parametrize("fmt,n,k", [("tq2_0", 57344, 8192), ("tq2_0", 8192, 28672), ("q4_0", 128256, 8192),
                                     ("q4_0", 28672, 4096), ("q4_0", 6144, 4096), ("q8_0", 128256, 4096),
                                     ("iq4_nl", 28672, 4096)])
def test_gemv_large_layers_sampled_rows(cuda, fmt, n, k):
    """Configs 3/4 at full size, through the fused call (the bench's path) and the separate quantize + GEMV with the
    int32 block-dot dump: on a sample of rows (a row's result does not depend on the other rows) the block dots equal
    the C oracle's bit for bit, Y is within the rule of the oracle's exact reference, and the fused Y equals the
    separate call's."""
    rng = np.random.default_rng(23)
    wq, ws = ref.random_split(fmt, rng, n, k)
    x = rng.standard_normal((1, k)).astype(np.float32)
    twq, tws = _t(wq, cuda), _t(ws, cuda)
    y = host.quant_gemv(fmt, twq, tws, _t(x, cuda), n, k).cpu().numpy()
    xq, xd = host.quantize(fmt, _t(x, cuda))
    y2, s = host.gemv(fmt, twq, tws, xq, xd, n, k, mode=2, store_s=True)
    rows = np.unique(np.concatenate([rng.choice(n, 512, replace=False), [0, n - 1]]))
    s = s[:, torch.from_numpy(rows).to(cuda)].cpu().numpy()
    oq, od = ref.quantize(fmt, x)
    assert np.array_equal(xq.cpu().numpy(), oq) and _same_f32(xd.cpu().numpy(), od)
    r, os_ = native.gemv(fmt, wq[rows], ws[rows], oq, od, k, want_s=True)
    assert np.array_equal(s, os_)
    assert ref.relerr(y[:, rows], r) <= TOL
    assert _same_f32(y, y2.cpu().numpy())
    del twq, tws, y2
    torch.cuda.empty_cache()


def test_gemv_many_columns_and_row_stride(cuda):
    """M > 4 (column groups) and a weight row stride larger than the quant bytes."""
    rng = np.random.default_rng(3)
    for fmt, n, k, m in (("q4_0", 37, 416, 9), ("tq2_0", 37, 768, 6), ("q8_0", 37, 416, 7), ("iq4_nl", 37, 416, 11)):
        wq, ws = ref.random_split(fmt, rng, n, k)
        wide = np.zeros((n, wq.shape[1] + 48), np.uint8)
        wide[:, : wq.shape[1]] = wq
        x = rng.standard_normal((m, k)).astype(np.float32)
        xq, xd = host.quantize(fmt, _t(x, cuda))
        twide = _t(wide, cuda)[:, : wq.shape[1]]
        y, s = host.gemv(fmt, twide, _t(ws, cuda), xq, xd, n, k, mode=2, store_s=True)
        r, os_ = ref.gemv(fmt, wq, ws, xq.cpu().numpy(), xd.cpu().numpy(), k)
        assert np.array_equal(s.cpu().numpy(), os_)
        assert ref.relerr(y.cpu().numpy(), r) <= TOL


def test_gemv_edge_sizes(cuda):
    rng = np.random.default_rng(4)
    for fmt in ("q4_0", "tq2_0", "q8_0", "iq4_nl"):
        blk = ref.BLOCK[fmt]
        for n, k, m in ((0, blk, 1), (3, blk, 0), (1, blk, 1), (2, 0, 2)):
            wq, ws = ref.random_split(fmt, rng, n, k)
            if wq.shape[1] == 0:
                wq = np.zeros((n, 16), np.uint8)
            x = rng.standard_normal((m, k)).astype(np.float32)
            xq, xd = host.quantize(fmt, _t(x, cuda)) if m else (
                torch.empty((0, k), dtype=torch.int8, device=cuda), torch.empty((0, k // blk), device=cuda))
            y, s = host.gemv(fmt, _t(wq, cuda), _t(ws, cuda), xq, xd, n, k, mode=2, store_s=True)
            assert tuple(y.shape) == (m, n)
            r, os_ = ref.gemv(fmt, wq, ws, xq.cpu().numpy(), xd.cpu().numpy(), k)
            assert np.array_equal(s.cpu().numpy(), os_)
            assert np.array_equal(y.cpu().numpy(), r.astype(np.float32)) or ref.relerr(y.cpu().numpy(), r) <= TOL


def test_gemv_rejects_bad_arguments(cuda):
    wq = torch.zeros((4, 32), dtype=torch.uint8, device=cuda)
    ws = torch.zeros((4, 2), dtype=torch.int16, device=cuda)
    xq = torch.zeros((1, 64), dtype=torch.int8, device=cuda)
    xd = torch.zeros((1, 2), dtype=torch.float32, device=cuda)
    with pytest.raises(ValueError):  # misaligned quant plane
        raw = torch.zeros(4 * 32 + 16, dtype=torch.uint8, device=cuda)
        host.gemv("q4_0", raw[1:129].view(4, 32), ws, xq, xd, 4, 64)
    with pytest.raises(ValueError):  # K not a multiple of the block
        host.gemv("q4_0", wq, ws, xq, xd, 4, 48)
    with pytest.raises(RuntimeError):  # CPU tensors: no CPU path
        host.gemv("q4_0", wq.cpu(), ws.cpu(), xq.cpu(), xd.cpu(), 4, 64)
    with pytest.raises(ValueError):  # C-ABI direct: K % 32 != 0
        _lib.call("b2q_gemv_q4_0", wq.data_ptr(), 32, ws.data_ptr(), xq.data_ptr(), xd.data_ptr(), xd.data_ptr(),
                  None, 4, 48, 1, 2, None)


def test_gemv_deterministic(cuda):
    wq, ws, x, twq, tws, tx = _layer("tq2_0", 8192, 8192, 1, 5, cuda)
    a = host.quant_gemv("tq2_0", twq, tws, tx, 8192, 8192).cpu().numpy()
    b = host.quant_gemv("tq2_0", twq, tws, tx, 8192, 8192).cpu().numpy()
    assert _same_f32(a, b)


def test_launch_counter_counts_kernels(cuda):
    before = _lib.launch_count()
    wq, ws, x, twq, tws, tx = _layer("q4_0", 64, 512, 1, 2, cuda)
    xq, xd = host.quantize("q4_0", tx)
    host.gemv("q4_0", twq, tws, xq, xd, 64, 512, mode=2)
    assert _lib.launch_count() - before == 2


@pytest.mark.parametrize("fmt,n,k,m", [("q4_0", 1000, 4096, 1), ("tq2_0", 998, 8192, 3), ("q4_0", 301, 28672, 2),
                                       ("tq2_0", 37, 2048, 1), ("q8_0", 1000, 4096, 1), ("q8_0", 301, 14336, 2),
                                       ("iq4_nl", 1000, 4096, 1), ("iq4_nl", 301, 14336, 2)])
def test_ring_and_register_paths_identical(cuda, fmt, n, k, m):
    """The TMA bulk-copy ring and the register-streaming path give the same int32 dots and bit-identical Y, for every
    ring depth and rows-per-group setting; the bounded waits never fire."""
    import ctypes

    wq, ws, x, twq, tws, tx = _layer(fmt, n, k, m, 8, cuda)
    xq, xd = host.quantize(fmt, tx)
    r, os_ = ref.gemv(fmt, wq, ws, xq.cpu().numpy(), xd.cpu().numpy(), k)
    lib = _lib.load()
    outs = []
    try:
        for path, rows, stages in ((2, 0, 0), (1, 0, 0), (1, 1, 2), (1, 2, 3), (1, 4, 8), (1, 8, 4), (2, 1, 0), (2, 4, 0), (2, 8, 0)):
            _lib.call("b2q_set_tuning", rows, 0, 0)
            _lib.call("b2q_set_pipeline", path, stages)
            try:
                y, s = host.gemv(fmt, twq, tws, xq, xd, n, k, mode=2, store_s=True)
            except ValueError as e:  # a forced schedule larger than shared memory is refused, not run
                assert "does not fit" in str(e) or "not applicable" in str(e)
                continue
            assert np.array_equal(s.cpu().numpy(), os_), (path, rows, stages)
            outs.append(y.cpu().numpy())
            yf = host.quant_gemv(fmt, twq, tws, tx, n, k, split=False)
            assert _same_f32(yf.cpu().numpy(), outs[-1])
    finally:
        _lib.call("b2q_set_tuning", 0, 0, 0)
        _lib.call("b2q_set_pipeline", 0, 0)
    for y in outs[1:]:
        assert _same_f32(y, outs[0])
    assert ref.relerr(outs[0], r) <= TOL
    code = ctypes.c_int(-1)
    _lib.call("b2q_device_error", ctypes.byref(code), 1)
    assert code.value == 0


def test_allgather_receive_times_out_and_reports(cuda):
    """The fused all-gather's receive polls are bounded: with a 'peer' that never runs (its rows never arrive), every
    poll gives up after spin_limit tries, the kernel sets the status word and completes, and the context stays usable.
    Everything lives on this GPU: the peer's receive buffer is a plain local buffer, so no GPU waits on another.
    Entries are 64-bit words (high half flag, low half value bits). Some of the peer's entries are planted as already
    arrived: after a timeout a thread stops polling but still clears its remaining entries, so none stays flagged."""
    n_total, k, rows = 64, 512, 32
    wq, ws, x, twq, tws, tx = _layer("q4_0", rows, k, 1, 21, cuda)
    y = torch.zeros((1, n_total), device=cuda)
    rx = torch.zeros((2, n_total), dtype=torch.int64, device=cuda)        # this rank's receive buffer
    rx_peer = torch.zeros((2, n_total), dtype=torch.int64, device=cuda)   # stands in for rank 1's
    planted = np.arange(rows, n_total)[::3]                               # peer rows that "arrived" (value 2.5)
    rx[0, torch.from_numpy(planted).to(cuda)] = (1 << 32) | int(np.float32(2.5).view(np.uint32))
    done = torch.zeros(1, dtype=torch.int64, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    rxp = torch.tensor([rx.data_ptr(), rx_peer.data_ptr()], dtype=torch.int64, device=cuda)
    _lib.call("b2q_gemv_allgather", 0, twq.data_ptr(), twq.stride(0), tws.data_ptr(), tx.data_ptr(), k, y.data_ptr(),
              rx.data_ptr(), rxp.data_ptr(), n_total, done.data_ptr(), status.data_ptr(), 0, rows, n_total, k, 1, 0, 2,
              2000, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert int(status.item()) == 1                        # rank 1's rows never arrived
    want = host.quant_gemv("q4_0", twq, tws, tx, rows, k).cpu().numpy()
    assert _same_f32(y[:, :rows].cpu().numpy(), want)      # own rows computed
    sent = rx_peer[0, :rows].cpu().numpy()                 # and sent to the 'peer' as (flag 1, value), parity 0
    assert np.array_equal(sent >> 32, np.ones(rows, np.int64))
    assert _same_f32((sent & 0xFFFFFFFF).astype(np.uint32).view(np.float32), want[0])
    assert not rx.cpu().numpy().any()                      # every receive entry cleared, planted ones included
    assert int(done.item()) > 0                            # every CTA counted itself in
    # the context is still usable
    assert _same_f32(host.quant_gemv("q4_0", twq, tws, tx, rows, k).cpu().numpy(), want)


@pytest.mark.parametrize("fmt,n,k,m", [("tq2_0", 8192, 28672, 1), ("q4_0", 4100, 14336, 1), ("q4_0", 333, 28672, 3),
                                       ("tq2_0", 37, 28672, 2), ("q8_0", 4100, 14336, 1), ("q8_0", 333, 8192, 3),
                                       ("iq4_nl", 4100, 14336, 1)])
def test_split_k_matches_oracle_and_is_deterministic(cuda, fmt, n, k, m):
    """Tall-K layers through the split-K schedule (workspace of partial sums + ordered combine): same quantized
    activations, Y within the rule of the exact reference, within f32 rounding of the single-launch Y, and repeatable."""
    assert host.workspace_size(fmt, n, k, m) == 0  # off by default
    _lib.call("b2q_set_splitk", 1)
    try:
        _split_k_checks(cuda, fmt, n, k, m)
    finally:
        _lib.call("b2q_set_splitk", 0)


def _split_k_checks(cuda, fmt, n, k, m):
    assert host.workspace_size(fmt, n, k, m) > 0
    wq, ws, x, twq, tws, tx = _layer(fmt, n, k, m, 17, cuda)
    before = _lib.launch_count()
    ys, fq, fd = host.quant_gemv(fmt, twq, tws, tx, n, k, return_act=True)
    assert _lib.launch_count() - before == 2  # split GEMV + combine
    oq, od = ref.quantize(fmt, x)
    assert np.array_equal(fq.cpu().numpy(), oq) and _same_f32(fd.cpu().numpy(), od)
    r, _ = native.gemv(fmt, wq, ws, oq, od, k)
    ys = ys.cpu().numpy()
    assert ref.relerr(ys, r) <= TOL
    y1 = host.quant_gemv(fmt, twq, tws, tx, n, k, split=False).cpu().numpy()
    assert ref.relerr(ys, y1) <= 1e-6
    assert _same_f32(host.quant_gemv(fmt, twq, tws, tx, n, k).cpu().numpy(), ys)
    # too small a workspace: no split, exactly the single-launch result
    tiny = torch.empty(16, dtype=torch.uint8, device=cuda)
    assert _same_f32(host.quant_gemv(fmt, twq, tws, tx, n, k, workspace=tiny).cpu().numpy(), y1)


@pytest.mark.parametrize("fmt,n,k", [("tq2_0", 998, 8192), ("q4_0", 1001, 4096), ("tq2_0", 8192, 28672),
                                     ("q4_0", 301, 28672), ("tq2_0", 37, 2048), ("tq2_0", 5, 4096),
                                     ("q8_0", 1001, 4096), ("q8_0", 300, 14336), ("iq4_nl", 1001, 4096)])
def test_warp_rows_path_matches_oracle(cuda, fmt, n, k):
    """The warp-rows schedule (each warp owns whole rows, own TMA ring, one column) for several warps / rows-per-group
    / ring-depth settings: exact int32 dots, Y within the rule of the exact reference, the same Y from the fused
    quantizer prologue as from pre-quantized activations, repeatable; the bounded waits never fire."""
    import ctypes

    wq, ws, x, twq, tws, tx = _layer(fmt, n, k, 1, 31, cuda)
    xq, xd = host.quantize(fmt, tx)
    oq, od = ref.quantize(fmt, x)
    r, os_ = native.gemv(fmt, wq, ws, oq, od, k, want_s=True)
    ran = 0
    try:
        for warps, rows, stages in ((0, 0, 0), (16, 1, 2), (8, 2, 3), (4, 4, 2), (12, 1, 4), (6, 2, 2), (4, 1, 2)):
            _lib.call("b2q_set_warps", warps)
            _lib.call("b2q_set_tuning", rows, 0, 0)
            _lib.call("b2q_set_pipeline", 5, stages)
            try:
                y, s = host.gemv(fmt, twq, tws, xq, xd, n, k, mode=2, store_s=True)
            except ValueError as e:  # a forced schedule larger than shared memory is refused, not run
                assert "does not fit" in str(e), str(e)
                continue
            ran += 1
            assert np.array_equal(s.cpu().numpy(), os_), (warps, rows, stages)
            y = y.cpu().numpy()
            assert ref.relerr(y, r) <= TOL, (warps, rows, stages)
            assert _same_f32(host.gemv(fmt, twq, tws, xq, xd, n, k, mode=2)[0].cpu().numpy(), y)
            assert _same_f32(host.quant_gemv(fmt, twq, tws, tx, n, k, split=False).cpu().numpy(), y)
    finally:
        _lib.call("b2q_set_warps", 0)
        _lib.call("b2q_set_tuning", 0, 0, 0)
        _lib.call("b2q_set_pipeline", 0, 0)
    assert ran >= 2  # the planner's choice and at least one forced setting
    code = ctypes.c_int(-1)
    _lib.call("b2q_device_error", ctypes.byref(code), 1)
    assert code.value == 0


@pytest.mark.parametrize("fmt,n,k", [("tq2_0", 998, 8192), ("tq2_0", 8192, 28672), ("q4_0", 1001, 4096),
                                     ("q4_0", 300, 28672), ("tq2_0", 5, 4096), ("tq2_0", 64, 14336),
                                     ("q8_0", 1001, 4096), ("q8_0", 300, 14336), ("iq4_nl", 1001, 4096)])
def test_cluster_shared_prologue_identical(cuda, fmt, n, k):
    """No cluster, and clusters of 2, 4 and 8 CTAs splitting the fused activation prologue (each member quantizes its
    share and sends it into every other member's shared memory, completing on that member's mbarrier): the same
    quantized bytes written out, bit-identical Y, the bounded waits never fire -- also when the layer has fewer row
    groups than the cluster has members."""
    import ctypes

    wq, ws, x, twq, tws, tx = _layer(fmt, n, k, 1, 41, cuda)
    y0, q0, d0 = host.quant_gemv(fmt, twq, tws, tx, n, k, return_act=True, split=False)
    oq, od = ref.quantize(fmt, x)
    assert np.array_equal(q0.cpu().numpy(), oq) and _same_f32(d0.cpu().numpy(), od)
    y0 = y0.cpu().numpy()
    try:
        for cs in (1, 2, 4, 8):
            _lib.call("b2q_set_cluster", cs)
            y, q, d = host.quant_gemv(fmt, twq, tws, tx, n, k, return_act=True, split=False)
            assert np.array_equal(q.cpu().numpy(), oq), cs
            assert _same_f32(d.cpu().numpy(), od), cs
            assert _same_f32(y.cpu().numpy(), y0), cs
    finally:
        _lib.call("b2q_set_cluster", 0)
    code = ctypes.c_int(-1)
    _lib.call("b2q_device_error", ctypes.byref(code), 1)
    assert code.value == 0


def test_quant_gemv_into_given_output(cuda):
    """quant_gemv(out=...) writes Y into the caller's buffer (no allocation), identical to the allocating call; a
    buffer of the wrong shape, dtype or device is refused before any launch."""
    wq, ws, x, twq, tws, tx = _layer("tq2_0", 300, 4096, 2, 51, cuda)
    want = host.quant_gemv("tq2_0", twq, tws, tx, 300, 4096).cpu().numpy()
    out = torch.full((2, 300), float("nan"), device=cuda)
    got = host.quant_gemv("tq2_0", twq, tws, tx, 300, 4096, out=out)
    assert got.data_ptr() == out.data_ptr()
    assert _same_f32(out.cpu().numpy(), want)
    for bad in (torch.empty((2, 299), device=cuda), torch.empty((2, 300), dtype=torch.float64, device=cuda),
                torch.empty((300, 2), device=cuda).t()):
        with pytest.raises(ValueError):
            host.quant_gemv("tq2_0", twq, tws, tx, 300, 4096, out=bad)


@pytest.mark.parametrize("fmt,n,k", [("q4_0", 37, 416), ("tq2_0", 5, 768), ("q4_0", 4100, 4096), ("tq2_0", 999, 8192),
                                     ("q4_0", 1, 32), ("tq2_0", 3, 28672), ("q8_0", 37, 416), ("q8_0", 999, 4096),
                                     ("q8_0", 1, 32), ("iq4_nl", 37, 416), ("iq4_nl", 999, 4096)])
def test_split_device_matches_host_split(cuda, fmt, n, k):
    """The on-device cut of ggml blocks into WQ / WS (b2q_split_blocks) is byte-identical to host.split, also with a
    padded row stride, an unaligned source and a partial last CTA."""
    rng = np.random.default_rng(71)
    raw = ref.weight_blocks(fmt, rng, n, k, extreme=(n % 2 == 1))
    wq, ws = host.split(fmt, raw, n, k)
    blocks = torch.from_numpy(np.frombuffer(raw, dtype=np.uint8).copy()).to(cuda)
    dwq, dws = host.split_device(fmt, blocks, n, k)
    assert np.array_equal(dwq.cpu().numpy(), wq) and np.array_equal(dws.cpu().numpy(), ws)
    pad = wq.shape[1] + 16
    dwq2, _ = host.split_device(fmt, blocks, n, k, ldwq=pad)
    assert dwq2.stride(0) == pad and np.array_equal(dwq2.cpu().numpy(), wq)
    shifted = torch.empty(blocks.numel() + 2, dtype=torch.uint8, device=cuda)[2:]  # 2-byte offset source
    shifted.copy_(blocks)
    dwq3, dws3 = host.split_device(fmt, shifted, n, k)
    assert np.array_equal(dwq3.cpu().numpy(), wq) and np.array_equal(dws3.cpu().numpy(), ws)


def test_gguf_file_to_gemv_matches_oracle(cuda, tmp_path):
    """A GGUF file's Q4_0, TQ2_0 and Q8_0 tensors, uploaded as stored and split on the GPU, give the oracle's GEMV."""
    gguf = pytest.importorskip("gguf")
    from comp_b200 import gguf_io

    rng = np.random.default_rng(72)
    specs = [("blk.0.attn_output.weight", "q4_0", 300, 4096), ("blk.0.ffn_up.weight", "tq2_0", 200, 8192),
             ("blk.0.ffn_down.weight", "q8_0", 150, 4096), ("blk.0.attn_q.weight", "iq4_nl", 130, 4096)]
    w = gguf.GGUFWriter(str(tmp_path / "m.gguf"), "llama")
    raws = {}
    for name, fmt, n, k in specs:
        raws[name] = ref.weight_blocks(fmt, rng, n, k)
        w.add_tensor(name, np.frombuffer(raws[name], dtype=np.uint8).reshape(n, -1),
                     raw_dtype=getattr(gguf.GGMLQuantizationType, fmt.upper()))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    for name, fmt, n, k in specs:
        f, twq, tws, rn, rk = gguf_io.load_split(str(tmp_path / "m.gguf"), name, device=cuda)
        assert (f, rn, rk) == (fmt, n, k)
        x = rng.standard_normal((2, k)).astype(np.float32)
        y = host.quant_gemv(fmt, twq, tws, _t(x, cuda), n, k).cpu().numpy()
        wq, ws = host.split(fmt, raws[name], n, k)
        oq, od = ref.quantize(fmt, x)
        r, _ = native.gemv(fmt, wq, ws, oq, od, k)
        assert ref.relerr(y, r) <= TOL


@pytest.mark.parametrize("fmt,n,k,m", [("q4_0", 300, 4096, 8), ("q4_0", 1000, 4096, 16), ("q4_0", 128, 14336, 33),
                                       ("tq2_0", 257, 8192, 8), ("tq2_0", 999, 4096, 64), ("tq2_0", 128, 2048, 130),
                                       ("q4_0", 4100, 4096, 100), ("q4_0", 37, 416, 9), ("tq2_0", 5, 768, 12),
                                       ("q8_0", 300, 4096, 8), ("q8_0", 999, 4096, 64), ("q8_0", 128, 14336, 33),
                                       ("q8_0", 37, 416, 9)])
def test_tensor_core_gemm_matches_oracle(cuda, fmt, n, k, m):
    """Many columns run on the tcgen05 int8 GEMM (weights read once for all columns): exact int32 block dots, Y within
    the rule of the exact reference, the fused call (quantizer + GEMM, 2 launches) equal to the separate calls, and
    repeatable; also below the threshold when forced (padded columns) and with the byte-wise variant."""
    import ctypes

    _lib.call("b2q_set_gemm_min_columns", 1)  # also on layers too narrow to fill the GPU (the planner's rule)
    try:
        _tensor_core_checks(cuda, fmt, n, k, m)
    finally:
        _lib.call("b2q_set_gemm_min_columns", 8)
    code = ctypes.c_int(-1)
    _lib.call("b2q_device_error", ctypes.byref(code), 1)
    assert code.value == 0


def _tensor_core_checks(cuda, fmt, n, k, m):
    wq, ws, x, twq, tws, tx = _layer(fmt, n, k, m, 81, cuda)
    xq, xd = host.quantize(fmt, tx)
    oq, od = ref.quantize(fmt, x)
    assert np.array_equal(xq.cpu().numpy(), oq) and _same_f32(xd.cpu().numpy(), od)
    r, os_ = native.gemv(fmt, wq, ws, oq, od, k, want_s=True)
    y, s = host.gemv(fmt, twq, tws, xq, xd, n, k, mode=2, store_s=True)
    assert np.array_equal(s.cpu().numpy(), os_)
    y = y.cpu().numpy()
    assert ref.relerr(y, r) <= TOL
    assert _same_f32(host.gemv(fmt, twq, tws, xq, xd, n, k, mode=0)[0].cpu().numpy(), y)
    before = _lib.launch_count()
    yf = host.quant_gemv(fmt, twq, tws, tx, n, k)
    assert _lib.launch_count() - before == 2
    assert _same_f32(yf.cpu().numpy(), y)
    assert _same_f32(host.quant_gemv(fmt, twq, tws, tx, n, k, split=False).cpu().numpy(), y)
    # the quantized activations the fused call returns are the standalone quantizer's bytes
    ya, fq, fd = host.quant_gemv(fmt, twq, tws, tx, n, k, return_act=True)
    assert np.array_equal(fq.cpu().numpy(), oq) and _same_f32(fd.cpu().numpy(), od)
    assert _same_f32(ya.cpu().numpy(), y)
    # both fused schedules (warp-specialized where the shape allows it, per-block) give the same Y
    _lib.call("b2q_set_gemm_schedule", 1)
    try:
        assert _same_f32(host.quant_gemv(fmt, twq, tws, tx, n, k).cpu().numpy(), y)
    finally:
        _lib.call("b2q_set_gemm_schedule", 0)


@pytest.mark.parametrize("fmt,n,k,m", [("q4_0", 300, 4096, 1), ("tq2_0", 130, 8192, 3), ("q4_0", 64, 4096, 5),
                                       ("q8_0", 300, 4096, 2)])
def test_tensor_core_gemm_forced_on_few_columns(cuda, fmt, n, k, m):
    wq, ws, x, twq, tws, tx = _layer(fmt, n, k, m, 82, cuda)
    xq, xd = host.quantize(fmt, tx)
    r, os_ = native.gemv(fmt, wq, ws, xq.cpu().numpy(), xd.cpu().numpy(), k, want_s=True)
    _lib.call("b2q_set_gemm_min_columns", 1)
    try:
        y, s = host.gemv(fmt, twq, tws, xq, xd, n, k, mode=2, store_s=True)
    finally:
        _lib.call("b2q_set_gemm_min_columns", 8)
    assert np.array_equal(s.cpu().numpy(), os_)
    assert ref.relerr(y.cpu().numpy(), r) <= TOL


@pytest.mark.parametrize("fmt,n,k,m", [("q4_0", 40000, 4096, 16), ("tq2_0", 40000, 4096, 12), ("q8_0", 40000, 2048, 16),
                                       ("q4_0", 20000, 2048, 40), ("tq2_0", 9000, 8192, 130),
                                       ("q8_0", 12000, 4096, 100)])
def test_tensor_core_persistent_tiles(cuda, fmt, n, k, m):
    """More (row tile, column tile) pairs than resident CTAs, so each persistent CTA of the warp-specialized GEMM walks
    several tiles with its stage ring running on across them: sampled rows against the C oracle, and every row
    bit-identical to the per-block schedule; the bounded waits never fire."""
    import ctypes

    rng = np.random.default_rng(91)
    wq, ws = ref.random_split(fmt, rng, n, k)
    x = rng.standard_normal((m, k)).astype(np.float32)
    twq, tws, tx = _t(wq, cuda), _t(ws, cuda), _t(x, cuda)
    _lib.call("b2q_set_gemm_min_columns", 1)  # also where the planner would keep a narrow layer on the GEMV path
    try:
        before = _lib.launch_count()
        y = host.quant_gemv(fmt, twq, tws, tx, n, k).cpu().numpy()
        assert _lib.launch_count() - before == 2  # prep (quantizer) + GEMM
        _lib.call("b2q_set_gemm_schedule", 1)
        y1 = host.quant_gemv(fmt, twq, tws, tx, n, k).cpu().numpy()
    finally:
        _lib.call("b2q_set_gemm_schedule", 0)
        _lib.call("b2q_set_gemm_min_columns", 8)
    assert _same_f32(y, y1)
    rows = np.unique(np.concatenate([rng.choice(n, 256, replace=False), [0, 127, 128, n - 1]]))
    oq, od = ref.quantize(fmt, x)
    r, _ = native.gemv(fmt, wq[rows], ws[rows], oq, od, k)
    assert ref.relerr(y[:, rows], r) <= TOL
    code = ctypes.c_int(-1)
    _lib.call("b2q_device_error", ctypes.byref(code), 1)
    assert code.value == 0



@pytest.mark.parametrize("fmt,n,k,m", [("q4_0", 2048, 8192, 16), ("q4_0", 1300, 8192, 9), ("tq2_0", 4096, 16384, 16),
                                       ("q8_0", 2048, 4096, 16), ("q4_0", 2048, 8192, 40), ("tq2_0", 4096, 16384, 100)])
def test_tensor_core_split_k(cuda, fmt, n, k, m):
    """A layer whose 128-row tiles alone do not fill the GPU runs the warp-specialized GEMM with K split into ranges
    (three launches: prep, GEMM, the ordered combine of the ranges' partial sums), under the default planner: sampled
    rows (row tails and padding columns included) against the C oracle within the f32 tolerance, two calls bit-identical
    (the combine adds the ranges in order), and no bounded wait fired."""
    import ctypes

    rng = np.random.default_rng(93)
    wq, ws = ref.random_split(fmt, rng, n, k)
    x = rng.standard_normal((m, k)).astype(np.float32)
    twq, tws, tx = _t(wq, cuda), _t(ws, cuda), _t(x, cuda)
    before = _lib.launch_count()
    y = host.quant_gemv(fmt, twq, tws, tx, n, k).cpu().numpy()
    assert _lib.launch_count() - before == 3  # prep + split-K GEMM + combine
    y2 = host.quant_gemv(fmt, twq, tws, tx, n, k).cpu().numpy()
    assert _same_f32(y, y2)
    rows = np.unique(np.concatenate([rng.choice(n, 256, replace=False), [0, 127, 128, n - 1]]))
    oq, od = ref.quantize(fmt, x)
    r, _ = native.gemv(fmt, wq[rows], ws[rows], oq, od, k)
    assert ref.relerr(y[:, rows], r) <= TOL
    code = ctypes.c_int(-1)
    _lib.call("b2q_device_error", ctypes.byref(code), 1)
    assert code.value == 0


@pytest.mark.parametrize("fmt,n,k,m", [("iq4_nl", 37, 416, 3), ("iq4_nl", 1000, 4096, 1), ("iq4_nl", 300, 4096, 16)])
def test_iq4_nl_variants_and_many_columns(cuda, fmt, n, k, m):
    """IQ4_NL (ggml's 16-level non-linear 4-bit format): the byte-wise and the byte-permute lookup variants give the
    oracle's exact int32 block dots and the same Y; the fused call equals the separate ones; 8+ columns stay on the
    GEMV path (no tensor-core kernel for this format) and still match; extreme nibbles (levels -127 and 113) too."""
    for extreme in (False, True):
        W, x = ref.problem(fmt, n, k, m, seed=31, extreme=extreme)
        wq, ws = ref.split(fmt, W, n, k)
        twq, tws, tx = _t(wq, cuda), _t(ws, cuda), _t(x, cuda)
        xq, xd = host.quantize(fmt, tx)
        oq, od = ref.quantize(fmt, x)
        assert np.array_equal(xq.cpu().numpy(), oq) and _same_f32(xd.cpu().numpy(), od)
        r, os_ = ref.gemv(fmt, wq, ws, oq, od, k)
        y2, s2 = host.gemv(fmt, twq, tws, xq, xd, n, k, mode=2, store_s=True)
        y0, s0 = host.gemv(fmt, twq, tws, xq, xd, n, k, mode=0, store_s=True)
        assert np.array_equal(s2.cpu().numpy(), os_) and np.array_equal(s0.cpu().numpy(), os_)
        assert _same_f32(y0.cpu().numpy(), y2.cpu().numpy())
        assert ref.relerr(y2.cpu().numpy(), r) <= TOL
        assert _same_f32(host.quant_gemv(fmt, twq, tws, tx, n, k, split=False).cpu().numpy(), y2.cpu().numpy())
        assert ref.relerr(host.quant_gemv(fmt, twq, tws, tx, n, k).cpu().numpy(), r) <= TOL

"""Host-side logic and the C-ABI library, without a GPU."""

import ctypes
import os
import re

import numpy as np
import pytest
import torch

from comp_b200 import _lib, host
from comp_b200.dist import partition, slice_rows
from oracle import ref

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "comp_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(b2q_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_symbols()
    assert len(names) >= 15
    for name in names:
        assert hasattr(lib, name), f"{name} declared in include/comp_b200.h but not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature in comp_b200._lib"
    assert set(_lib.SIGNATURES) == set(names)


def test_library_metadata_calls_need_no_gpu():
    assert _lib.version().startswith("comp_b200")
    assert _lib.launch_count() >= 0
    # argument validation happens before any CUDA call: a bad K is rejected on the host
    with pytest.raises(ValueError, match="multiple"):
        _lib.call("b2q_quant_q8_0", 16, 48, 16, 16, 1, 40, None)
    with pytest.raises(ValueError, match="variant|multiple|null"):
        _lib.call("b2q_gemv_tq2_0", 16, 64, 16, 16, 16, 16, None, 4, 100, 1, 2, None)
    assert "multiple" in _lib.last_error()
    lib = _lib.load()
    # the newer entry points validate on the host too, before any CUDA call
    with pytest.raises(ValueError, match="multiple"):
        _lib.call("b2q_gemv_iq4_nl", 16, 16, 16, 16, 16, 16, None, 4, 100, 1, 2, None)
    # Q4_K: K a multiple of 256 but not of 1024 (its scale records would not fill whole 16-byte units)
    with pytest.raises(ValueError, match="Q4_K needs K a multiple of 1024"):
        _lib.call("b2q_gemv_q4_k", 16, 384, 16, 16, 16, 16, None, 4, 768, 1, 2, None)
    assert lib.b2q_quant_gemv_pinned(9, None, 0, None, None, 0, None, 4, 64, 1, None, 0, None) == -1
    assert "Q4_K (4)" in _lib.last_error()
    assert lib.b2q_quant_gemv_pinned(0, None, 0, None, None, 0, None, -1, 64, 1, None, 0, None) == -1
    assert lib.b2q_quant_gemv_pinned(0, None, 0, None, None, 0, None, 0, 64, 1, None, 0, None) == 0  # empty: no-op
    assert lib.b2q_stage_pinned(None, 0, None, -1, 64, None) == -1
    assert lib.b2q_stage_pinned(None, 0, None, 0, 64, None) == 0  # empty: no-op
    assert lib.b2q_host_device_pointer(None, None) == -1


def test_split_layout_is_kurns():
    """host.split == the raw ggml block slicing, byte for byte (the reference's test_split_layout_is_kurns,
    tests/test_komp.py:69-82)."""
    n, k = 3, 96
    W, _ = ref.problem("q4_0", n, k, 1, seed=0)
    wq, ws = host.split_q4_0(W, n, k)
    for r in range(n):
        for b in range(k // 32):
            blk = W[(r * (k // 32) + b) * 18 : (r * (k // 32) + b + 1) * 18]
            assert bytes(wq[r, b * 16 : b * 16 + 16]) == blk[2:18]
            assert ws[r, b].tobytes() == blk[:2]
    assert wq.dtype == np.uint8 and ws.dtype == np.int16
    W, _ = ref.problem("tq2_0", 2, 512, 1, seed=0)
    wq, ws = host.split("tq2_0", W, 2, 512)
    assert np.array_equal(host.tq2_0_qplane(W, 4), wq.reshape(4, 64))
    for b in range(4):
        assert ws.reshape(-1)[b].tobytes() == W[b * 66 + 64 : b * 66 + 66]
    with pytest.raises(ValueError):
        host.split("q4_0", W, 2, 500)


def test_act_blocks_layout():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((2, 512)).astype(np.float32)
    xq, xd = ref.quant_q8_0(x)
    b = host.act_blocks("q4_0", xq, xd)
    assert len(b) == 2 * 16 * 34
    assert np.frombuffer(b[:2], np.float16)[0] == np.float16(xd[0, 0])
    assert np.array_equal(np.frombuffer(b[2:34], np.int8), xq[0, :32])
    kq, kd, bs = ref.quant_q8_K(x)
    b = host.act_blocks("tq2_0", kq, kd)
    assert len(b) == 2 * 2 * 292
    assert np.frombuffer(b[:4], np.float32)[0] == kd[0, 0]
    assert np.array_equal(np.frombuffer(b[260:292], np.int16), bs[0, 0])


def test_compute_calls_refuse_cpu_tensors():
    """There is no CPU path: CPU tensors raise instead of silently computing elsewhere."""
    x = torch.zeros((1, 64), dtype=torch.float32)
    with pytest.raises(RuntimeError, match="CUDA"):
        host.quantize("q4_0", x)
    with pytest.raises(RuntimeError, match="CUDA"):
        host.gemv("q4_0", torch.zeros((2, 32), dtype=torch.uint8), torch.zeros((2, 2), dtype=torch.int16),
                  torch.zeros((1, 64), dtype=torch.int8), torch.zeros((1, 2)), 2, 64)
    with pytest.raises(ValueError, match="unknown weight format"):
        host.quantize("q5_K", x)
    # the pinned-host form needs the weights on a GPU too
    with pytest.raises(RuntimeError, match="CUDA"):
        host.quant_gemv_pinned("q4_0", torch.zeros((2, 32), dtype=torch.uint8), torch.zeros((2, 2), dtype=torch.int16),
                               x, 2, 64, torch.zeros((1, 2)))


def test_workspace_sizes_need_no_gpu():
    """Workspace queries are host arithmetic: the pinned form stages M*K f32 (rounded up to 256 bytes) in front of the
    GEMV's own workspace; empty layers need none; an unknown format gives 0."""
    for fmt in ("q4_0", "tq2_0", "q8_0", "iq4_nl"):
        for n, k, m in ((4096, 4096, 1), (37, 1024, 3), (128256, 8192, 16)):
            g = host.workspace_size(fmt, n, k, m)
            assert host.pinned_workspace_size(fmt, n, k, m) == -(-m * k * 4 // 256) * 256 + g
        assert host.pinned_workspace_size(fmt, 0, 4096, 1) == 0
    # IQ4_NL has no tensor-core path, so many columns need no activation tiles
    assert host.workspace_size("iq4_nl", 128256, 8192, 16) == 0 < host.workspace_size("q4_0", 128256, 8192, 16)
    assert _lib.load().b2q_pinned_workspace_size(7, 64, 1024, 1) == 0


def test_partition_covers_rows_once():
    for n in (0, 1, 5, 4096, 4100, 57344, 128256):
        for p in (1, 2, 3, 4, 8):
            parts = partition(n, p)
            assert len(parts) == p
            per = slice_rows(n, p)
            covered = []
            for r, (r0, cnt) in enumerate(parts):
                assert 0 <= cnt <= per and (cnt == 0 or r0 == r * per)
                covered.extend(range(r0, r0 + cnt))
            assert covered == list(range(n))


def test_ctypes_signatures_match_header_arity():
    text = re.sub(r"/\*.*?\*/", "", open(os.path.join(ROOT, "include", "comp_b200.h")).read(), flags=re.S)
    for name, (_, args) in _lib.SIGNATURES.items():
        m = re.search(rf"\b{name}\s*\(([^)]*)\)", text)
        assert m, name
        params = [p for p in m.group(1).split(",") if p.strip() and p.strip() != "void"]
        assert len(params) == len(args), f"{name}: header has {len(params)} parameters, ctypes {len(args)}"
    assert ctypes.sizeof(ctypes.c_void_p) == 8


def test_verify_json_line_fields():
    """verify --all --json: COMP's per-check fields as JSON, plus us / GB/s / HBM fraction when the check was timed."""
    import json

    from comp_b200 import verify

    r = {"fmt": "q4_0", "n": 4096, "k": 4096, "m": 1, "quant": True, "idots": True, "rebuilt": False,
         "relerr": 2e-7, "ok": False, "us": 2.0}
    d = json.loads(verify.json_line(r, 2, label="bn=32", extreme=True, peak=6000.0))
    assert d["ok"] is False and d["mode"] == "dp4a" and d["extreme"] is True and d["config"] == "bn=32"
    assert d["quant"] == "exact" and d["idots"] == "exact" and d["reference_dot"] == "DIFFERS"
    want = (4096 * 4096 * 18 // 32 + 4096 + 4 * 4096 // 32 + 4 * 4096) / 2.0 / 1e3
    assert abs(d["gbs"] - want) < 0.1 and abs(d["hbm_frac"] - want / 6000.0) < 1e-4 and d["us"] == 2.0
    r.pop("us")
    assert "gbs" not in json.loads(verify.json_line(r, 0))


@pytest.mark.parametrize("fmt,n,k,m", [("q4_0", 37, 416, 3), ("tq2_0", 5, 1280, 2), ("tq2_0", 64, 1024, 1),
                                       ("q8_0", 37, 416, 3), ("iq4_nl", 37, 416, 3)])
def test_verify_torch_references_equal_the_oracle(fmt, n, k, m):
    """comp_b200.verify checks the kernels against torch restatements of the exact references; run here on CPU
    tensors, they must equal the oracle (itself pinned to the reference's recorded outputs): quantizer bytes and
    scales, decoded weights, int32 block dots and the f64 reference dot, on random and extreme data."""
    from comp_b200 import verify

    for seed, extreme in ((1, False), (2, True)):
        wq, ws, x = verify.problem(fmt, n, k, m, seed, extreme, torch.device("cpu"))
        xq, xd = verify.ref_quantize(fmt, x)
        oq, od = ref.quantize(fmt, x.numpy())
        assert np.array_equal(xq.numpy(), oq) and np.array_equal(xd.numpy().view(np.uint32), od.view(np.uint32))
        assert np.array_equal(verify.ref_values(fmt, wq, k).numpy(), ref.decode(fmt, wq.numpy(), k))
        r, s = ref.gemv(fmt, wq.numpy(), ws.numpy(), oq, od, k)
        dots = verify.ref_dots(fmt, wq, xq, k)
        assert np.array_equal(dots.numpy(), s)
        assert np.array_equal(verify.ref_dot(fmt, ws, xd, dots).numpy().view(np.uint64), r.view(np.uint64))

"""The split-K entry point that allocates nothing (b2q_quant_gemv_splitk_noalloc), for callers that cannot allocate
device memory: an inference engine that reserves all GPU memory at start-up, or an FFI caller with no device
allocator. Its partial sums live in a fixed 4 MiB array inside the library instead of a caller-provided workspace.

Checked through the C ABI against the existing entry point b2q_quant_gemv (one launch, no scratch) within the
tests' tolerance, on calls in a row: first one whose partial sums fill the array exactly (splits * M * N * 4 bytes
== the array's size), then two layers of other shapes, each running on the previous call's leftovers in the shared
array. Self-contained: passes alone in a fresh process and after the other tests."""

import ctypes

import numpy as np
import pytest
import torch

from comp_b200 import _lib
from oracle import ref

pytestmark = pytest.mark.gpu

TOL = 1e-5  # KURN's relative-error rule, as in the other GPU tests


def _layer(fmt, n, k, m, seed, dev):
    rng = np.random.default_rng(seed)
    wq, ws = ref.random_split(fmt, rng, n, k)
    x = rng.standard_normal((m, k)).astype(np.float32)
    return (torch.from_numpy(wq).to(dev), torch.from_numpy(np.ascontiguousarray(ws)).to(dev),
            torch.from_numpy(x).to(dev))


def _run(name, fid, wq, ws, x, y, n, k, m, *extra):
    lib = _lib.load()
    rc = getattr(lib, name)(fid, wq.data_ptr(), wq.stride(0), ws.data_ptr(), x.data_ptr(), x.stride(0), *extra[:2],
                            y.data_ptr(), n, k, m, *extra[2:], torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lib.last_error()


def _relerr(got, want):
    return ref.relerr(got.cpu().numpy(), want.cpu().numpy())


def test_noalloc_split_gemv_matches_existing_entry_point_twice(cuda):
    lib = _lib.load()
    assert lib.b2q_noalloc_scratch_bytes() == 4 << 20
    # (fmt, id, N, K, M, splits, seed); the first fills the 4 MiB exactly: 16 splits x 4 columns x 16384 rows x 4 B
    calls = [("q4_0", 0, 16384, 512, 4, 16, 4), ("tq2_0", 1, 8192, 28672, 1, 2, 5), ("q4_0", 0, 4100, 14336, 3, 4, 6)]
    assert calls[0][4] * calls[0][2] * calls[0][5] * 4 == lib.b2q_noalloc_scratch_bytes()
    for fmt, fid, n, k, m, splits, seed in calls:
        wq, ws, x = _layer(fmt, n, k, m, seed, cuda)
        want = torch.empty((m, n), device=cuda)
        _run("b2q_quant_gemv", fid, wq, ws, x, want, n, k, m, None, None)
        got = torch.full((m, n), float("nan"), device=cuda)
        torch.cuda.synchronize()
        allocated = torch.cuda.memory_allocated(cuda)
        lib_rc = lib.b2q_quant_gemv_splitk_noalloc(fid, wq.data_ptr(), wq.stride(0), ws.data_ptr(), x.data_ptr(),
                                                   x.stride(0), got.data_ptr(), n, k, m, splits,
                                                   torch.cuda.current_stream().cuda_stream)
        assert lib_rc == 0, _lib.last_error()
        torch.cuda.synchronize()
        assert torch.cuda.memory_allocated(cuda) == allocated  # nothing allocated through torch
        assert not torch.isnan(got).any()
        assert _relerr(got, want) <= TOL


def test_noalloc_rejects_what_does_not_fit(cuda):
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    # 16 splits x 4 columns x 16385 rows x 4 bytes = 4194560 > 4 MiB. Every buffer is full size for the call, so
    # nothing could be read out of bounds even if the size check were missing.
    n, k, m = 16385, 512, 4
    assert 16 * m * n * 4 > lib.b2q_noalloc_scratch_bytes()
    wq, ws, x = _layer("q4_0", n, k, m, 9, cuda)
    y = torch.empty((m, n), device=cuda)
    rc = lib.b2q_quant_gemv_splitk_noalloc(0, wq.data_ptr(), wq.stride(0), ws.data_ptr(), x.data_ptr(), k,
                                           y.data_ptr(), n, k, m, 16, stream)
    assert rc == -4 and "built-in scratch" in _lib.last_error()
    rc = lib.b2q_quant_gemv_splitk_noalloc(0, wq.data_ptr(), wq.stride(0), ws.data_ptr(), x.data_ptr(), k,
                                           y.data_ptr(), n, k, m, 3, stream)  # 3 does not divide 16 blocks
    assert rc == -1 and "splits" in _lib.last_error()
    torch.cuda.synchronize()
    code = ctypes.c_int(-1)
    assert lib.b2q_device_error(ctypes.byref(code), 0) == 0 and code.value == 0

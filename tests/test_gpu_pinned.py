"""b2q_quant_gemv_pinned / host.quant_gemv_pinned: activations and output in pinned host memory.

The copy kernel and the fused GEMV run through the host buffers' device mappings. Y must equal the device-memory call
(host.quant_gemv) bit for bit on every schedule, also when calls reuse one workspace back to back with programmatic
dependent launch, and memory the GPU cannot reach must be refused before anything is launched.
"""

import ctypes

import numpy as np
import pytest
import torch

from comp_b200 import _lib, host
from oracle import native, ref

pytestmark = pytest.mark.gpu

TOL = 1e-5  # KURN's rule (src/komp/verify.py:28)


def _same_f32(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


def _layer(fmt, n, k, m, seed, dev, ldx=None):
    rng = np.random.default_rng(seed)
    wq, ws = ref.random_split(fmt, rng, n, k)
    x = rng.standard_normal((m, k)).astype(np.float32)
    xh = torch.empty((m, ldx or k), dtype=torch.float32).pin_memory()[:, :k]
    xh.copy_(torch.from_numpy(x))
    return wq, ws, x, torch.from_numpy(wq).to(dev), torch.from_numpy(ws).to(dev), xh


def _no_device_error():
    code = ctypes.c_int(-1)
    _lib.call("b2q_device_error", ctypes.byref(code), 1)
    return code.value == 0


@pytest.mark.parametrize("fmt,n,k,m,ldx", [("q4_0", 300, 4096, 1, None), ("tq2_0", 999, 8192, 3, None),
                                           ("q8_0", 130, 4096, 2, 4100), ("tq2_0", 8192, 28672, 1, None),
                                           ("q4_0", 4100, 4096, 1, 4104), ("q4_0", 1000, 4096, 16, None),
                                           ("tq2_0", 999, 4096, 12, None), ("q4_0", 37, 416, 5, None),
                                           ("iq4_nl", 999, 4096, 2, None)])
def test_pinned_matches_device_call(cuda, fmt, n, k, m, ldx):
    """Same Y as the device-memory fused call, bit for bit (GEMV schedules, and the quantizer + tensor-core GEMM for
    8+ columns), within the rule of the exact reference; two launches for the one-kernel schedules."""
    wq, ws, x, twq, tws, xh = _layer(fmt, n, k, m, 101, cuda, ldx)
    xd = xh.to(cuda)
    before = _lib.launch_count()
    want = host.quant_gemv(fmt, twq, tws, xd, n, k).cpu().numpy()
    device_launches = _lib.launch_count() - before
    out = torch.full((m, n), float("nan")).pin_memory()
    before = _lib.launch_count()
    got = host.quant_gemv_pinned(fmt, twq, tws, xh, n, k, out)
    launches = _lib.launch_count() - before
    torch.cuda.current_stream().synchronize()
    assert got.data_ptr() == out.data_ptr()
    assert _same_f32(out.numpy(), want)
    assert launches == device_launches + 1  # the copy kernel, then the device call's own kernels
    oq, od = ref.quantize(fmt, x)
    r = native.gemv(fmt, wq, ws, oq, od, k, want_s=False)[0]
    assert ref.relerr(out.numpy(), r) <= TOL
    assert _no_device_error()


def test_pinned_calls_back_to_back_share_a_workspace(cuda):
    """Twelve calls over three layers, enqueued without a host wait and all staging their activations in one
    workspace: each call's copy kernel waits for the previous kernel before overwriting the staging area, so every Y
    is the device-memory call's."""
    shapes = [("tq2_0", 2048, 8192), ("tq2_0", 512, 28672), ("q4_0", 4096, 8192)]
    layers = [_layer(f, n, k, 1, 200 + i, cuda) for i, (f, n, k) in enumerate(shapes)]
    need = max(host.pinned_workspace_size(f, n, k, 1) for f, n, k in shapes)
    work = torch.empty(need, dtype=torch.uint8, device=cuda)
    wants, outs = [], []
    for rep in range(4):
        for (f, n, k), (_, _, _, twq, tws, xh) in zip(shapes, layers):
            xr = (xh * (rep + 1)).pin_memory()  # a different input per call
            wants.append(host.quant_gemv(f, twq, tws, xr.to(cuda), n, k).cpu().numpy())
            outs.append((xr, torch.empty((1, n)).pin_memory()))
    torch.cuda.synchronize()
    i = 0
    for rep in range(4):
        for (f, n, k), (_, _, _, twq, tws, _) in zip(shapes, layers):
            xr, out = outs[i]
            host.quant_gemv_pinned(f, twq, tws, xr, n, k, out, workspace=work)
            i += 1
    torch.cuda.current_stream().synchronize()
    for (xr, out), want in zip(outs, wants):
        assert _same_f32(out.numpy(), want)
    assert _no_device_error()


def test_pinned_refuses_unreachable_memory(cuda):
    """Pageable host memory, device memory in place of a host buffer, a short workspace and a misaligned x are
    refused with an error status before any launch."""
    f, n, k, m = "q4_0", 64, 1024, 1
    _, _, x, twq, tws, xh = _layer(f, n, k, m, 7, cuda)
    out = torch.empty((m, n)).pin_memory()
    need = host.pinned_workspace_size(f, n, k, m)
    work = torch.empty(need, dtype=torch.uint8, device=cuda)
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    pageable_x = np.ascontiguousarray(x)
    pageable_y = np.zeros((m, n), np.float32)
    xdev = xh.to(cuda)

    def call(xp, ldx, yp, wp, wbytes):
        return lib.b2q_quant_gemv_pinned(0, twq.data_ptr(), twq.stride(0), tws.data_ptr(), xp, ldx, yp, n, k, m, wp,
                                         wbytes, stream)

    before = _lib.launch_count()
    assert call(pageable_x.ctypes.data, k, out.data_ptr(), work.data_ptr(), need) == -1      # pageable x
    assert call(xh.data_ptr(), k, pageable_y.ctypes.data, work.data_ptr(), need) == -1        # pageable y
    assert call(xdev.data_ptr(), k, out.data_ptr(), work.data_ptr(), need) == -1              # device x
    assert call(xh.data_ptr(), k, out.data_ptr(), work.data_ptr(), need - 256) == -1          # short workspace
    assert call(xh.data_ptr(), k, out.data_ptr(), None, 0) == -1                              # no workspace
    assert call(xh.data_ptr() + 4, k, out.data_ptr(), work.data_ptr(), need) == -2            # misaligned x
    assert _lib.launch_count() == before
    with pytest.raises(ValueError):
        host.quant_gemv_pinned(f, twq, tws, torch.from_numpy(pageable_x), n, k, out)
    with pytest.raises(ValueError):
        host.quant_gemv_pinned(f, twq, tws, xh, n, k, torch.empty((m, n)))
    # a valid call still works after the refusals; empty layers touch nothing; K = 0 writes Y = 0
    assert call(xh.data_ptr(), k, out.data_ptr(), work.data_ptr(), need) == 0
    torch.cuda.current_stream().synchronize()
    assert lib.b2q_quant_gemv_pinned(0, twq.data_ptr(), twq.stride(0), tws.data_ptr(), None, k, None, 0, k, m, None,
                                     0, stream) == 0
    assert lib.b2q_quant_gemv_pinned(0, None, 0, None, None, 0, out.data_ptr(), n, 0, m, None, 0, stream) == 0
    torch.cuda.current_stream().synchronize()
    assert not out.numpy().any()
    assert _no_device_error()


def test_stage_pinned_and_host_device_pointer(cuda):
    """b2q_stage_pinned copies pinned rows (padded row stride) into device memory exactly; b2q_host_device_pointer
    gives a pinned buffer's device address; both refuse pageable and device memory (and staging into host memory)
    before any launch."""
    m, k, ldx = 3, 8192, 8200
    _, _, x, _, _, xh = _layer("tq2_0", 4, k, m, 11, cuda, ldx)
    stage = torch.full((m, k), float("nan"), device=cuda)
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    before = _lib.launch_count()
    assert lib.b2q_stage_pinned(xh.data_ptr(), ldx, stage.data_ptr(), m, k, stream) == 0
    assert _lib.launch_count() - before == 1
    assert _same_f32(stage.cpu().numpy(), x)
    pageable = np.ascontiguousarray(x)
    before = _lib.launch_count()
    assert lib.b2q_stage_pinned(pageable.ctypes.data, k, stage.data_ptr(), m, k, stream) == -1
    assert lib.b2q_stage_pinned(stage.data_ptr(), k, stage.data_ptr(), m, k, stream) == -1   # device memory as x
    assert lib.b2q_stage_pinned(xh.data_ptr(), ldx, xh.data_ptr(), m, k, stream) == -1       # host memory as stage
    assert lib.b2q_stage_pinned(xh.data_ptr() + 4, ldx, stage.data_ptr(), m, k, stream) == -2
    assert _lib.launch_count() == before
    dp = ctypes.c_void_p()
    assert lib.b2q_host_device_pointer(xh.data_ptr(), ctypes.byref(dp)) == 0 and dp.value
    assert lib.b2q_host_device_pointer(pageable.ctypes.data, ctypes.byref(dp)) == -1 and not dp.value
    assert lib.b2q_host_device_pointer(stage.data_ptr(), ctypes.byref(dp)) == -1 and not dp.value
    assert _no_device_error()

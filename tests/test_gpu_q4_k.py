"""Q4_K weights (ggml block_q4_K, an extension beyond the reference) on the GPU, through the C-ABI via comp_b200.host:
exact q8_K bytes and int32 block dots (S = sum_j sc_j * sub-block dot) against the C oracle, Y within KURN's 1e-5 rule
of the f64 reference, the fused call equal to the separate calls, both variants, column groups, split-K, the on-device
split of ggml blocks, a GGUF file end to end and pinned host buffers. The oracle is pinned to gguf-py's Q4_K codec
(tests/test_oracle_golden.py)."""

import numpy as np
import pytest
import torch

from comp_b200 import _lib, host
from oracle import native, ref

pytestmark = pytest.mark.gpu

TOL = 1e-5  # KURN's rule (src/komp/verify.py:28)


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _same_f32(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


@pytest.mark.parametrize("n,k,m", [(37, 1024, 3), (4096, 4096, 1), (4100, 14336, 2), (300, 4096, 9), (1, 1024, 1),
                                   (999, 8192, 4)])
def test_q4_k_matches_oracle(cuda, n, k, m):
    for extreme in (False, True):
        W, x = ref.problem("q4_k", n, k, m, seed=41, extreme=extreme)
        wq, ws = host.split("q4_k", W, n, k)
        twq, tws, tx = _t(wq, cuda), _t(ws, cuda), _t(x, cuda)
        xq, xd = host.quantize("q4_k", tx)
        oq, od = ref.quantize("q4_k", x)
        assert np.array_equal(xq.cpu().numpy(), oq) and _same_f32(xd.cpu().numpy(), od)
        r, os_ = native.gemv("q4_k", wq, ws, oq, od, k, want_s=True)
        y2, s2 = host.gemv("q4_k", twq, tws, xq, xd, n, k, mode=2, store_s=True)
        y0, s0 = host.gemv("q4_k", twq, tws, xq, xd, n, k, mode=0, store_s=True)
        assert np.array_equal(s2.cpu().numpy(), os_) and np.array_equal(s0.cpu().numpy(), os_)
        assert _same_f32(y0.cpu().numpy(), y2.cpu().numpy())
        assert ref.relerr(y2.cpu().numpy(), r) <= TOL
        y_f = host.quant_gemv("q4_k", twq, tws, tx, n, k, split=False).cpu().numpy()
        if m <= 4:  # one column group: the fused call runs the same schedule as the separate ones
            assert _same_f32(y_f, y2.cpu().numpy())
        assert ref.relerr(y_f, r) <= TOL
        yq, xq2, xd2 = host.quant_gemv("q4_k", twq, tws, tx, n, k, return_act=True, split=False)
        assert np.array_equal(xq2.cpu().numpy(), oq) and _same_f32(xd2.cpu().numpy(), od)


def test_q4_k_split_k_matches_oracle(cuda):
    n, k, m = 4100, 16384, 2
    W, x = ref.problem("q4_k", n, k, m, seed=43)
    wq, ws = host.split("q4_k", W, n, k)
    twq, tws, tx = _t(wq, cuda), _t(ws, cuda), _t(x, cuda)
    oq, od = ref.quantize("q4_k", x)
    r, _ = native.gemv("q4_k", wq, ws, oq, od, k)
    _lib.call("b2q_set_splitk", 2)
    try:
        assert host.workspace_size("q4_k", n, k, m) > 0
        y = host.quant_gemv("q4_k", twq, tws, tx, n, k).cpu().numpy()
        y_again = host.quant_gemv("q4_k", twq, tws, tx, n, k).cpu().numpy()
    finally:
        _lib.call("b2q_set_splitk", 0)
    assert ref.relerr(y, r) <= TOL and _same_f32(y, y_again)


def test_q4_k_rejects_k_not_a_multiple_of_1024(cuda):
    W, x = ref.problem("q4_k", 8, 768, 1, seed=44)
    wq, ws = host.split("q4_k", W, 8, 768)
    xq, xd = host.quantize("q4_k", _t(x, cuda))
    with pytest.raises(ValueError, match="1024"):
        host.gemv("q4_k", _t(wq, cuda), _t(ws, cuda), xq, xd, 8, 768)


@pytest.mark.parametrize("n,k", [(37, 1024), (999, 4096), (1, 1024), (300, 14336)])
def test_q4_k_split_device_matches_host_split(cuda, n, k):
    rng = np.random.default_rng(45)
    raw = ref.weight_blocks("q4_k", rng, n, k, extreme=(n % 2 == 1))
    wq, ws = host.split("q4_k", raw, n, k)
    blocks = torch.from_numpy(np.frombuffer(raw, dtype=np.uint8).copy()).to(cuda)
    dwq, dws = host.split_device("q4_k", blocks, n, k)
    assert np.array_equal(dwq.cpu().numpy(), wq) and np.array_equal(dws.cpu().numpy(), ws)
    dwq2, _ = host.split_device("q4_k", blocks, n, k, ldwq=wq.shape[1] + 16)
    assert np.array_equal(dwq2.cpu().numpy(), wq)


def test_q4_k_gguf_file_to_gemv_matches_oracle(cuda, tmp_path):
    gguf = pytest.importorskip("gguf")
    from comp_b200 import gguf_io

    rng = np.random.default_rng(46)
    n, k = 300, 4096
    raw = ref.weight_blocks("q4_k", rng, n, k)
    w = gguf.GGUFWriter(str(tmp_path / "m.gguf"), "llama")
    w.add_tensor("blk.0.ffn_gate.weight", np.frombuffer(raw, dtype=np.uint8).reshape(n, -1),
                 raw_dtype=gguf.GGMLQuantizationType.Q4_K)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    f, twq, tws, rn, rk = gguf_io.load_split(str(tmp_path / "m.gguf"), "blk.0.ffn_gate.weight", device=cuda)
    assert (f, rn, rk) == ("q4_k", n, k)
    x = rng.standard_normal((2, k)).astype(np.float32)
    y = host.quant_gemv("q4_k", twq, tws, _t(x, cuda), n, k).cpu().numpy()
    wq, ws = host.split("q4_k", raw, n, k)
    oq, od = ref.quantize("q4_k", x)
    r, _ = native.gemv("q4_k", wq, ws, oq, od, k)
    assert ref.relerr(y, r) <= TOL


def test_q4_k_pinned_host_buffers(cuda):
    n, k, m = 999, 4096, 2
    W, x = ref.problem("q4_k", n, k, m, seed=47)
    wq, ws = host.split("q4_k", W, n, k)
    twq, tws = _t(wq, cuda), _t(ws, cuda)
    xh = torch.from_numpy(x).pin_memory()
    out = torch.full((m, n), float("nan")).pin_memory()
    host.quant_gemv_pinned("q4_k", twq, tws, xh, n, k, out)
    torch.cuda.synchronize()
    want = host.quant_gemv("q4_k", twq, tws, xh.to(cuda), n, k).cpu().numpy()
    assert _same_f32(out.numpy(), want)

"""Worker for tests/test_gpu_vs_komp.py: runs COMP itself (the reference package installed under baseline/_ref, its
Triton kernels JIT-compiled for this GPU, mode 2) and this library on the same seeded inputs, at BASELINE's full sizes,
and prints one JSON line per case: quantized bytes equal, int32 block dots (store_s) equal, and the relative error of
this library's Y (separate quantize + gemv, and the fused quant_gemv) against the reference's Y.

Runs in its own process because TRITON_INTERPRET must be unset before triton is imported."""

import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import torch  # noqa: E402
from komp import host as khost  # noqa: E402  (the reference, from baseline/_ref on PYTHONPATH)

from bench import make_layer_gpu, make_x  # noqa: E402
from comp_b200 import host  # noqa: E402

# BASELINE configs 0, 1 (M = 1 and 3), 3 (the N = 4100 row tail and the tall-K down layer) and 4, at full size
CASES = [("q4_0", 4096, 4096, 1), ("tq2_0", 4096, 4096, 1), ("tq2_0", 4096, 4096, 3), ("q4_0", 4100, 14336, 2),
         ("q4_0", 6144, 4096, 3), ("tq2_0", 57344, 8192, 1), ("tq2_0", 8192, 28672, 1), ("q4_0", 128256, 8192, 1)]


def relerr(y, r):
    r = r.double()
    return float((y.double() - r).abs().max() / r.abs().max().clamp_min(1e-300))


def main():
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    for i, (fmt, n, k, m) in enumerate(CASES):
        wq, ws = make_layer_gpu(fmt, n, k, 500 + i, dev)
        x = torch.from_numpy(make_x(k, m, 600 + i)).to(dev)
        kq, kd = khost.quantize(fmt, x)
        ky, ks = khost.gemv(fmt, wq, ws, kq, kd, n, k, mode=2, store_s=True)
        oq, od = host.quantize(fmt, x)
        oy, os_ = host.gemv(fmt, wq, ws, oq, od, n, k, mode=2, store_s=True)
        fused = host.quant_gemv(fmt, wq, ws, x, n, k)
        torch.cuda.synchronize()
        print(json.dumps({
            "case": f"{fmt} {n}x{k} m={m}",
            "quant_bytes_equal": bool(torch.equal(kq, oq) and torch.equal(kd.view(torch.int32), od.view(torch.int32))),
            "int32_block_dots_equal": bool(torch.equal(ks, os_)),
            "relerr_separate": relerr(oy, ky), "relerr_fused": relerr(fused, ky)}), flush=True)
        del wq, ws, ks, os_, ky, oy, fused
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()

"""Generates tests/golden/komp_golden.npz: outputs of the REFERENCE itself (COMP's Triton kernels run on the CPU by
the Triton interpreter, TRITON_INTERPRET=1) on seeded inputs, used to pin the oracle and to check the CUDA kernels.

Run in a container that has the reference checked out (it is read, never modified):

    python tests/golden/make_golden.py --reference /path/to/komp-project

What is recorded (every array is the reference's own output for the stored input):
  quant/*     config-2 quantizer input x f32 [4][14336]; komp host.quantize("q4_0") -> q8_0 (xq, xd) and
              host.quantize("tq2_0") -> q8_K (xq, xd)
  gemv/<id>/* for each problem of src/komp/verify.py:141 (plus two config-0/1 row slices), random and extreme data:
              ggml weight bytes W, activations x, komp quantize -> (xq, xd), komp gemv store_s=True in mode 0
              (bytes) and mode 1 (dp4a fallback) -> (y0, s0), (y1, s1)
  dp4a/*      the check_dp4a word mix of src/komp/verify.py:44-54 and kernels.dp4a_probe(MODE=1) outputs
  decode/*    kernels.q4_0_decode / tq2_0_decode outputs on random quant planes (tq2_0 includes crumb 3)

Inputs come from oracle.ref's seeded generators (numpy PCG64); the arrays themselves are stored, so the tests do not
depend on regenerating them.
"""

import argparse
import json
import os
import random
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))

PROBLEMS = {  # src/komp/verify.py:141, plus a 32-row slice of BASELINE configs 0 and 1 (K=4096)
    "q4_0": ((64, 512, 1), (37, 416, 3), (5, 96, 2), (32, 4096, 1)),
    "tq2_0": ((64, 1024, 1), (37, 768, 3), (5, 1280, 2), (32, 4096, 3)),
}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of the komp project (contains src/komp)")
    ap.add_argument("--out", default=os.path.join(HERE, "komp_golden.npz"))
    args = ap.parse_args()

    os.environ["TRITON_INTERPRET"] = "1"
    os.environ.setdefault("KOMP_CACHE", tempfile.mkdtemp(prefix="komp_cache_"))
    sys.path.insert(0, os.path.join(args.reference, "src"))
    sys.path.insert(0, ROOT)
    import numpy as np
    import torch
    from komp import host, kernels

    from oracle import ref

    out, manifest = {}, {"gemv": [], "source": "komp (COMP) kernels under TRITON_INTERPRET=1"}

    # quantizers
    x = ref.quant_config_input(seed=0)
    out["quant/x"] = x
    for fmt in ("q4_0", "tq2_0"):
        xq, xd = host.quantize(fmt, torch.from_numpy(x.copy()))
        out[f"quant/{ref.ACT[fmt]}/xq"] = xq.numpy()
        out[f"quant/{ref.ACT[fmt]}/xd"] = xd.numpy()

    # GEMVs
    for fmt, probs in PROBLEMS.items():
        for n, k, m in probs:
            for seed, extreme in ((1, False), (2, True)):
                cid = f"{fmt}_{n}x{k}x{m}_{'extreme' if extreme else 'random'}"
                W, xa = ref.problem(fmt, n, k, m, seed=seed, extreme=extreme)
                wq, ws = host.split(fmt, W, n, k)
                xq, xd = host.quantize(fmt, torch.from_numpy(xa.copy()))
                p = f"gemv/{cid}/"
                out[p + "W"] = np.frombuffer(W, dtype=np.uint8).copy()
                out[p + "x"] = xa
                out[p + "xq"] = xq.numpy()
                out[p + "xd"] = xd.numpy()
                for mode in (0, 1):
                    y, s = host.gemv(fmt, torch.from_numpy(wq), torch.from_numpy(ws), xq, xd, n, k, 32, 4, mode, 4,
                                     store_s=True)
                    out[p + f"y{mode}"] = y.numpy()
                    out[p + f"s{mode}"] = s.numpy()
                manifest["gemv"].append(dict(id=cid, fmt=fmt, n=n, k=k, m=m, seed=seed, extreme=extreme))
                print("gemv", cid, flush=True)

    # dp4a word mix (src/komp/verify.py:44-54)
    rng = random.Random(3)
    edge = [0, -1, 0x7F7F7F7F, -0x7F7F7F80, 0x01010101, 0x0F0F0F0F, 0x03030303, 2**31 - 1, -(2**31), 0x80000000 - 2**32]
    n = 1024
    vals = lambda: [rng.choice(edge) if rng.random() < 0.3 else rng.randrange(-(2**31), 2**31) for _ in range(n)]  # noqa: E731
    a, b = vals(), vals()
    c = [rng.randrange(-(2**20), 2**20) for _ in range(n)]
    o = torch.zeros(n, dtype=torch.int32)
    kernels.dp4a_probe[(n // 256,)](torch.tensor(a, dtype=torch.int32), torch.tensor(b, dtype=torch.int32),
                                    torch.tensor(c, dtype=torch.int32), o, MODE=1)
    out["dp4a/a"], out["dp4a/b"], out["dp4a/c"] = (np.array(v, dtype=np.int32) for v in (a, b, c))
    out["dp4a/out"] = o.numpy()

    # decode probes
    nrng = np.random.default_rng(7)
    q4 = nrng.integers(0, 256, size=(37, 16), dtype=np.uint8)
    o4 = torch.zeros((37, 32), dtype=torch.int32)
    kernels.q4_0_decode[(3,)](torch.from_numpy(q4), o4, 37)
    out["decode/q4_0/wq"], out["decode/q4_0/out"] = q4, o4.numpy()
    tq = nrng.integers(0, 256, size=(5, 64), dtype=np.uint8)  # every crumb value, 3 included
    ot = torch.zeros((5, 256), dtype=torch.int32)
    kernels.tq2_0_decode[(5,)](torch.from_numpy(tq), ot, 5)
    out["decode/tq2_0/wq"], out["decode/tq2_0/out"] = tq, ot.numpy()

    out["manifest"] = np.frombuffer(json.dumps(manifest).encode(), dtype=np.uint8)
    np.savez_compressed(args.out, **out)
    print(f"wrote {args.out} ({os.path.getsize(args.out)} bytes)")


if __name__ == "__main__":
    main()

"""Worker for tests/test_gpu_dist.py (run by torch.distributed.run, one process per GPU): row-sharded GEMVs with the
fused P2P all-gather and with NCCL, checked bit-for-bit against the unsharded GEMV of the same layer on this GPU,
over repeated calls and CUDA-graph replays, and against the C oracle (exact block dots, f64 reference dot) on sampled
rows of every rank's slice. Prints one line `RESULT <rank> ok|FAIL <details>`."""

import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from comp_b200 import host  # noqa: E402
from comp_b200.dist import RowShardedGemv, partition  # noqa: E402
from oracle import native, ref  # noqa: E402

TOL = 1e-5  # KURN's rule (src/komp/verify.py:28)


def oracle_rows(fmt, wq, ws, x, n, k, world, seed):
    """Sampled rows (up to 64 of every rank's slice, plus each slice's first and last row) and the oracle's exact
    reference Y for them, f64 [M][rows]."""
    rng = np.random.default_rng(seed)
    picks = []
    for r0, cnt in partition(n, world):
        if cnt:
            picks += [r0, r0 + cnt - 1, *rng.choice(np.arange(r0, r0 + cnt), min(cnt, 64), replace=False)]
    rows = np.unique(np.array(picks))
    oq, od = ref.quantize(fmt, x.cpu().numpy())
    r, _ = native.gemv(fmt, wq.cpu().numpy()[rows], ws.cpu().numpy()[rows], oq, od, k)
    return rows, r


def layer(fmt, n, k, dev, seed):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    nb = k // (32 if fmt == "q4_0" else 256)
    if fmt == "q4_0":
        wq = torch.randint(0, 256, (n, k // 2), dtype=torch.uint8, device=dev, generator=g)
    else:
        t = torch.randint(0, 81, (n, k // 4), dtype=torch.uint8, device=dev, generator=g)
        wq = (t % 3) | (((t // 3) % 3) << 2) | (((t // 9) % 3) << 4) | (((t // 27) % 3) << 6)
    ws = (torch.randn((n, nb), device=dev, generator=g) * 0.03).abs().half().view(torch.int16)
    return wq.contiguous(), ws.contiguous()


def main():
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=60))
    fails = []
    cases = [("q4_0", 4100, 4096, 1), ("tq2_0", 8192, 8192, 3), ("q4_0", 1000, 14336, 2), ("tq2_0", 64 * world, 2048, 1)]
    for ci, (fmt, n, k, m) in enumerate(cases):
        wq, ws = layer(fmt, n, k, dev, 100 + ci)
        g = torch.Generator(device=dev)
        g.manual_seed(200 + ci)
        x = torch.randn((m, k), device=dev, generator=g)
        want = host.quant_gemv(fmt, wq, ws, x, n, k, split=False)  # the GEMV schedule the shards run
        rows_o, r_o = oracle_rows(fmt, wq, ws, x, n, k, world, 300 + ci)
        row0, rows = partition(n, world)[rank]
        shard = (wq[row0 : row0 + rows].contiguous(), ws[row0 : row0 + rows].contiguous())
        for exchange in ("p2p", "nccl"):
            L = RowShardedGemv(fmt, *shard, n, k, exchange=exchange)
            for t in range(3):
                y = L(x).clone()
                if not torch.equal(y.view(torch.int32), want.view(torch.int32)):
                    fails.append(f"{fmt} {n}x{k} m={m} {exchange} call {t}: max diff {(y - want).abs().max().item()}")
                err = ref.relerr(y.cpu().numpy()[:, rows_o], r_o)
                if not err <= TOL:
                    fails.append(f"{fmt} {n}x{k} m={m} {exchange} call {t}: relerr {err:.2e} vs the oracle")
            # host buffers: pinned x copied in by a kernel, Y stored into pinned host memory (two calls in a row)
            xh = x.cpu().pin_memory()
            outs = [torch.full((m, n), float("nan")).pin_memory() for _ in range(2)]
            for o in outs:
                if L(xh, out=o) is not o:
                    fails.append(f"{fmt} {n}x{k} {exchange} pinned: out not returned")
            torch.cuda.current_stream(dev).synchronize()
            for t, o in enumerate(outs):
                if not torch.equal(o.view(torch.int32), want.cpu().view(torch.int32)):
                    fails.append(f"{fmt} {n}x{k} m={m} {exchange} pinned call {t}: mismatch")
            if L.exchange == "p2p":
                # capture two calls (both output buffers) in a graph and replay it
                s = torch.cuda.Stream(dev)
                s.wait_stream(torch.cuda.current_stream(dev))
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.stream(s):
                    with torch.cuda.graph(graph, stream=s):
                        ya = L(x)
                        yb = L(x)
                torch.cuda.current_stream(dev).wait_stream(s)
                for _ in range(3):
                    graph.replay()
                torch.cuda.synchronize(dev)
                for name, yy in (("graph a", ya), ("graph b", yb)):
                    if not torch.equal(yy.view(torch.int32), want.view(torch.int32)):
                        fails.append(f"{fmt} {n}x{k} {name}: mismatch")
                del graph, ya, yb
                if L.status_code() != 0:
                    fails.append(f"{fmt} {n}x{k} barrier status {L.status_code()}")
            L.close()
    torch.cuda.synchronize(dev)
    dist.barrier()
    print(f"\nRESULT {rank} {'ok' if not fails else 'FAIL ' + '; '.join(fails)}", flush=True)
    dist.destroy_process_group()
    sys.exit(1 if fails else 0)


if __name__ == "__main__":
    main()

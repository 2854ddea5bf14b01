"""Benchmark of the quantized decode path on B200: weight-stream GB/s and us per GEMV (fraction of HBM peak).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload config4] [--impl ours|reference]

One step = one pass of the hot path over every layer of the workload, M = 1 activation column: quantize the f32
activation (q8_0 for Q4_0 layers, q8_K for TQ2_0 layers) and run the GEMV. Default workload = BASELINE config 4 (the
largest single-GPU configuration, quoted at 1/2/4/8 GPUs): TQ2_0 gate_up 57344x8192, TQ2_0 down 8192x28672, Q4_0
lm_head 128256x8192 -- 773 MB of weights, > 6x the 126 MB L2, so every step streams the weights from HBM (no flush).

Metric units: algorithmic bytes per GEMV = N*K*(18/32 | 66/256) weights + M*(K + 4*K/blk) q8 activations + 4*M*N
output; value = sum over layers / step time. Weights random-initialised with the BASELINE distributions (synthetic).

N > 1 (torchrun, one process per GPU): every layer is row-sharded across the ranks (strong scaling: the same layers at
every N); each rank runs its rows, then the output slices are all-gathered so every rank holds the full Y.

End to end (the "e2e" key): the same layers through the public API with host buffers, every step -- pinned host x
in, Y stored into pinned host memory by the kernels, a host stream synchronize (N = 1: b2q_quant_gemv_pinned per
layer; N > 1: RowShardedGemv(x_host, out=y_host)); --e2e-api device uses device buffers with torch memcpys instead.

--impl reference: the reference's CPU path (the C + OpenMP restatement of COMP's quantizers and KURN's reference dot,
oracle/c/oracle.c, all host threads) on the same workload; rank 0 only.
"""

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

WORKLOADS = {
    "config4": [("tq2_0", 57344, 8192, "gate_up"), ("tq2_0", 8192, 28672, "down"), ("q4_0", 128256, 8192, "lm_head")],
    "config3": [("q4_0", 6144, 4096, "qkv"), ("q4_0", 4096, 4096, "o_proj"), ("q4_0", 28672, 4096, "gate_up"),
                ("q4_0", 4096, 14336, "down")],
    "config0": [("q4_0", 4096, 4096, "config0")],
    "config1": [("tq2_0", 4096, 4096, "config1")],
    # Q8_0 weights (an extension beyond the reference): the config-3 decoder shapes plus the lm_head, all Q8_0
    "q8_0": [("q8_0", 6144, 4096, "qkv"), ("q8_0", 4096, 4096, "o_proj"), ("q8_0", 28672, 4096, "gate_up"),
             ("q8_0", 4096, 14336, "down"), ("q8_0", 128256, 4096, "lm_head")],
    # IQ4_NL weights (a second extension): the same shapes, all IQ4_NL
    "iq4_nl": [("iq4_nl", 6144, 4096, "qkv"), ("iq4_nl", 4096, 4096, "o_proj"), ("iq4_nl", 28672, 4096, "gate_up"),
               ("iq4_nl", 4096, 14336, "down"), ("iq4_nl", 128256, 4096, "lm_head")],
}
BLOCK = {"q4_0": 32, "tq2_0": 256, "q8_0": 32, "iq4_nl": 32}
BLOCK_BYTES = {"q4_0": 18, "tq2_0": 66, "q8_0": 34, "iq4_nl": 18}  # ggml block bytes (quant bytes + f16 scale)
FMT_ID = {"q4_0": 0, "tq2_0": 1, "q8_0": 2, "iq4_nl": 3}
METRIC = "weight-stream GB/s and us/GEMV (% of HBM peak) at 1/2/4/8 B200 vs host CPU ref"
L2_BYTES = 126 * 2**20


def weight_bytes(fmt, n, k):
    return n * k * BLOCK_BYTES[fmt] // BLOCK[fmt]


def algo_bytes(fmt, n, k, m):
    """Algorithmic bytes of one GEMV: weights once, q8 activations, f32 output (the S dump is excluded)."""
    return weight_bytes(fmt, n, k) + m * (k + 4 * k // BLOCK[fmt]) + 4 * m * n


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
            p = json.load(fh)
        return float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def profiled_traffic(kernel_tag):
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary (profiles/*.md), or None."""
    d = os.path.join(ROOT, "profiles")
    if not os.path.isdir(d):
        return None
    for f in sorted(os.listdir(d)):
        if not f.endswith(".md"):
            continue
        for line in open(os.path.join(d, f)):
            if line.startswith(f"traffic_bytes_per_launch[{kernel_tag}]:"):
                try:
                    return int(line.split(":", 1)[1].strip().split()[0])
                except ValueError:
                    return None
    return None


class ClockSampler:
    """Polls NVML (SM clock, max SM clock, throttle reasons) on a thread while the timed region runs."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4,
               "hw_power_brake_slowdown": 0x80}

    def __init__(self, dev, period=0.005):
        self.period = period
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._t = None
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            self.nv = pynvml
            pr = torch.cuda.get_device_properties(dev)
            try:  # the CUDA ordinal may be remapped (CUDA_VISIBLE_DEVICES): find the GPU by PCI address
                bus = f"{pr.pci_domain_id:08X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0"
                self.h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:  # noqa: BLE001
                self.h = pynvml.nvmlDeviceGetHandleByIndex(dev.index or 0)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:  # noqa: BLE001 -- clocks are reported as unavailable, never fatal
            self.nv = None

    def _poll(self):
        sm = self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)
        r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
        self.samples.append(sm)
        for name, bit in self.REASONS.items():
            if r & bit:
                self.reasons.add(name)

    def _run(self):
        while not self._stop.is_set():
            try:
                self._poll()
            except Exception:  # noqa: BLE001
                return
            time.sleep(self.period)

    def __enter__(self):
        if self.nv:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join()
            try:
                self._poll()  # at least one sample at the end of the region
            except Exception:  # noqa: BLE001
                pass

    def summary(self):
        if not self.nv:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"], "samples": 0}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ---------------------------------------------------------------------------------------------------------------
# synthetic layers
# ---------------------------------------------------------------------------------------------------------------


def make_layer_gpu(fmt, n, k, seed, dev, rows=None):
    """Split planes with the BASELINE distributions, generated on the GPU (torch RNG, seeded); rows=(row0, count)
    keeps only that row slice."""
    import torch

    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    nb = k // BLOCK[fmt]
    if fmt in ("q4_0", "iq4_nl"):
        wq = torch.randint(0, 256, (n, k // 2), dtype=torch.uint8, device=dev, generator=g)
        sd = 0.02 if fmt == "q4_0" else 0.002
        ws = (torch.randn((n, nb), device=dev, generator=g) * sd).abs().half().view(torch.int16)
    elif fmt == "q8_0":
        wq = torch.randint(-127, 128, (n, k), dtype=torch.int8, device=dev, generator=g).view(torch.uint8)
        ws = (torch.randn((n, nb), device=dev, generator=g) * 0.002).abs().half().view(torch.int16)
    else:
        t = torch.randint(0, 81, (n, k // 4), dtype=torch.uint8, device=dev, generator=g)
        wq = (t % 3) | (((t // 3) % 3) << 2) | (((t // 9) % 3) << 4) | (((t // 27) % 3) << 6)
        ws = (torch.randn((n, nb), device=dev, generator=g) * 0.05).abs().half().view(torch.int16)
        del t
    if rows is not None:
        r0, cnt = rows
        wq, ws = wq[r0 : r0 + cnt].clone(), ws[r0 : r0 + cnt].clone()
    return wq.contiguous(), ws.contiguous()


def make_x(k, m, seed):
    rng = np.random.default_rng(seed)
    return rng.standard_normal((m, k)).astype(np.float32)


# ---------------------------------------------------------------------------------------------------------------
# CPU reference path (oracle/c/oracle.c) -- the reference arm and the cpu_baseline leg
# ---------------------------------------------------------------------------------------------------------------


def cpu_reference_run(layers_np, steps, warmup):
    """Times quantize + GEMV of the C/OpenMP restatement on host cores. Returns (seconds per step, threads)."""
    from oracle import native

    threads = native.max_threads()

    def one():
        for fmt, wq, ws, x, k in layers_np:
            if fmt in ("q4_0", "q8_0"):
                xq, xd = native.quant_q8_0(x)
            else:
                xq, xd, _ = native.quant_q8_K(x)
            native.gemv(fmt, wq, ws, xq, xd, k)

    for _ in range(warmup):
        one()
    t0 = time.perf_counter()
    for _ in range(steps):
        one()
    return (time.perf_counter() - t0) / steps, threads


def cpu_layers(workload, m, budget_rows=None):
    """Host copies of the workload's layers for the CPU path; budget_rows limits each layer to its first rows."""
    import torch

    out, meta = [], []
    for i, (fmt, n, k, name) in enumerate(WORKLOADS[workload]):
        rows = n if budget_rows is None else min(n, budget_rows)
        rng = np.random.default_rng(100 + i)
        from oracle import ref

        wq, ws = ref.random_split(fmt, rng, rows, k)
        out.append((fmt, wq, ws, make_x(k, m, 200 + i), k))
        meta.append((fmt, rows, k))
    del torch
    return out, meta


def run_reference_arm(args, rank):
    if rank != 0:
        return
    m = args.m
    full = WORKLOADS[args.workload]
    full_bytes = sum(algo_bytes(f, n, k, m) for f, n, k, _ in full)
    # bound the run: a step is a row sample sized so warmup + steps stay within ~90 s of host time
    probe_layers, _ = cpu_layers(args.workload, m, budget_rows=512)
    probe_s, _ = cpu_reference_run(probe_layers, 1, 1)
    probe_bytes = sum(algo_bytes(f, 512 if n > 512 else n, k, m) for f, n, k, _ in full)
    est_full = probe_s * full_bytes / probe_bytes
    budget = 90.0 / max(1, args.steps + args.warmup)
    frac = min(1.0, budget / est_full) if est_full > 0 else 1.0
    rows = max(64, int(max(n for _, n, _, _ in full) * frac))
    layers, meta = cpu_layers(args.workload, m, budget_rows=rows)
    step_bytes = sum(algo_bytes(f, r, k, m) for f, r, k in meta)
    sec, threads = cpu_reference_run(layers, args.steps, args.warmup)
    gbs = step_bytes / sec / 1e9
    full_rows = all(r == n for (f, r, k), (_, n, _, _) in zip(meta, full))
    what = "full layers" if full_rows else f"first {rows} rows of each layer"
    sample = (f"{what} ({', '.join(f'{f} {r}x{k}' for f, r, k in meta)}), M={m}; quantize + GEMV + f64 reference dot "
              f"per layer, each step")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(sec * 1e3 * full_bytes / step_bytes, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8/int32 dots, f64 sum",
        "data": "synthetic (BASELINE distributions, seeded)",
        "config": {"workload": args.workload, "layers": [f"{f} {n}x{k}" for f, n, k, _ in full], "m": m,
                   "parallelism": "host cores"},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ---------------------------------------------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------------------------------------------


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--workload", default="config4", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--m", type=int, default=1, help="activation columns")
    ap.add_argument("--e2e-steps", type=int, default=None, help="steps of the end-to-end leg (default: --steps)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end leg (profiling runs)")
    ap.add_argument("--layers", default=None, help="comma-separated layer names of the workload to keep (profiling)")
    ap.add_argument("--exchange", default="p2p", choices=["p2p", "nccl"], help="N > 1 output all-gather")
    ap.add_argument("--pdl", default="on", choices=["on", "off"], help="programmatic dependent launch of the GEMVs")
    ap.add_argument("--e2e-api", default="pinned", choices=["pinned", "device"],
                    help="end-to-end leg: pinned host x in and Y stored into pinned host memory by the kernels "
                         "(N = 1: b2q_quant_gemv_pinned, N > 1: RowShardedGemv(x_host, out=y_host)), or device "
                         "buffers with torch memcpys around each call")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference_arm(args, rank)
        return

    import datetime

    import torch
    import torch.distributed as dist

    from comp_b200 import _lib, host
    from comp_b200.dist import RowShardedGemv, partition

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    lib = _lib.load()
    if args.pdl == "off":
        _lib.call("b2q_set_pipeline", 4, 0)
    m = args.m
    layers_def = WORKLOADS[args.workload]
    if args.layers:
        keep = set(args.layers.split(","))
        layers_def = [d for d in layers_def if d[3] in keep]
        if not layers_def:
            ap.error(f"--layers {args.layers}: no such layer in {args.workload}")
    total_bytes = sum(algo_bytes(f, n, k, m) for f, n, k, _ in layers_def)
    weights_total = sum(weight_bytes(f, n, k) for f, n, k, _ in layers_def)
    # every step must stream its weights from HBM: keep >= 4x L2 of distinct weights per GPU, rotating copies
    per_gpu = max(1, weights_total // world)
    copies = 1 if per_gpu >= 4 * L2_BYTES else -(-4 * L2_BYTES // per_gpu)

    class Layer:
        pass

    layers = []
    for i, (fmt, n, k, name) in enumerate(layers_def):
        L = Layer()
        L.fmt, L.n, L.k, L.name = fmt, n, k, name
        L.row0, L.rows = partition(n, world)[rank]
        L.w = [make_layer_gpu(fmt, n, k, 100 + i + 1000 * c, dev, rows=(L.row0, L.rows)) for c in range(copies)]
        L.x_host = torch.from_numpy(make_x(k, m, 200 + i)).pin_memory()
        L.x = L.x_host.to(dev)
        L.y = torch.empty((m, n), dtype=torch.float32, device=dev)
        L.fid = FMT_ID[fmt]
        L.wsb = host.workspace_size(fmt, n, k, m) if world == 1 else 0
        L.work = torch.empty(max(16, L.wsb), dtype=torch.uint8, device=dev)
        if world > 1:
            L.objs = [RowShardedGemv(fmt, wq, ws, n, k, exchange=args.exchange) for wq, ws in L.w]
        layers.append(L)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    sptr = stream.cuda_stream
    dominant = max(range(len(layers)), key=lambda i: weight_bytes(layers[i].fmt, layers[i].n, layers[i].k))
    exchange_name = None if world == 1 else layers[0].objs[0].exchange

    def launch(L, c):
        """N = 1: fused quantize + GEMV straight through the C ABI (tall-K layers: split-K, two launches)."""
        wq, ws = L.w[c]
        rc = lib.b2q_quant_gemv_ws(L.fid, wq.data_ptr(), wq.stride(0), ws.data_ptr(), L.x.data_ptr(), L.x.stride(0),
                                   None, None, L.y.data_ptr(), L.rows, L.k, m, L.work.data_ptr(), L.wsb, sptr)
        if rc != 0:
            raise RuntimeError(_lib.last_error())

    def step(c, ev=None):
        for i, L in enumerate(layers):
            if ev is not None and i == dominant:
                ev[0].record(stream)
            if world == 1:
                launch(L, c)
            else:
                L.objs[c](L.x)
            if ev is not None and i == dominant:
                ev[1].record(stream)

    for w in range(args.warmup):
        step(w % copies)
    torch.cuda.synchronize()

    # N > 1: the step is captured once per weight copy as a CUDA graph (three fused GEMV + all-gather launches, or
    # GEMV + NCCL all-gather), so host launch time does not bound the multi-GPU step
    graphs = []
    launches_per_graph = 0
    if world > 1:
        cs = torch.cuda.Stream(dev)
        cs.wait_stream(stream)
        for c in range(copies):
            graphs.append(torch.cuda.CUDAGraph())
            n0 = _lib.launch_count()
            with torch.cuda.stream(cs), torch.cuda.graph(graphs[-1], stream=cs):
                step(c)
            launches_per_graph = _lib.launch_count() - n0
        stream.wait_stream(cs)
        for c in range(copies):
            graphs[c].replay()
        torch.cuda.synchronize()
        dist.barrier()

    # ---- device-timed region: inputs resident in HBM ----
    dom_events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                  for _ in range(args.steps if world == 1 else 0)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = _lib.launch_count()
    with ClockSampler(dev) as clocks:
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        start.record(stream)
        for s in range(args.steps):
            if world == 1:
                step(s % copies, dom_events[s])
            else:
                graphs[s % copies].replay()
        end.record(stream)
        end.synchronize()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    launches = _lib.launch_count() - launches0 if world == 1 else launches_per_graph * args.steps
    ms = start.elapsed_time(end)
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    sec = ms / 1e3
    value = total_bytes * args.steps / sec / 1e9
    dom = layers[dominant]
    if world == 1:
        dom_ms = statistics.mean(a.elapsed_time(b) for a, b in dom_events)
        dom_note = "mean CUDA-event duration of its launches inside the timed steps"
    else:
        # the dominant layer alone (its fused GEMV + all-gather), graph-replayed, event-timed on its stream
        dg = []
        cs2 = torch.cuda.Stream(dev)
        cs2.wait_stream(stream)
        for c in range(copies):
            dg.append(torch.cuda.CUDAGraph())
            with torch.cuda.stream(cs2), torch.cuda.graph(dg[-1], stream=cs2):
                dom.objs[c](dom.x)
        stream.wait_stream(cs2)
        reps = max(20, min(400, args.steps))
        for r in range(4):
            dg[r % copies].replay()
        torch.cuda.synchronize()
        dist.barrier()
        d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        d0.record(stream)
        for r in range(reps):
            dg[r % copies].replay()
        d1.record(stream)
        d1.synchronize()
        td = torch.tensor([d0.elapsed_time(d1) / reps], dtype=torch.float64, device=dev)
        dist.all_reduce(td, op=dist.ReduceOp.MAX)
        dom_ms = float(td.item())
        dom_note = f"dominant layer alone, {reps} graph replays after the timed steps, max over ranks"
        dg.clear()
        del dg
        for L in layers:
            for o in L.objs:
                if o.status_code() != 0:
                    raise RuntimeError(f"rank {rank}: all-gather barrier timed out ({o.status_code()})")
    dom_bytes = algo_bytes(dom.fmt, dom.rows, dom.k, m)
    peak, peak_kind = peaks()
    achieved = dom_bytes / (dom_ms / 1e3) / 1e9
    tag = f"{dom.fmt}_{dom.rows}x{dom.k}"
    traffic = profiled_traffic(tag)

    # ---- end to end through the public API: pinned host x -> device, quantize + gemv, Y -> host ----
    e2e_steps = 0 if args.no_e2e else (args.e2e_steps or args.steps)
    y_host = [torch.empty((m, L.n), dtype=torch.float32).pin_memory() for L in layers]

    y_dev = [torch.empty((m, L.n), dtype=torch.float32, device=dev) for L in layers] if world == 1 else None
    pinned = args.e2e_api == "pinned"
    if pinned and world == 1:
        pin_ws = [torch.empty(max(256, host.pinned_workspace_size(L.fmt, L.n, L.k, m)), dtype=torch.uint8,
                              device=dev) for L in layers]

    def e2e_step_pinned():
        # every step, one call per layer with host buffers: a copy kernel pulls the layer's x from pinned host memory,
        # the fused GEMV (N > 1: with the all-gather) stores Y into pinned host memory; the host then waits and reads
        # the results
        for i, L in enumerate(layers):
            if world > 1:
                L.objs[0](L.x_host, out=y_host[i])
                continue
            wq, ws = L.w[0]
            rc = lib.b2q_quant_gemv_pinned(L.fid, wq.data_ptr(), wq.stride(0), ws.data_ptr(), L.x_host.data_ptr(),
                                           L.x_host.stride(0), y_host[i].data_ptr(), L.n, L.k, m,
                                           pin_ws[i].data_ptr(), pin_ws[i].numel(), sptr)
            if rc != 0:
                raise RuntimeError(_lib.last_error())
        stream.synchronize()  # the step's results are read on the host

    def e2e_step():
        if pinned:
            return e2e_step_pinned()
        # every step: the layers' inputs from pinned host memory, the GEMVs back to back through the public API (so
        # each one's weight stream can start while the previous one finishes), every layer's output back to pinned
        # host memory, then the host waits for all of it
        xs = [L.x_host.to(dev, non_blocking=True) for L in layers]
        ys = []
        for i, L in enumerate(layers):
            if world == 1:
                wq, ws = L.w[0]
                ys.append(host.quant_gemv(L.fmt, wq, ws, xs[i], L.n, L.k, out=y_dev[i]))
            else:
                # the fused exchange reuses its output buffer on the layer's next call
                ys.append(L.objs[0](xs[i]) if i + 1 == len(layers) else L.objs[0](xs[i]).clone())
        for i, y in enumerate(ys):
            y_host[i].copy_(y, non_blocking=True)
        stream.synchronize()  # the step's results are read on the host

    e2e_gbs = None
    if e2e_steps:
        for _ in range(3):
            e2e_step()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(e2e_steps):
            e2e_step()
        e1.record(stream)
        e1.synchronize()
        te = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e_gbs = round(total_bytes * e2e_steps / (float(te.item()) / 1e3) / 1e9, 3)
    h2d = sum(L.x_host.numel() * 4 for L in layers)
    d2h = sum(L.n * m * 4 for L in layers)
    # graphs that hold NCCL calls must be released before the process group is destroyed
    graphs.clear()
    del graphs
    torch.cuda.synchronize()
    if world > 1:
        for L in layers:
            for o in L.objs:
                o.close()

    # ---- CPU baseline (rank 0, N = 1): bounded sample of the same workload ----
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rows = 8192
        cl, meta = cpu_layers(args.workload, m, budget_rows=rows)
        csec, threads = cpu_reference_run(cl, 3, 1)
        cbytes = sum(algo_bytes(f, r, k, m) for f, r, k in meta)
        cpu = {"value": round(cbytes / csec / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
               "sample": f"first {rows} rows of each layer, M={m}, 3 steps of quantize + GEMV + f64 reference dot "
                         f"(oracle/c/oracle.c, OpenMP)"}

    # the dominant layer runs as quantizer + tensor-core GEMM when it has 8+ columns and a workspace for them
    L_tc = world == 1 and m >= 8 and getattr(layers[dominant], "wsb", 0) > 0
    if rank == 0:
        cs = clocks.summary()
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8 dp4a dots, f32 scale+sum",
            "data": "synthetic (BASELINE distributions, seeded, random-init weights)",
            "config": {"workload": args.workload, "layers": [f"{f} {n}x{k} ({nm})" for f, n, k, nm in layers_def],
                       "m": m, "parallelism": f"row-shard x{world}" if world > 1 else "single GPU",
                       "exchange": {None: None, "p2p": "fused all-gather: (value, flag) peer stores from the GEMV epilogue",
                                    "nccl": "NCCL all_gather_into_tensor"}[exchange_name],
                       "graph": world > 1, "pdl": args.pdl,
                       "l2": f"weights {per_gpu / 2**20:.0f} MiB per GPU x {copies} rotating copies >= 4x L2 "
                             f"(no flush needed)"},
            "us_per_gemv": round(ms * 1e3 / args.steps / len(layers), 3),
            "hbm_frac": round(value / world / peak, 4),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic,
                         "kernel": (f"quantizer + tcgen05 GEMM {tag} (2 launches, timed together)" if L_tc else
                                    f"gemv {tag} (quant prologue fused{', all-gather fused' if world > 1 else ''})"),
                         "timing": dom_note, "peak_source": f"{peak_kind} hbm_gbs",
                         "us_per_launch": round(dom_ms * 1e3, 3), "algorithmic_bytes_per_launch": dom_bytes},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_gbs, "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "steps": e2e_steps,
                    "api": ("C-ABI b2q_quant_gemv_pinned per layer (pinned host x in, the kernels copy x in and store "
                            "Y into pinned host memory; host sync every step)" if pinned else
                            "comp_b200.host.quant_gemv (fused quantize + GEMV per layer; torch memcpy of x in, Y out)")
                    if world == 1 else f"comp_b200.dist.RowShardedGemv ({exchange_name}" +
                    ("; pinned host x in, Y stored into pinned host memory)" if pinned else
                     "; torch memcpy of x in, Y out)")},
            "gpu_launches": launches,
            "clocks": cs,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

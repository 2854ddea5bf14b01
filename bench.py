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

Also in the line:
  per_layer  every layer alone, launched back to back over rotating weight copies (>= 4x L2 of distinct weights),
             event-timed on the launching stream (max over ranks): us per GEMV, GB/s, fraction of the HBM peak.
  parity     N = 1: the first 512 rows of every layer against the C oracle (quantized bytes and int32 block dots
             bit-exact, Y within 1e-5 of the exact reference), inside the CPU-baseline leg. N > 1: every rank's
             gathered Y of every layer bit-identical to the unsharded GEMV of the full layer on its own GPU.
  e2e        the same layers through the public API with host buffers, every step -- pinned host x in, Y stored into
             pinned host memory by the kernels, a host stream synchronize (N = 1: b2q_quant_gemv_pinned per layer;
             N > 1: RowShardedGemv(x_host, out=y_host)); --e2e-api device uses device buffers with torch memcpys.
  e2e_dropin N = 1: COMP's own call sequence, host.quantize + host.gemv (the reference's signatures), x copied in
             from pinned host memory and Y copied back every step.
  clocks     NVML sampled every millisecond during the timed region (the count of samples inside it is given).
  sustained  >= 1 s of the same steps after the per-layer timing, event-timed, with its own NVML record: the rate
             once the 1 kW power cap has acted (the timed region itself is short and starts from cool clocks).

--impl reference: the reference's CPU path on the same workload, rank 0 only: the C + OpenMP restatement of COMP's
quantizers and KURN's reference dot (oracle/c/oracle.c, all host cores) is the line's value; next to it COMP itself
(baseline/_ref, installed by baseline/install_ref.sh) under TRITON_INTERPRET=1 on a row sample, extrapolated, and
COMP's Triton kernels JIT-compiled on this B200 (best of the spec tune space) as the GPU bar.
"""

import argparse
import json
import os
import statistics
import subprocess
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
    # Q4_K weights (a third extension): the same shapes, all Q4_K
    "q4_k": [("q4_k", 6144, 4096, "qkv"), ("q4_k", 4096, 4096, "o_proj"), ("q4_k", 28672, 4096, "gate_up"),
             ("q4_k", 4096, 14336, "down"), ("q4_k", 128256, 4096, "lm_head")],
}
BLOCK = {"q4_0": 32, "tq2_0": 256, "q8_0": 32, "iq4_nl": 32, "q4_k": 256}
# ggml block bytes (quant bytes + scales); Q4_K's split planes carry 148 bytes per block (4 more than ggml's 144: the
# scale record unpacked), and only ggml's 144 count as algorithmic bytes
BLOCK_BYTES = {"q4_0": 18, "tq2_0": 66, "q8_0": 34, "iq4_nl": 18, "q4_k": 144}
FMT_ID = {"q4_0": 0, "tq2_0": 1, "q8_0": 2, "iq4_nl": 3, "q4_k": 4}
METRIC = "weight-stream GB/s and us/GEMV (% of HBM peak) at 1/2/4/8 B200 vs host CPU ref"
L2_BYTES = 126 * 2**20
TOL = 1e-5  # KURN's relative-error rule (src/komp/verify.py:28)
REF_DIR = os.path.join(ROOT, "baseline", "_ref")
# COMP's spec tune space per weight format (block_n, nb), mode dp4a, 4 warps (examples/*_gemv_triton.kurn)
KOMP_TUNE = {"q4_0": [(32, 4), (32, 8), (64, 4), (64, 8)], "tq2_0": [(32, 1), (32, 2), (64, 1), (64, 2)]}


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


def select_layers(args):
    layers_def = WORKLOADS[args.workload]
    if args.layers:
        keep = set(args.layers.split(","))
        layers_def = [d for d in layers_def if d[3] in keep]
    return layers_def


def bench_config(workload, layers_def, m):
    """The workload as both arms name it (the same dict, so the two lines compare)."""
    return {"workload": workload, "layers": [f"{f} {n}x{k} ({nm})" for f, n, k, nm in layers_def], "m": m,
            "l2": "inputs larger than L2: >= 4x the 126 MiB L2 of distinct weights per GPU per step (rotating "
                  "copies where a GPU's share is smaller), no flush"}


class ClockSampler:
    """Polls NVML (SM clock, max SM clock, throttle reasons) on a thread; mark() brackets the timed region so the
    summary can say how many samples fell inside it."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20, "sw_power_cap": 0x4,
               "hw_power_brake_slowdown": 0x80}

    def __init__(self, dev, period=0.005):
        self.period = period
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self.t_begin = self.t_end = None
        self._stop = threading.Event()
        self._t = None
        self._t0 = None
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
        self.samples.append((time.perf_counter(), sm))
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

    def mark(self, begin):
        if begin:
            self.t_begin = time.perf_counter()
        else:
            self.t_end = time.perf_counter()

    def __enter__(self):
        self._t0 = time.perf_counter()
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
        mhz = [s for _, s in self.samples]
        timed = [s for t, s in self.samples if self.t_begin is not None and self.t_begin <= t <= (self.t_end or t)]
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(mhz), "samples_in_timed_region": len(timed),
                "sm_mhz_timed_region": statistics.median(timed) if timed else None,
                "window_s": round(time.perf_counter() - self._t0, 3) if self._t0 else None,
                "period_ms": self.period * 1e3}


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
    elif fmt == "q4_k":  # the split planes: nibbles, and 20-byte records (f16 d, f16 dmin, sc/m bytes 0..63)
        wq = torch.randint(0, 256, (n, k // 2), dtype=torch.uint8, device=dev, generator=g)
        rec = torch.empty((n, nb, 20), dtype=torch.uint8, device=dev)
        rec[:, :, 0:2] = (torch.randn((n, nb), device=dev, generator=g) * 0.002).abs().half().view(torch.uint8) \
            .reshape(n, nb, 2)
        rec[:, :, 2:4] = (torch.randn((n, nb), device=dev, generator=g) * 0.004).abs().half().view(torch.uint8) \
            .reshape(n, nb, 2)
        rec[:, :, 4:] = torch.randint(0, 64, (n, nb, 16), dtype=torch.uint8, device=dev, generator=g)
        ws = rec.reshape(n, nb * 20).view(torch.int16)
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


def copies_for(nbytes):
    """Rotating copies so that a loop over them streams >= 4x L2 of distinct weights."""
    return 1 if nbytes >= 4 * L2_BYTES else -(-4 * L2_BYTES // max(1, nbytes))


# ---------------------------------------------------------------------------------------------------------------
# CPU reference path (oracle/c/oracle.c) -- the reference arm and the cpu_baseline leg
# ---------------------------------------------------------------------------------------------------------------


def cpu_reference_run(layers_np, steps, warmup):
    """Times quantize + GEMV of the C/OpenMP restatement on host cores. Returns (seconds per step, threads)."""
    from oracle import native

    threads = native.max_threads()

    def one():
        for fmt, wq, ws, x, k in layers_np:
            if fmt in ("q4_0", "q8_0", "iq4_nl"):
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


def cpu_layers(layers_def, m, budget_rows=None):
    """Host copies of the workload's layers for the CPU path; budget_rows limits each layer to its first rows."""
    from oracle import ref

    out, meta = [], []
    for i, (fmt, n, k, name) in enumerate(layers_def):
        rows = n if budget_rows is None else min(n, budget_rows)
        rng = np.random.default_rng(100 + i)
        wq, ws = ref.random_split(fmt, rng, rows, k)
        out.append((fmt, wq, ws, make_x(k, m, 200 + i), k))
        meta.append((fmt, rows, k))
    return out, meta


def _komp_env():
    env = dict(os.environ)
    env["KOMP_PATCHES"] = os.path.join(REF_DIR, "patches")
    env.setdefault("KOMP_CACHE", os.path.join(ROOT, "gpurun_out", "komp_cache"))
    env["PYTHONPATH"] = REF_DIR + os.pathsep + env.get("PYTHONPATH", "")
    return env


def _run_komp_worker(kind, args, timeout, extra=()):
    """Runs `bench.py --komp-worker kind` (the reference's own code from baseline/_ref) in a subprocess, because
    TRITON_INTERPRET must be set (interpreter) or unset (compiled kernels) before triton is imported. Returns the
    worker's JSON dict, or {"unavailable": reason}."""
    if not os.path.exists(os.path.join(REF_DIR, "komp", "host.py")) or \
            not os.path.exists(os.path.join(REF_DIR, "patches", "0001-language-extra-kurn.patch")):
        return {"unavailable": "the reference is not installed under baseline/_ref (run baseline/install_ref.sh)"}
    env = _komp_env()
    if kind == "interp":
        env["TRITON_INTERPRET"] = "1"
    else:
        env.pop("TRITON_INTERPRET", None)
    cmd = [sys.executable, os.path.abspath(__file__), "--komp-worker", kind, "--workload", args.workload,
           "--m", str(args.m), *extra]
    if args.layers:
        cmd += ["--layers", args.layers]
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout, env=env, cwd=ROOT)
    except subprocess.TimeoutExpired:
        return {"unavailable": f"komp {kind} worker did not finish within {timeout} s"}
    for line in reversed(r.stdout.strip().splitlines()):
        if line.startswith("{"):
            return json.loads(line)
    tail = (r.stderr.strip().splitlines() or ["no output"])[-1]
    return {"unavailable": f"komp {kind} worker exited {r.returncode}: {tail[:300]}"}


def komp_interp_worker(args):
    """COMP itself on the host cores: host.quantize + host.gemv (mode 1, the interpreter's dp4a) under
    TRITON_INTERPRET=1 on the first rows of each layer; the GEMV time is scaled to the full layer (each row is an
    independent program of the same cost), the quantizer (one pass over K) is timed whole."""
    import torch
    from komp import host as khost

    from oracle import ref  # the reference arm's data generator (seeded split planes)

    rows = args.komp_rows
    m = args.m
    # one small call first: module imports and the interpreter's first-use costs stay out of the timing
    wq, ws = ref.random_split("q4_0", np.random.default_rng(0), 4, 64)
    xq, xd = khost.quantize("q4_0", torch.from_numpy(make_x(64, 1, 0)))
    khost.gemv("q4_0", torch.from_numpy(wq), torch.from_numpy(ws), xq, xd, 4, 64, mode=1)
    per = []
    step_s = 0.0
    for i, (fmt, n, k, name) in enumerate(select_layers(args)):
        r = min(n, rows)
        wq, ws = ref.random_split(fmt, np.random.default_rng(100 + i), r, k)
        x = torch.from_numpy(make_x(k, m, 200 + i))
        t0 = time.perf_counter()
        xq, xd = khost.quantize(fmt, x)
        t1 = time.perf_counter()
        khost.gemv(fmt, torch.from_numpy(wq), torch.from_numpy(ws), xq, xd, r, k, mode=1)
        t2 = time.perf_counter()
        full = (t1 - t0) + (t2 - t1) * n / r
        step_s += full
        per.append({"name": name, "rows_run": r, "quant_s": round(t1 - t0, 4), "gemv_s": round(t2 - t1, 4),
                    "full_layer_s_extrapolated": round(full, 3)})
    total = sum(algo_bytes(f, n, k, m) for f, n, k, _ in select_layers(args))
    print(json.dumps({"value": total / step_s / 1e9, "unit": "GB/s", "cores": 1, "kind": "reference",
                      "extrapolated": True, "step_s_extrapolated": round(step_s, 2), "per_layer": per,
                      "torch_threads": torch.get_num_threads(),
                      "sample": f"COMP (baseline/_ref) host.quantize + host.gemv mode 1 under TRITON_INTERPRET=1 on the "
                                f"first {rows} rows of each layer, GEMV time scaled by N/rows; the interpreter runs "
                                f"the grid's programs one after another in one Python thread"}), flush=True)


def komp_triton_worker(args):
    """COMP's Triton kernels JIT-compiled for this B200 (mode 2, dp4a in inline PTX): per layer, the best of the spec
    tune space, quantize + GEMV captured in a CUDA graph per rotating weight copy and replayed, event-timed. Only the
    reference's code runs here (its outputs are compared with this library's in tests/test_gpu_vs_komp.py)."""
    import torch
    from komp import host as khost

    dev = torch.device("cuda", args.device)
    torch.cuda.set_device(dev)
    m = args.m
    peak, _ = peaks()
    per, step_us, notes = [], 0.0, []
    for i, (fmt, n, k, name) in enumerate(select_layers(args)):
        if fmt not in KOMP_TUNE:
            per.append({"name": name, "unavailable": f"COMP has no {fmt} kernel"})
            continue
        wq0, ws0 = make_layer_gpu(fmt, n, k, 100 + i, dev)
        copies = copies_for(weight_bytes(fmt, n, k))
        ws_list = [(wq0, ws0)] + [(wq0.clone(), ws0.clone()) for _ in range(copies - 1)]
        x = torch.from_numpy(make_x(k, m, 200 + i)).to(dev)
        best = None
        for block_n, nb in KOMP_TUNE[fmt]:
            def call(c, block_n=block_n, nb=nb):
                xq, xd = khost.quantize(fmt, x)
                khost.gemv(fmt, ws_list[c][0], ws_list[c][1], xq, xd, n, k, block_n=block_n, nb=nb, mode=2)

            try:
                for c in range(copies):
                    call(c)  # compile + warm
                torch.cuda.synchronize()
                graphs = []
                s = torch.cuda.Stream(dev)
                s.wait_stream(torch.cuda.current_stream(dev))
                try:
                    for c in range(copies):
                        g = torch.cuda.CUDAGraph()
                        with torch.cuda.stream(s), torch.cuda.graph(g, stream=s):
                            call(c)
                        graphs.append(g)
                    run = lambda r: graphs[r % copies].replay()  # noqa: E731
                    how = "CUDA graph replays"
                except Exception as e:  # noqa: BLE001 -- fall back to eager launches
                    graphs = []
                    run = lambda r: call(r % copies)  # noqa: E731
                    how = f"eager launches (graph capture failed: {str(e)[:80]})"
                torch.cuda.current_stream(dev).wait_stream(s)
                reps = max(20, 4 * copies)
                for r in range(2 * copies):
                    run(r)
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for r in range(reps):
                    run(r)
                e1.record()
                e1.synchronize()
                us = e0.elapsed_time(e1) * 1e3 / reps
                del graphs
            except Exception as e:  # noqa: BLE001 -- a config that does not compile is skipped, and said so
                notes.append(f"{name} block_n={block_n} nb={nb}: {str(e).splitlines()[0][:120]}")
                continue
            if best is None or us < best[0]:
                best = (us, block_n, nb, how)
        del ws_list, wq0, ws0
        torch.cuda.empty_cache()
        if best is None:
            per.append({"name": name, "unavailable": "no tune config ran"})
            continue
        us, block_n, nb, how = best
        step_us += us
        gbs = algo_bytes(fmt, n, k, m) / (us * 1e-6) / 1e9
        per.append({"name": name, "us": round(us, 2), "gbs": round(gbs, 1), "frac": round(gbs / peak, 4),
                    "best": {"block_n": block_n, "nb": nb, "num_warps": 4, "mode": "dp4a (2)"}, "timing": how})
    total = sum(algo_bytes(f, n, k, m) for f, n, k, _ in select_layers(args) if f in KOMP_TUNE)
    out = {"value": round(total / (step_us * 1e-6) / 1e9, 2) if step_us else None, "unit": "GB/s",
           "us_per_step": round(step_us, 2), "per_layer": per,
           "what": "COMP's Triton kernels (baseline/_ref, triton " + __import__("triton").__version__ +
                   ") JIT-compiled on this B200, mode 2; per layer the best of the spec tune space; quantize + GEMV "
                   "per layer, graph-replayed over rotating weight copies (>= 4x L2)"}
    if notes:
        out["skipped_configs"] = notes
    print(json.dumps(out), flush=True)


def run_reference_arm(args, rank, world):
    if rank != 0:
        return
    m = args.m
    layers_def = select_layers(args)
    full_bytes = sum(algo_bytes(f, n, k, m) for f, n, k, _ in layers_def)
    # bound the run: a step is a row sample sized so warmup + steps stay within ~90 s of host time
    probe_layers, _ = cpu_layers(layers_def, m, budget_rows=512)
    probe_s, _ = cpu_reference_run(probe_layers, 1, 1)
    probe_bytes = sum(algo_bytes(f, min(n, 512), k, m) for f, n, k, _ in layers_def)
    est_full = probe_s * full_bytes / probe_bytes
    budget = 90.0 / max(1, args.steps + args.warmup)
    frac = min(1.0, budget / est_full) if est_full > 0 else 1.0
    rows = max(64, int(max(n for _, n, _, _ in layers_def) * frac))
    layers, meta = cpu_layers(layers_def, m, budget_rows=rows)
    step_bytes = sum(algo_bytes(f, r, k, m) for f, r, k in meta)
    sec, threads = cpu_reference_run(layers, args.steps, args.warmup)
    gbs = step_bytes / sec / 1e9
    full_rows = all(r == n for (f, r, k), (_, n, _, _) in zip(meta, layers_def))
    what = "full layers" if full_rows else f"first {rows} rows of each layer"
    sample = (f"{what} ({', '.join(f'{f} {r}x{k}' for f, r, k in meta)}), M={m}; quantize + GEMV + f64 reference dot "
              f"per layer, each step (oracle/c/oracle.c, C + OpenMP, one thread per core this process may use)")
    interp = {"unavailable": "skipped (--no-komp)"} if args.no_komp else \
        _run_komp_worker("interp", args, timeout=300, extra=["--komp-rows", str(args.komp_rows)])
    triton_gpu = {"unavailable": "skipped (--no-komp)"} if args.no_komp else \
        _run_komp_worker("triton", args, timeout=600, extra=["--device", os.environ.get("LOCAL_RANK", "0")])
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(sec * 1e3 * full_bytes / step_bytes, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8/int32 dots, f64 sum",
        "data": "synthetic (BASELINE distributions, seeded)",
        "config": bench_config(args.workload, layers_def, m),
        "setup": {"parallelism": "host cores, rank 0 only", "world": world},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port", "sample": sample},
        "reference_interpreter": interp,
        "triton_b200": triton_gpu,
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
    ap.add_argument("--e2e-steps", type=int, default=None, help="steps of the end-to-end legs (default: --steps)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end legs (profiling runs)")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip per-layer timing, parity and the clock window (profiling runs)")
    ap.add_argument("--layers", default=None, help="comma-separated layer names of the workload to keep (profiling)")
    ap.add_argument("--exchange", default="p2p", choices=["p2p", "nccl"], help="N > 1 output all-gather")
    ap.add_argument("--pdl", default="on", choices=["on", "off"], help="programmatic dependent launch of the GEMVs")
    ap.add_argument("--e2e-api", default="pinned", choices=["pinned", "device"],
                    help="end-to-end leg: pinned host x in and Y stored into pinned host memory by the kernels "
                         "(N = 1: b2q_quant_gemv_pinned, N > 1: RowShardedGemv(x_host, out=y_host)), or device "
                         "buffers with torch memcpys around each call")
    ap.add_argument("--no-komp", action="store_true", help="reference arm: skip COMP's interpreter and Triton legs")
    ap.add_argument("--komp-rows", type=int, default=16, help="reference arm: rows per layer run by the interpreter")
    ap.add_argument("--komp-worker", default=None, choices=["interp", "triton"], help=argparse.SUPPRESS)
    ap.add_argument("--device", type=int, default=0, help=argparse.SUPPRESS)
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.layers and not select_layers(args):
        ap.error(f"--layers {args.layers}: no such layer in {args.workload}")
    if args.komp_worker == "interp":
        return komp_interp_worker(args)
    if args.komp_worker == "triton":
        return komp_triton_worker(args)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return

    import datetime

    import torch
    import torch.distributed as dist

    from comp_b200 import _lib, host
    from comp_b200.dist import RowShardedGemv, partition, slice_rows

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    lib = _lib.load()
    if args.pdl == "off":
        _lib.call("b2q_set_pipeline", 4, 0)
    m = args.m
    layers_def = select_layers(args)
    total_bytes = sum(algo_bytes(f, n, k, m) for f, n, k, _ in layers_def)
    weights_total = sum(weight_bytes(f, n, k) for f, n, k, _ in layers_def)
    # every step must stream its weights from HBM: keep >= 4x L2 of distinct weights per GPU, rotating copies
    per_gpu = max(1, weights_total // world)
    copies = copies_for(per_gpu)
    peak, peak_kind = peaks()

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
            L.obj = RowShardedGemv(fmt, L.w[0][0], L.w[0][1], n, k, exchange=args.exchange)
        layers.append(L)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    sptr = stream.cuda_stream
    dominant = max(range(len(layers)), key=lambda i: weight_bytes(layers[i].fmt, layers[i].n, layers[i].k))
    exchange_name = None if world == 1 else layers[0].obj.exchange

    def launch(L, wq, ws, y=None):
        """N = 1: fused quantize + GEMV straight through the C ABI."""
        y = L.y if y is None else y
        rc = lib.b2q_quant_gemv_ws(L.fid, wq.data_ptr(), wq.stride(0), ws.data_ptr(), L.x.data_ptr(), L.x.stride(0),
                                   None, None, y.data_ptr(), L.rows, L.k, m, L.work.data_ptr(), L.wsb, sptr)
        if rc != 0:
            raise RuntimeError(_lib.last_error())

    def sharded(L, wq, ws):
        """N > 1: the layer's fused GEMV + all-gather on the given weight slice (one RowShardedGemv per layer, so one
        set of receive buffers; its weights are swapped per rotating copy)."""
        L.obj.wq, L.obj.ws = wq, ws
        return L.obj(L.x)

    def step(c):
        for L in layers:
            if world == 1:
                launch(L, *L.w[c])
            else:
                sharded(L, *L.w[c])

    for w in range(args.warmup):
        step(w % copies)
    torch.cuda.synchronize()

    def capture(fn, count):
        """count CUDA graphs, graph j = fn(j), captured on a side stream."""
        gs = []
        cs = torch.cuda.Stream(dev)
        cs.wait_stream(stream)
        for j in range(count):
            gs.append(torch.cuda.CUDAGraph())
            with torch.cuda.stream(cs), torch.cuda.graph(gs[-1], stream=cs):
                fn(j)
        stream.wait_stream(cs)
        return gs

    # N > 1: steps are captured as CUDA graphs (fused GEMV + all-gather launches, or GEMV + NCCL all-gather), so host
    # launch time does not bound the multi-GPU step: one graph of G consecutive steps (whole cycles over the weight
    # copies, >= 8 steps, so launches inside it keep their programmatic overlap) and one graph per single step for
    # the remainder of a step count
    graphs, big = [], None
    launches_per_step = 0
    G = copies * -(-8 // copies)
    if world > 1:
        n0 = _lib.launch_count()
        graphs = capture(step, copies)
        launches_per_step = (_lib.launch_count() - n0) // copies
        big = capture(lambda j: [step(s % copies) for s in range(G)], 1)[0]
        for c in range(copies):
            graphs[c].replay()
        big.replay()
        torch.cuda.synchronize()
        dist.barrier()

    def run_steps(n):
        """n consecutive steps (the same calls on every rank)."""
        if world == 1:
            for s in range(n):
                step(s % copies)
            return
        for _ in range(n // G):
            big.replay()
        for s in range(n % G):
            graphs[s % copies].replay()

    # ---- device-timed region: inputs resident in HBM, nothing but the steps between the two events (an event
    # between two kernels would end their programmatic overlap); NVML sampled every millisecond inside it ----
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev, period=0.001) as clocks:
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        launches0 = _lib.launch_count()
        clocks.mark(True)
        start.record(stream)
        run_steps(args.steps)
        end.record(stream)
        end.synchronize()
        torch.cuda.synchronize()
        clocks.mark(False)
        launches = _lib.launch_count() - launches0 if world == 1 else launches_per_step * args.steps
    if world > 1:
        dist.barrier()
    ms = start.elapsed_time(end)
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    sec = ms / 1e3
    value = total_bytes * args.steps / sec / 1e9
    if world > 1:
        for L in layers:
            if L.obj.status_code() != 0:
                raise RuntimeError(f"rank {rank}: fused all-gather poll timed out on {L.name} ({L.obj.status_code()})")

    # ---- every layer alone, back to back over rotating copies (>= 4x L2), event-timed, max over ranks; right after
    # the timed steps, before the sustained window heats the GPU, so both see the same clocks ----
    per_layer = []
    dom_alone_ms = None
    if not args.no_extras:
        for i, L in enumerate(layers):
            nc = copies_for(weight_bytes(L.fmt, slice_rows(L.n, world), L.k))  # the same on every rank
            ws_list = [L.w[c % copies] if c < copies else (L.w[0][0].clone(), L.w[0][1].clone()) for c in range(nc)]
            if world == 1:
                per_run = 1
                run = lambda r, L=L, ws_list=ws_list, nc=nc: launch(L, *ws_list[r % nc])  # noqa: E731
                lg = None
            else:  # one graph of whole cycles over the copies (>= 16 launches, chained as in a step)
                per_run = nc * -(-16 // nc)
                lg = capture(lambda j, L=L, ws_list=ws_list, nc=nc, per_run=per_run:
                             [sharded(L, *ws_list[r % nc]) for r in range(per_run)], 1)
                run = lambda r, lg=lg: lg[0].replay()  # noqa: E731
            runs = max(-(-4 * nc // per_run), -(-min(400, max(50, args.steps)) // per_run))
            reps = runs * per_run
            for r in range(max(2, -(-2 * nc // per_run))):
                run(r)
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for r in range(runs):
                run(r)
            e1.record(stream)
            e1.synchronize()
            td = torch.tensor([e0.elapsed_time(e1) / reps], dtype=torch.float64, device=dev)
            if world > 1:
                dist.all_reduce(td, op=dist.ReduceOp.MAX)
            us = float(td.item()) * 1e3
            gbs = algo_bytes(L.fmt, L.n, L.k, m) / (us * 1e-6) / 1e9
            per_layer.append({"name": L.name, "shape": f"{L.fmt} {L.n}x{L.k}", "rows_per_gpu": L.rows,
                              "us": round(us, 3), "gbs": round(gbs, 1), "frac": round(gbs / world / peak, 4),
                              "copies": nc, "launches_timed": reps})
            if i == dominant:
                dom_alone_ms = us / 1e3
            if lg is not None:
                lg.clear()
            del ws_list, lg
        torch.cuda.empty_cache()
        if world > 1:
            for L in layers:
                L.obj.wq, L.obj.ws = L.w[0]

    # ---- N = 1, decode at M = 1 only: the same layers with 2, 4 and 16 activation columns (speculative or batched
    # decode) through the same fused call (the planner's path: the GEMV with every column in registers, or the
    # tcgen05 GEMM), each layer alone back to back over its rotating copies, event-timed ----
    batched = {}
    if not args.no_extras and world == 1 and m == 1:
        for mb in (2, 4, 16):
            rows_b = []
            for i, L in enumerate(layers):
                xb = torch.from_numpy(make_x(L.k, mb, 300 + i)).to(dev)
                yb = torch.empty((mb, L.n), dtype=torch.float32, device=dev)
                wsb = host.workspace_size(L.fmt, L.n, L.k, mb)
                wk = torch.empty(max(16, wsb), dtype=torch.uint8, device=dev)
                nc = copies_for(weight_bytes(L.fmt, L.n, L.k))
                ws_list = [L.w[c % copies] if c < copies else (L.w[0][0].clone(), L.w[0][1].clone())
                           for c in range(nc)]

                def run_b(r, L=L, xb=xb, yb=yb, wk=wk, wsb=wsb, ws_list=ws_list, nc=nc, mb=mb):
                    wq, ws = ws_list[r % nc]
                    rc = lib.b2q_quant_gemv_ws(L.fid, wq.data_ptr(), wq.stride(0), ws.data_ptr(), xb.data_ptr(),
                                               xb.stride(0), None, None, yb.data_ptr(), L.n, L.k, mb, wk.data_ptr(),
                                               wsb, sptr)
                    if rc != 0:
                        raise RuntimeError(_lib.last_error())
                reps = max(4 * nc, 40)
                for r in range(2 * nc):
                    run_b(r)
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                for r in range(reps):
                    run_b(r)
                e1.record(stream)
                e1.synchronize()
                us = e0.elapsed_time(e1) * 1e3 / reps
                gbs = algo_bytes(L.fmt, L.n, L.k, mb) / (us * 1e-6) / 1e9
                rows_b.append({"name": L.name, "shape": f"{L.fmt} {L.n}x{L.k}", "m": mb, "us": round(us, 3),
                               "gbs": round(gbs, 1), "frac": round(gbs / peak, 4), "launches_timed": reps})
                del xb, yb, wk, ws_list
            batched[mb] = rows_b
        torch.cuda.empty_cache()

    # ---- sustained: >= 1 s of the same steps after the per-layer timing, event-timed, with its own clock record (a
    # short timed region starts from cool clocks; this shows the rate once the power cap has had time to act). The
    # step count comes from the timed region's rate, max over ranks, so every rank makes the same calls ----
    sustained = None
    if not args.no_extras:
        n_sus = int(min(200000, -(-1000.0 // max(1e-3, ms / args.steps))))
        q0, q1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(dev, period=0.005) as sclocks:
            if world > 1:
                dist.barrier()
            sclocks.mark(True)
            q0.record(stream)
            run_steps(n_sus)
            q1.record(stream)
            q1.synchronize()
            sclocks.mark(False)
        ts = torch.tensor([q0.elapsed_time(q1)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(ts, op=dist.ReduceOp.MAX)
        sms = float(ts.item())
        sustained = {"value": round(total_bytes * n_sus / (sms / 1e3) / 1e9, 2), "unit": "GB/s", "steps": n_sus,
                     "ms_per_step": round(sms / n_sus, 5), "clocks": sclocks.summary()}

    dom = layers[dominant]
    if dom_alone_ms is not None:
        dom_ms = dom_alone_ms
        dom_note = ("dominant kernel alone: CUDA events around back-to-back launches of it over rotating weight copies "
                    "(>= 4x L2), on its launching stream, after the timed steps" +
                    (" (graph replays), max over ranks" if world > 1 else ""))
    else:
        dom_ms = ms / args.steps
        dom_note = "whole step (per-layer timing skipped)"
    dom_bytes = algo_bytes(dom.fmt, dom.rows, dom.k, m)
    achieved = dom_bytes / (dom_ms / 1e3) / 1e9
    tag = f"{dom.fmt}_{dom.rows}x{dom.k}"
    traffic = profiled_traffic(tag)

    # ---- N > 1 parity: every rank's gathered Y == the unsharded GEMV of the full layer on its own GPU ----
    parity = None
    if world > 1 and not args.no_extras:
        mism, checked = 0, 0
        for i, L in enumerate(layers):
            wq_f, ws_f = make_layer_gpu(L.fmt, L.n, L.k, 100 + i, dev)  # copy 0, all rows
            want = host.quant_gemv(L.fmt, wq_f, ws_f, L.x, L.n, L.k, split=False)
            got = sharded(L, *L.w[0]).clone()
            torch.cuda.synchronize()
            mism += int((got.view(torch.int32) != want.view(torch.int32)).sum().item())
            checked += got.numel()
            del wq_f, ws_f, want, got
        torch.cuda.empty_cache()
        bad = torch.tensor([mism, 0 if all(L.obj.status_code() == 0 for L in layers) else 1], dtype=torch.int64,
                           device=dev)
        dist.all_reduce(bad, op=dist.ReduceOp.SUM)
        parity = {"bitexact": int(bad[0].item()) == 0 and int(bad[1].item()) == 0,
                  "mismatched_values": int(bad[0].item()), "ranks_with_timeouts": int(bad[1].item()),
                  "values_checked_per_rank": checked,
                  "check": "every layer, after the timed region: the full Y gathered on every rank (its own rows and "
                           "the rows received from its peers) bit-identical to the unsharded fused GEMV of the full "
                           "layer on the same GPU (rows are independent: src/komp/kernels.py:55-56, 94)"}

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
                L.obj(L.x_host, out=y_host[i])
                continue
            wq, ws = L.w[0]
            rc = lib.b2q_quant_gemv_pinned(L.fid, wq.data_ptr(), wq.stride(0), ws.data_ptr(), L.x_host.data_ptr(),
                                           L.x_host.stride(0), y_host[i].data_ptr(), L.n, L.k, m,
                                           pin_ws[i].data_ptr(), pin_ws[i].numel(), sptr)
            if rc != 0:
                raise RuntimeError(_lib.last_error())
        stream.synchronize()  # the step's results are read on the host

    def e2e_step_device():
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
                ys.append(L.obj(xs[i]) if i + 1 == len(layers) else L.obj(xs[i]).clone())
        for i, y in enumerate(ys):
            y_host[i].copy_(y, non_blocking=True)
        stream.synchronize()  # the step's results are read on the host

    def e2e_step_dropin():
        # COMP's call sequence with the reference's signatures (src/komp/host.py:63-85): x copied in from pinned host
        # memory, host.quantize, host.gemv (dp4a), Y copied back to pinned host memory; the host waits every step
        for i, L in enumerate(layers):
            x = L.x_host.to(dev, non_blocking=True)
            xq, xd = host.quantize(L.fmt, x)
            y, _ = host.gemv(L.fmt, L.w[0][0], L.w[0][1], xq, xd, L.n, L.k, mode=host.MODES["dp4a"])
            y_host[i].copy_(y, non_blocking=True)
        stream.synchronize()

    def time_e2e(fn, steps):
        for _ in range(3):
            fn()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(steps):
            fn()
        e1.record(stream)
        e1.synchronize()
        te = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        return round(total_bytes * steps / (float(te.item()) / 1e3) / 1e9, 3)

    e2e_gbs = time_e2e(e2e_step_pinned if pinned else e2e_step_device, e2e_steps) if e2e_steps else None
    dropin_gbs = time_e2e(e2e_step_dropin, e2e_steps) if (e2e_steps and world == 1) else None
    h2d = sum(L.x_host.numel() * 4 for L in layers)
    d2h = sum(L.n * m * 4 for L in layers)
    # graphs that hold NCCL calls must be released before the process group is destroyed
    graphs.clear()
    del graphs, big
    torch.cuda.synchronize()
    if world > 1:
        for L in layers:
            L.obj.close()

    # ---- CPU baseline (rank 0, N = 1): bounded sample of the same layers; the oracle also checks the GPU here ----
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import native, ref

        rows = 8192
        cl, meta = [], []
        for L in layers:
            r = min(rows, L.n)
            cl.append((L.fmt, L.w[0][0][:r].cpu().numpy(), L.w[0][1][:r].cpu().numpy(), L.x_host.numpy(), L.k))
            meta.append((L.fmt, r, L.k))
        csec, threads = cpu_reference_run(cl, 3, 1)
        cbytes = sum(algo_bytes(f, r, k, m) for f, r, k in meta)
        cpu = {"value": round(cbytes / csec / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
               "sample": f"first {rows} rows of each layer (the GPU's weights and activations), M={m}, 3 steps of "
                        f"quantize + GEMV + f64 reference dot (oracle/c/oracle.c, OpenMP)"}
        # parity at N = 1: the first 512 rows of every layer, the bench's own fused launch against the oracle
        checks = []
        for L, (fmt, wq, ws, x, k) in zip(layers, cl):
            r = min(512, L.n)
            launch(L, *L.w[0])
            xq, xd = host.quantize(fmt, L.x)
            _, s = host.gemv(fmt, L.w[0][0][:r], L.w[0][1][:r], xq, xd, r, k, mode=2, store_s=True)
            y = L.y[:, :r].cpu().numpy()
            if fmt in ("q4_0", "q8_0", "iq4_nl"):
                oq, od = native.quant_q8_0(x)
            else:
                oq, od, _ = native.quant_q8_K(x)
            ry, rs = native.gemv(fmt, wq[:r], ws[:r], oq, od, k, want_s=True)
            q_ok = bool(np.array_equal(xq.cpu().numpy(), oq) and
                        np.array_equal(xd.cpu().numpy().view(np.uint32), od.view(np.uint32)))
            s_ok = bool(np.array_equal(s.cpu().numpy(), rs))
            err = ref.relerr(y, ry)
            checks.append({"name": L.name, "rows": r, "quant_bytes": q_ok, "int32_block_dots": s_ok,
                           "relerr": err, "ok": q_ok and s_ok and err <= TOL})
        parity = {"bitexact": all(c["quant_bytes"] and c["int32_block_dots"] for c in checks),
                  "ok": all(c["ok"] for c in checks), "layers": checks,
                  "check": "first 512 rows of every layer against the C oracle (oracle/c/oracle.c): quantized bytes "
                           "and int32 block dots bit-exact, the bench's fused Y within 1e-5 of the exact reference"}

    # the dominant layer runs as quantizer + tensor-core GEMM when it has 8+ columns and a workspace for them
    L_tc = world == 1 and m >= 8 and getattr(layers[dominant], "wsb", 0) > 0
    if rank == 0:
        cs = clocks.summary()
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8 dp4a dots, f32 scale+sum",
            "data": "synthetic (BASELINE distributions, seeded, random-init weights)",
            "config": bench_config(args.workload, layers_def, m),
            "setup": {"parallelism": f"row-shard x{world}" if world > 1 else "single GPU",
                      "graph_steps": G if world > 1 else None,
                      "exchange": {None: None,
                                   "p2p": "fused all-gather: 64-bit (flag, value) peer stores from the GEMV epilogue",
                                   "nccl": "NCCL all_gather_into_tensor"}[exchange_name],
                      "graph": world > 1, "pdl": args.pdl,
                      "weights_per_gpu_mib": round(per_gpu / 2**20), "rotating_copies": copies},
            "us_per_gemv": round(ms * 1e3 / args.steps / len(layers), 3),
            "hbm_frac": round(value / world / peak, 4),
            "per_layer": per_layer,
            "batched_m2": batched.get(2),
            "batched_m4": batched.get(4),
            "batched_m16": batched.get(16),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic,
                         "kernel": (f"quantizer + tcgen05 GEMM {tag} (2 launches, timed together)" if L_tc else
                                    f"gemv {tag} (quant prologue fused{', all-gather fused' if world > 1 else ''})"),
                         "timing": dom_note, "peak_source": f"{peak_kind} hbm_gbs",
                         "us_per_launch": round(dom_ms * 1e3, 3), "algorithmic_bytes_per_launch": dom_bytes},
            "parity": parity,
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_gbs, "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "steps": e2e_steps,
                    "api": ("C-ABI b2q_quant_gemv_pinned per layer (pinned host x in, the kernels copy x in and store "
                            "Y into pinned host memory; host sync every step)" if pinned else
                            "comp_b200.host.quant_gemv (fused quantize + GEMV per layer; torch memcpy of x in, Y out)")
                    if world == 1 else f"comp_b200.dist.RowShardedGemv ({exchange_name}" +
                    ("; pinned host x in, Y stored into pinned host memory)" if pinned else
                     "; torch memcpy of x in, Y out)")},
            "e2e_dropin": None if dropin_gbs is None else {
                "value": dropin_gbs, "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "steps": e2e_steps,
                "api": "comp_b200.host.quantize + comp_b200.host.gemv(mode=dp4a), COMP's signatures "
                       "(src/komp/host.py:63-85); torch memcpy of x in from pinned memory, Y out; host sync every step"},
            "gpu_launches": launches,
            "clocks": cs,
            "sustained": sustained,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

"""Self-check of the CUDA kernels on the GPU (the role of komp.verify, src/komp/verify.py).

The checks mirror COMP's: quantizer bytes, int32 block dots, KURN's reference dot rebuilt bit-identically from those
dots, and the f32 output within KURN's relative-error rule. The exact references here are computed on the GPU with
plain torch operations, independently of this package's kernels:
  quantizers  the ggml formulas in f32 torch ops (IEEE division, single multiplies, explicit half-away / half-even
              rounding), q8_0 scale through torch's f16 conversion;
  block dots  weights decoded with integer ops, dots as f64 matmuls (exact: every partial sum is an integer < 2^53);
  reference   f64 sequential sum over blocks in KURN's order (q4_0: dw*dx*s, tq2_0: dx*dw*s).
The repository's parity tests additionally pin the kernels to the reference's recorded outputs.
"""

import json
import os

import numpy as np
import torch

from . import _lib, host

TOL = 1e-5
# ggml's IQ4_NL levels (kvalues_iq4nl)
IQ4_NL_LEVELS = (-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113)
MODE_NAMES = {0: "bytes", 1: "dp4a", 2: "dp4a"}


def _round_half_away(v):
    a = v.abs()
    f = a.floor()
    r = torch.where(a - f >= 0.5, f + 1.0, f)
    return torch.where(v < 0, -r, r)


def ref_quantize(fmt, x):
    """Exact q8_0 / q8_K of f32 x [M][K] in torch ops -> (xq int8, xd f32)."""
    m, k = x.shape
    if host.FORMATS[fmt]["act"] == "q8_0":
        b = x.reshape(m, k // 32, 32)
        amax = b.abs().amax(dim=-1)
        # every division tensor by tensor: torch may evaluate a scalar divisor or dividend as a multiply by a
        # reciprocal, which is not the correctly rounded quotient the quantizers use
        d = amax / torch.full_like(amax, 127.0)
        nz = d != 0
        idv = torch.where(nz, torch.ones_like(d) / torch.where(nz, d, torch.ones_like(d)), torch.zeros_like(d))
        q = _round_half_away(b * idv[..., None])
        return q.to(torch.int8).reshape(m, k), d.half().float()
    b = x.reshape(m, k // 256, 256)
    ax = b.abs()
    amax = ax.amax(dim=-1)
    idx = torch.arange(256, device=x.device).expand_as(b)
    first = torch.where(ax == amax[..., None], idx, torch.full_like(idx, 256)).amin(dim=-1)
    mx = torch.gather(b, -1, first.clamp(max=255)[..., None])[..., 0]
    nz = amax != 0
    iscale = torch.full_like(mx, -127.0) / torch.where(nz, mx, torch.ones_like(mx))
    q = torch.clamp(torch.round(iscale[..., None] * b), max=127.0)  # torch.round is half-to-even
    q = torch.where(nz[..., None], q, torch.zeros_like(q))
    d = torch.where(nz, torch.ones_like(iscale) / iscale, torch.zeros_like(iscale))
    return q.to(torch.int8).reshape(m, k), d


def ref_values(fmt, wq, k):
    """Decoded weight values [N][K] (int) from the quant plane."""
    n = wq.shape[0]
    if fmt == "q8_0":  # the stored int8 values (an extension beyond the reference)
        return wq[:, :k].view(torch.int8).to(torch.int32)
    w = wq[:, : k // (4 if fmt == "tq2_0" else 2)].to(torch.int32)
    if fmt == "q4_0":
        b = w.reshape(n, k // 32, 16)
        return torch.cat([(b & 15) - 8, (b >> 4) - 8], dim=-1).reshape(n, k)
    if fmt == "iq4_nl":  # Q4_0's nibble layout, each nibble a level of ggml's table (an extension)
        lv = torch.tensor(IQ4_NL_LEVELS, dtype=torch.int32, device=wq.device)
        b = w.reshape(n, k // 32, 16)
        return torch.cat([lv[b & 15], lv[b >> 4]], dim=-1).reshape(n, k)
    b = w.reshape(n, k // 256, 2, 32)  # [block][h][i] -> value h*128 + j*32 + i at bits 2j
    v = torch.stack([((b >> (2 * j)) & 3) - 1 for j in range(4)], dim=3)  # [n][blk][h][j][i]
    return v.reshape(n, k)


def ref_dots(fmt, wq, xq, k):
    blk = host.FORMATS[fmt]["block"]
    vals = ref_values(fmt, wq, k).double()
    n, m, nb = vals.shape[0], xq.shape[0], k // blk
    v = vals.reshape(n, nb, blk).permute(1, 0, 2)
    q = xq.double().reshape(m, nb, blk).permute(1, 2, 0)
    return torch.bmm(v, q).round().long().permute(2, 1, 0)  # [m][n][nb]


def ref_dot(fmt, ws, xd, s):
    dw = ws.view(torch.float16).double()
    dx = (xd.half() if fmt != "tq2_0" else xd).double()
    m, n, nb = s.shape
    total = torch.zeros((m, n), dtype=torch.float64, device=s.device)
    for b in range(nb):
        if fmt != "tq2_0":  # q4_0 (and the q8_0 / iq4_nl extensions): dw * dx * s
            total += (dw[None, :, b] * dx[:, None, b]) * s[:, :, b].double()
        else:
            total += (dx[:, None, b] * dw[None, :, b]) * s[:, :, b].double()
    return total


def relerr(y, r):
    scale = r.abs().max().item() if r.numel() else 0.0
    return (y.double() - r).abs().max().item() / (scale if scale > 0 else 1.0) if r.numel() else 0.0


def problem(fmt, n, k, m, seed, extreme, dev):
    """Seeded synthetic problem on the GPU: split planes and f32 activations (BASELINE distributions)."""
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    blk = host.FORMATS[fmt]["block"]
    if fmt in ("q4_0", "iq4_nl"):
        wq = torch.randint(0, 256, (n, k // 2), dtype=torch.uint8, generator=g)
        if extreme:  # nibbles only 0 or 15: values -8 and +7 (iq4_nl: levels -127 and 113)
            wq = torch.tensor([0x00, 0x0F, 0xF0, 0xFF], dtype=torch.uint8)[torch.randint(0, 4, (n, k // 2), generator=g)]
        ws = (torch.randn((n, k // blk), generator=g) * (0.02 if fmt == "q4_0" else 0.002)).abs().half().view(torch.int16)
    elif fmt == "q8_0":
        lo = -128 if extreme else -127
        wq = torch.randint(lo, 128, (n, k), dtype=torch.int16, generator=g).to(torch.int8).view(torch.uint8)
        ws = (torch.randn((n, k // blk), generator=g) * 0.002).abs().half().view(torch.int16)
    else:
        t = torch.randint(0, 81 if not extreme else 256, (n, k // 4), dtype=torch.int64, generator=g)
        wq = ((t % 3) | ((t // 3 % 3) << 2) | ((t // 9 % 3) << 4) | ((t // 27 % 3) << 6)).to(torch.uint8) \
            if not extreme else t.to(torch.uint8)
        ws = (torch.randn((n, k // blk), generator=g) * 0.05).abs().half().view(torch.int16)
    x = torch.randn((m, k), generator=g)
    if extreme and k:
        x[torch.rand((m, k), generator=g) < 0.05] = 0.0
        out = torch.rand((m, k), generator=g) < 0.01
        x[out] = torch.where(torch.rand(int(out.sum()), generator=g) < 0.5, -1e4, 1e4)
    return wq.to(dev), ws.to(dev), x.to(dev)


def algo_bytes(fmt, n, k, m):
    """Algorithmic bytes of one GEMV: the weights once (ggml block bytes), the q8 activations, the f32 output."""
    f = host.FORMATS[fmt]
    return n * k * f["nbytes"] // f["block"] + m * (k + 4 * k // host.ACT_BLOCK[f["act"]]) + 4 * m * n


def hbm_peak(value=None):
    """The HBM bandwidth (GB/s) the --json lines divide by: the given value, else the COMP_B200_HBM_GBS environment
    variable, else None (no fraction is reported)."""
    if value is None:
        value = os.environ.get("COMP_B200_HBM_GBS")
    try:
        return float(value) if value is not None else None
    except ValueError:
        raise ValueError(f"HBM peak {value!r} is not a number (GB/s)") from None


def check_gemv(fmt, n, k, m, seed=0, extreme=False, mode=2, dev=None, timed=False):
    dev = dev or torch.device("cuda")
    wq, ws, x = problem(fmt, n, k, m, seed, extreme, dev)
    xq, xd = host.quantize(fmt, x)
    rq, rd = ref_quantize(fmt, x)
    quant_ok = bool(torch.equal(xq, rq) and torch.equal(xd.view(torch.int32), rd.view(torch.int32)))
    y, s = host.gemv(fmt, wq, ws, xq, xd, n, k, mode=mode, store_s=True)
    exact = ref_dots(fmt, wq, xq, k)
    idots_ok = bool(torch.equal(s.long(), exact))
    r_ours = ref_dot(fmt, ws, xd, s.long())
    r = ref_dot(fmt, ws, xd, exact)
    rebuilt_ok = bool(torch.equal(r_ours.view(torch.int64), r.view(torch.int64)))
    err = relerr(y, r)
    out = {"fmt": fmt, "n": n, "k": k, "m": m, "quant": quant_ok, "idots": idots_ok, "rebuilt": rebuilt_ok,
           "relerr": err, "ok": quant_ok and idots_ok and rebuilt_ok and err <= TOL}
    if timed:  # the GEMV alone (no S dump), event-timed on the current stream after warm-up
        stream = torch.cuda.current_stream(dev)
        for _ in range(3):
            host.gemv(fmt, wq, ws, xq, xd, n, k, mode=mode)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 20
        a.record(stream)
        for _ in range(reps):
            host.gemv(fmt, wq, ws, xq, xd, n, k, mode=mode)
        b.record(stream)
        b.synchronize()
        out["us"] = a.elapsed_time(b) * 1e3 / reps
    return out


def check_dp4a(seed=0, n=1024, dev=None):
    """The GPU dp4a.s32.s32 against its definition (src/komp/verify.py:37-54) on edge and random words."""
    dev = dev or torch.device("cuda")
    rng = np.random.default_rng(seed)
    edge = np.array([0, -1, 0x7F7F7F7F, -0x7F7F7F80, 0x01010101, 0x0F0F0F0F, 0x03030303, 2**31 - 1, -(2**31)],
                    dtype=np.int64)
    def words():
        w = rng.integers(-(2**31), 2**31, size=n, dtype=np.int64)
        pick = rng.random(n) < 0.3
        w[pick] = rng.choice(edge, size=int(pick.sum()))
        return w
    a, b = words(), words()
    c = rng.integers(-(2**20), 2**20, size=n, dtype=np.int64)
    ta, tb, tc = (torch.from_numpy(v.astype(np.int32)).to(dev) for v in (a, b, c))
    out = torch.empty_like(ta)
    _lib.call("b2q_probe_dp4a", ta.data_ptr(), tb.data_ptr(), tc.data_ptr(), out.data_ptr(), n,
              torch.cuda.current_stream(dev).cuda_stream)
    ref = c.copy()
    for i in range(4):
        sa = ((a >> (8 * i)) & 0xFF).astype(np.int64)
        sb = ((b >> (8 * i)) & 0xFF).astype(np.int64)
        ref += np.where(sa >= 128, sa - 256, sa) * np.where(sb >= 128, sb - 256, sb)
    ref = (ref + 2**31) % 2**32 - 2**31
    return bool(np.array_equal(out.cpu().numpy().astype(np.int64), ref))


def check_decode(seed=0, extreme=False, dev=None):
    """The decode probes against the weight values (the role of verify.check_decode, src/komp/verify.py:70-91):
    b2q_decode_q4_0 on [37][16] quant bytes and b2q_decode_tq2_0 on [5][64] against the integer decode above, every
    value; and for TQ2_0 the dot through the probe's values, scaled and summed in KURN's order, bit-identical to the
    reference dot through the exact block dots. Random data: uniform nibbles / trits; extreme: nibbles 0 and 15 only,
    and every crumb value (3 included) for TQ2_0."""
    dev = dev or torch.device("cuda")
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    stream = torch.cuda.current_stream(dev).cuda_stream
    res = {}
    if extreme:
        q4 = torch.tensor([0x00, 0x0F, 0xF0, 0xFF], dtype=torch.uint8)[torch.randint(0, 4, (37, 16), generator=g)]
        tq = torch.randint(0, 256, (5, 64), dtype=torch.int64, generator=g).to(torch.uint8)
    else:
        q4 = torch.randint(0, 256, (37, 16), dtype=torch.int64, generator=g).to(torch.uint8)
        t = torch.randint(0, 81, (5, 64), dtype=torch.int64, generator=g)
        tq = ((t % 3) | ((t // 3 % 3) << 2) | ((t // 9 % 3) << 4) | ((t // 27 % 3) << 6)).to(torch.uint8)
    q4, tq = q4.to(dev), tq.to(dev)
    out = torch.zeros((37, 32), dtype=torch.int32, device=dev)
    _lib.call("b2q_decode_q4_0", q4.data_ptr(), out.data_ptr(), 37, stream)
    res["q4_0"] = bool(torch.equal(out, ref_values("q4_0", q4, 32)))
    out = torch.zeros((5, 256), dtype=torch.int32, device=dev)
    _lib.call("b2q_decode_tq2_0", tq.data_ptr(), out.data_ptr(), 5, stream)
    vals_ok = bool(torch.equal(out, ref_values("tq2_0", tq.reshape(1, 5 * 64), 5 * 256).reshape(5, 256)))
    # one weight row of 5 blocks against one q8_K column: dots through the probe's values == exact dots
    x = torch.randn((1, 5 * 256), generator=g).to(dev)
    xq, xd = host.quantize("tq2_0", x)
    ws = (torch.randn((1, 5), generator=g) * 0.05).abs().half().view(torch.int16).to(dev)
    s_probe = (out.long() * xq.long().reshape(5, 256)).sum(dim=1).reshape(1, 1, 5)
    exact = ref_dots("tq2_0", tq.reshape(1, 5 * 64), xq, 5 * 256)
    same = torch.equal(ref_dot("tq2_0", ws, xd, s_probe).view(torch.int64),
                       ref_dot("tq2_0", ws, xd, exact).view(torch.int64))
    res["tq2_0"] = vals_ok and bool(same)
    return res


# the reference's shapes (src/komp/verify.py PROBLEMS) for its two formats, and the same Q4_0 shapes for the two
# extensions beyond it
PROBLEMS = {"q4_0": ((64, 512, 1), (37, 416, 3), (5, 96, 2)), "tq2_0": ((64, 1024, 1), (37, 768, 3), (5, 1280, 2)),
            "q8_0": ((64, 512, 1), (37, 416, 3), (5, 96, 2)), "iq4_nl": ((64, 512, 1), (37, 416, 3), (5, 96, 2))}


def line(r, mode, label=""):
    return (f"{'ok  ' if r['ok'] else 'FAIL'} {r['fmt']:5} gemv {MODE_NAMES[mode]:5} {label} n={r['n']} k={r['k']} "
            f"m={r['m']} quant={'exact' if r['quant'] else 'MISMATCH'} idots={'exact' if r['idots'] else 'MISMATCH'} "
            f"reference_dot={'bit-identical' if r['rebuilt'] else 'DIFFERS'} relerr={r['relerr']:.1e}")


def json_line(r, mode, label="", extreme=False, peak=None):
    """The fields of `line` as one JSON object, plus (when the check was timed) us per GEMV, algorithmic GB/s and
    the fraction of the measured HBM peak."""
    d = {"ok": r["ok"], "fmt": r["fmt"], "op": "gemv", "mode": MODE_NAMES[mode], "config": label, "n": r["n"],
         "k": r["k"], "m": r["m"], "extreme": extreme, "quant": "exact" if r["quant"] else "MISMATCH",
         "idots": "exact" if r["idots"] else "MISMATCH",
         "reference_dot": "bit-identical" if r["rebuilt"] else "DIFFERS", "relerr": float(r["relerr"])}
    if "us" in r:
        gbs = algo_bytes(r["fmt"], r["n"], r["k"], r["m"]) / r["us"] / 1e3
        d.update(us=round(r["us"], 3), gbs=round(gbs, 1), hbm_frac=round(gbs / peak, 4) if peak else None)
    return json.dumps(d)


def run_all(log=print, as_json=False, peak=None):
    """dp4a probe, decode probes (random and extreme), then every GEMV problem in both variants, random and extreme
    data (src/komp/verify.py:152-170). peak: HBM GB/s for the --json fractions (hbm_peak)."""
    fails = 0
    ok = check_dp4a(seed=3)
    fails += not ok
    peak = hbm_peak(peak)
    if as_json:
        log(json.dumps({"ok": ok, "op": "dp4a.s32.s32", "words": 1024}))
    else:
        log(f"{'ok  ' if ok else 'FAIL'} dp4a.s32.s32 on the GPU == its definition (1024 edge/random words)")
    for extreme in (False, True):
        for f, ok in check_decode(seed=7, extreme=extreme).items():
            fails += not ok
            kind = "extreme" if extreme else "random"
            if as_json:
                log(json.dumps({"ok": ok, "op": "decode", "fmt": f, "data": kind}))
            else:
                log(f"{'ok  ' if ok else 'FAIL'} decode {f:5} {kind:7} (values == integer decode)")
    for fmt, probs in PROBLEMS.items():
        for mode in (0, 2):
            for n, k, m in probs:
                for seed, extreme in ((1, False), (2, True)):
                    r = check_gemv(fmt, n, k, m, seed, extreme, mode, timed=as_json)
                    fails += not r["ok"]
                    log(json_line(r, mode, extreme=extreme, peak=peak) if as_json else
                        line(r, mode) + (" extreme" if extreme else ""))
    log(json.dumps({"failures": fails}) if as_json else f"{fails} failures")
    return fails

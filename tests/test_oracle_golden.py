"""Pins the oracle (oracle.ref in numpy, oracle.native in C) to the reference: every golden vector recorded from COMP's
own kernels under the Triton interpreter (tests/golden/make_golden.py), and gguf-py's independent Q8_0 quantizer and
Q4_0 / TQ2_0 dequantizers. CPU only."""

import numpy as np
import pytest

from oracle import native, ref

from .conftest import golden_case_ids


def _same_f32(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


@pytest.mark.parametrize("impl", ["numpy", "c"])
def test_quantizers_match_reference(golden, impl):
    x = golden["quant/x"]
    q0 = ref.quant_q8_0(x) if impl == "numpy" else native.quant_q8_0(x)
    assert np.array_equal(q0[0], golden["quant/q8_0/xq"]) and _same_f32(q0[1], golden["quant/q8_0/xd"])
    qk = ref.quant_q8_K(x) if impl == "numpy" else native.quant_q8_K(x)
    assert np.array_equal(qk[0], golden["quant/q8_K/xq"]) and _same_f32(qk[1], golden["quant/q8_K/xd"])


def test_quant_input_has_the_edge_cases(golden):
    """The config-2 input really contains what it is meant to exercise."""
    x = golden["quant/x"]
    xd0 = golden["quant/q8_0/xd"]
    xdK = golden["quant/q8_K/xd"]
    assert (xd0 == 0).any() and (xdK == 0).any()          # all-zero blocks
    assert (np.abs(x) == 1e4).any() and (x == 0).mean() > 0.04
    assert (xd0 == 1.0).any() and (xdK == 1.0).any()      # half-point blocks: d = 1 exactly
    assert (np.abs(x - np.round(x)) == 0.5).sum() > 100


def test_q8_0_bytes_match_gguf(golden):
    """gguf-py (gguf.quants, Q8_0.quantize_blocks) is an independent implementation of ggml's q8_0."""
    gq = pytest.importorskip("gguf.quants")
    gguf = pytest.importorskip("gguf")
    x = golden["quant/x"]
    xq, xd = ref.quant_q8_0(x)
    from comp_b200 import host

    ours = host.q8_0_blocks(xq, xd)
    theirs = gq.quantize(x, gguf.GGMLQuantizationType.Q8_0).tobytes()
    assert ours == theirs


@pytest.mark.parametrize("cid", golden_case_ids())
def test_gemv_oracle_matches_reference(golden, cid):
    c = next(c for c in golden.cases() if c["id"] == cid)
    g = golden.case(cid)
    fmt, n, k, m = c["fmt"], c["n"], c["k"], c["m"]
    wq, ws = ref.split(fmt, g["W"].tobytes(), n, k)
    oq, od = ref.quantize(fmt, g["x"])
    assert np.array_equal(oq, g["xq"]) and _same_f32(od, g["xd"])
    r, s = ref.gemv(fmt, wq, ws, g["xq"], g["xd"], k)
    assert np.array_equal(s, g["s0"]) and np.array_equal(s, g["s1"])
    assert ref.relerr(g["y0"], r) <= ref.TOL and ref.relerr(g["y1"], r) <= ref.TOL
    rc, sc = native.gemv(fmt, wq, ws, g["xq"], g["xd"], k, want_s=True)
    assert np.array_equal(sc, g["s0"])
    assert np.array_equal(rc.view(np.uint64), r.view(np.uint64))  # C and numpy reference dots: bit-identical


@pytest.mark.parametrize("fmt", ["q4_0", "tq2_0", "q8_0"])
def test_decode_matches_gguf_dequantize(fmt):
    gq = pytest.importorskip("gguf.quants")
    gguf = pytest.importorskip("gguf")
    n, k = 7, 1024
    W, _ = ref.problem(fmt, n, k, 1, seed=4, extreme=(fmt != "tq2_0"))
    wq, ws = ref.split(fmt, W, n, k)
    t = getattr(gguf.GGMLQuantizationType, fmt.upper())
    deq = gq.dequantize(np.frombuffer(W, dtype=np.uint8).reshape(n, -1), t).astype(np.float64)
    vals = ref.decode(fmt, wq, k).astype(np.float64)
    blk = ref.BLOCK[fmt]
    d = ws.view(np.float16).astype(np.float64).repeat(blk, axis=1)
    assert np.allclose(deq, vals * d, rtol=0, atol=1e-3 * np.abs(d).max())
    assert np.array_equal(np.sign(deq), np.sign(vals * d))


@pytest.mark.parametrize("extreme", [False, True])
def test_q8_0_gemv_oracle_pinned_to_gguf(extreme):
    """Q8_0 weights (an extension beyond the reference) against q8_0 activations: the oracle's int32 block dots and
    f64 reference dot equal the float64 product of gguf-py's own dequantization of both operands (weights read as
    ggml Q8_0 blocks, activations as the q8_0 blocks the quantizer stores), and the C oracle agrees bit for bit."""
    gq = pytest.importorskip("gguf.quants")
    gguf = pytest.importorskip("gguf")
    n, k, m = 9, 2048, 3
    W, x = ref.problem("q8_0", n, k, m, seed=12, extreme=extreme)
    wq, ws = ref.split("q8_0", W, n, k)
    xq, xd = ref.quantize("q8_0", x)
    r, s = ref.gemv("q8_0", wq, ws, xq, xd, k)
    # block dots: int8 x int8 of the stored values
    vals = ref.decode("q8_0", wq, k).astype(np.int64).reshape(n, k // 32, 32)
    want_s = np.einsum("nbv,mbv->mnb", vals, xq.astype(np.int64).reshape(m, k // 32, 32))
    assert np.array_equal(s, want_s)
    T = gguf.GGMLQuantizationType.Q8_0
    wdq = gq.dequantize(np.frombuffer(W, dtype=np.uint8).reshape(n, -1), T).astype(np.float64)
    from comp_b200 import host

    xdq = gq.dequantize(np.frombuffer(host.q8_0_blocks(xq, xd), dtype=np.uint8).reshape(m, -1), T).astype(np.float64)
    assert ref.relerr(xdq @ wdq.T, r) <= 1e-9
    rc, sc = native.gemv("q8_0", wq, ws, xq, xd, k, want_s=True)
    assert np.array_equal(sc, s) and np.array_equal(rc.view(np.uint64), r.view(np.uint64))


@pytest.mark.parametrize("extreme", [False, True])
def test_iq4_nl_oracle_pinned_to_gguf(extreme):
    """IQ4_NL weights (a second extension) against q8_0 activations: the oracle's decode equals gguf-py's IQ4_NL
    dequantization (level[nibble] * d), its int32 block dots are the int8-level x int8 products, its f64 reference dot
    equals the float64 product of gguf-py's dequantized operands, and the C oracle agrees bit for bit."""
    gq = pytest.importorskip("gguf.quants")
    gguf = pytest.importorskip("gguf")
    n, k, m = 9, 2048, 3
    W, x = ref.problem("iq4_nl", n, k, m, seed=13, extreme=extreme)
    wq, ws = ref.split("iq4_nl", W, n, k)
    T = gguf.GGMLQuantizationType.IQ4_NL
    wdq = gq.dequantize(np.frombuffer(W, dtype=np.uint8).reshape(n, -1), T).astype(np.float64)
    d = np.repeat(ws.view(np.float16).astype(np.float64), 32, axis=1)
    assert np.array_equal(ref.decode("iq4_nl", wq, k) * d, wdq)
    xq, xd = ref.quantize("iq4_nl", x)
    r, s = ref.gemv("iq4_nl", wq, ws, xq, xd, k)
    vals = ref.decode("iq4_nl", wq, k).astype(np.int64).reshape(n, k // 32, 32)
    assert np.array_equal(s, np.einsum("nbv,mbv->mnb", vals, xq.astype(np.int64).reshape(m, k // 32, 32)))
    from comp_b200 import host

    xdq = gq.dequantize(np.frombuffer(host.q8_0_blocks(xq, xd), dtype=np.uint8).reshape(m, -1),
                        gguf.GGMLQuantizationType.Q8_0).astype(np.float64)
    assert ref.relerr(xdq @ wdq.T, r) <= 1e-9
    rc, sc = native.gemv("iq4_nl", wq, ws, xq, xd, k, want_s=True)
    assert np.array_equal(sc, s) and np.array_equal(rc.view(np.uint64), r.view(np.uint64))


def test_dp4a_and_decode_probes_match_reference(golden):
    assert np.array_equal(ref.dp4a_ref(golden["dp4a/a"], golden["dp4a/b"], golden["dp4a/c"]), golden["dp4a/out"])
    assert np.array_equal(ref.decode_q4_0(golden["decode/q4_0/wq"], 32), golden["decode/q4_0/out"])
    assert np.array_equal(ref.decode_tq2_0(golden["decode/tq2_0/wq"], 256), golden["decode/tq2_0/out"])


def test_oracle_f16_conversion_is_exact():
    lib = native.load()
    h = np.arange(0, 65536, 3, dtype=np.uint32).astype(np.uint16)
    f = np.array([lib.orc_half_to_float(int(v)) for v in h], dtype=np.float32)
    want = h.view(np.float16).astype(np.float32)
    ok = ~np.isnan(want)
    assert np.array_equal(f.view(np.uint32)[ok], want.view(np.uint32)[ok])
    rng = np.random.default_rng(0)
    v = (rng.standard_normal(5000) * 10.0 ** rng.integers(-9, 6, 5000)).astype(np.float32)
    v = np.concatenate([v, np.float32([65504, 65519.99, 65520, 6e-8, 2.98e-8, 1e-10, -0.0, 0.0])])
    hb = np.array([lib.orc_float_to_half(float(x)) for x in v], dtype=np.uint16)
    with np.errstate(over="ignore"):
        assert np.array_equal(hb, v.astype(np.float16).view(np.uint16))


def test_plant_a_mistake_in_the_oracle_is_caught(golden):
    """The golden check has teeth: an oracle with half-even rounding for q8_0 fails on the half-point block."""
    x = golden["quant/x"]
    b = x.reshape(x.shape[0], -1, 32)
    d = (np.abs(b).max(-1) / np.float32(127)).astype(np.float32)
    idv = np.where(d != 0, np.float32(1) / np.where(d != 0, d, 1), 0).astype(np.float32)
    wrong = np.rint((b * idv[..., None]).astype(np.float32)).astype(np.int8).reshape(x.shape)
    assert not np.array_equal(wrong, golden["quant/q8_0/xq"])


@pytest.mark.parametrize("extreme", [False, True])
def test_q4_k_oracle_pinned_to_gguf(extreme):
    """Q4_K weights (a third extension) against q8_K activations: the oracle's decode of this backend's split planes
    equals gguf-py's Q4_K dequantization bit for bit, its block dots S are sum_j sc_j * (nibbles . x) of the
    sub-blocks, its f64 reference equals the float64 product of gguf-py's dequantized operands, the host split equals
    the oracle's, and the C oracle agrees bit for bit."""
    gq = pytest.importorskip("gguf.quants")
    gguf = pytest.importorskip("gguf")
    from comp_b200 import host

    n, k, m = 9, 2048, 3
    W, x = ref.problem("q4_k", n, k, m, seed=17, extreme=extreme)
    wq, ws = ref.split("q4_k", W, n, k)
    hq, hs = host.split("q4_k", W, n, k)
    assert np.array_equal(hq, wq) and np.array_equal(hs, ws) and ws.shape == (n, k // 256 * 10)
    wdq = gq.dequantize(np.frombuffer(W, dtype=np.uint8).reshape(n, -1), gguf.GGMLQuantizationType.Q4_K)
    assert np.array_equal(ref.decode_q4_k(wq, ws, k).view(np.uint32), wdq.astype(np.float32).view(np.uint32))
    xq, xd = ref.quantize("q4_k", x)
    r, s = ref.gemv("q4_k", wq, ws, xq, xd, k)
    q, _, _, sc, _ = ref.q4_k_parts(wq, ws, k)
    sub = np.einsum("nsv,msv->mns", q.astype(np.int64).reshape(n, k // 32, 32),
                    xq.astype(np.int64).reshape(m, k // 32, 32)).reshape(m, n, k // 256, 8)
    assert np.array_equal(s, (sub * sc[None].astype(np.int64)).sum(-1))
    xdq = (xq.astype(np.float64).reshape(m, k // 256, 256) * xd.astype(np.float64)[..., None]).reshape(m, k)
    assert ref.relerr(xdq @ wdq.astype(np.float64).T, r) <= 1e-6
    rc, sc_ = native.gemv("q4_k", wq, ws, xq, xd, k, want_s=True)
    assert np.array_equal(sc_, s) and np.array_equal(rc.view(np.uint64), r.view(np.uint64))

"""`target triton` specs routed to the B200 backend: KURN's spec syntax, COMP's keys (src/komp/spec.py).

    kernel     q4_0_gemv_triton
    op         gemv
    weights    q4_0           # q4_0 | tq2_0
    target     triton
    arch       sm_100a        # sm_80 | sm_86 | sm_89 | sm_90 (COMP) | sm_100a (this backend)
    mode       dp4a           # dp4a | bytes
    block_n    64             # Triton schedule hints: validated, accepted, not used by the CUDA planner
    nb         4
    num_warps  4
    tune       block_n=32,64 nb=4,8

Problem keys (n, k, m) give the shape `verify` runs on. Key set, legal values, defaults and error messages are
COMP's (spec.py:22-60); `sm_100a` is added to `arch` and is the default here.

The spec text format is KURN's (`key value`, `#` comments, one `tune k=a,b ...` line). KURN's parser (`kurn.spec`)
is used when the kurn package is importable; otherwise the built-in parser below reads the same format.
"""

import itertools

try:  # KURN present: its parser and its error type, so KURN's CLI catches our errors
    from kurn.spec import SpecError
    from kurn.spec import parse as _kurn_parse
    from kurn.spec import parse_overrides as _kurn_parse_overrides
except ImportError:  # standalone
    _kurn_parse = _kurn_parse_overrides = None

    class SpecError(ValueError):
        """An invalid spec (the role of kurn.spec.SpecError)."""


KEYS = {
    "op": ("gemv",),
    "weights": ("q4_0", "tq2_0"),
    "arch": ("sm_80", "sm_86", "sm_89", "sm_90", "sm_100a"),
    "mode": ("dp4a", "bytes"),
    "block_n": (8, 16, 32, 64, 128),
    "nb": (1, 2, 4, 8, 16),
    "num_warps": (1, 2, 4, 8),
}
DEFAULTS = {"arch": "sm_100a", "mode": "dp4a", "block_n": 64, "num_warps": 4}
FORMAT_DEFAULTS = {"q4_0": {"nb": 4}, "tq2_0": {"nb": 1}}
BLOCK = {"q4_0": 32, "tq2_0": 256}
PROBLEM = {"q4_0": {"n": 64, "k": 512, "m": 1}, "tq2_0": {"n": 64, "k": 1024, "m": 1}}
COMMON = ("kernel", "target")
MODE = {"bytes": 0, "dp4a": 2}


def _value(v):
    try:
        return int(v)
    except ValueError:
        return v


def parse(text):
    """Spec text -> (base dict, tune dict of lists). Same format as KURN's spec files."""
    if _kurn_parse is not None:
        return _kurn_parse(text)
    base, tune = {}, {}
    for lineno, raw in enumerate(text.splitlines(), 1):
        line = raw.split("#", 1)[0].strip()
        if not line:
            continue
        parts = line.split()
        key = parts[0]
        if key == "tune":
            single, lists = parse_overrides(parts[1:])
            for k, v in {**single, **lists}.items():
                tune[k] = v if isinstance(v, list) else [v]
            continue
        if len(parts) != 2:
            raise SpecError(f"line {lineno}: expected 'key value', got {raw.strip()!r}")
        if key in base:
            raise SpecError(f"line {lineno}: duplicate key {key!r}")
        base[key] = _value(parts[1])
    return base, tune


def parse_overrides(items):
    """['k=v', 'k=a,b', ...] -> (single overrides dict, list overrides dict)."""
    if _kurn_parse_overrides is not None:
        return _kurn_parse_overrides(items)
    single, lists = {}, {}
    for it in items:
        if "=" not in it:
            raise SpecError(f"override {it!r} is not key=value")
        k, v = it.split("=", 1)
        vals = [_value(x) for x in v.split(",") if x != ""]
        if not vals:
            raise SpecError(f"override {it!r} has no value")
        if len(vals) == 1:
            single[k] = vals[0]
        else:
            lists[k] = vals
    return single, lists


def resolve(spec, overrides=None):
    """Validated config with defaults filled in (src/komp/spec.py:39-60); raises SpecError."""
    c = {**spec, **(overrides or {})}
    if c.get("target") != "triton":
        raise SpecError(f"target {c.get('target')!r}: comp_b200 handles target triton")
    for k in ("op", "weights"):
        if k not in c:
            raise SpecError(f"missing required key {k!r}")
    if c["weights"] not in KEYS["weights"]:
        raise SpecError(f"weights={c['weights']!r} not allowed for target triton: expected one of {list(KEYS['weights'])}")
    for k in c:
        if k not in KEYS and k not in COMMON and k not in ("n", "k", "m"):
            raise SpecError(f"unknown key {k!r} for target triton: expected one of {sorted((*KEYS, *COMMON, 'n', 'k', 'm'))}")
    for k, allowed in KEYS.items():
        c.setdefault(k, FORMAT_DEFAULTS[c["weights"]].get(k, DEFAULTS.get(k)))
        if c[k] not in allowed:
            raise SpecError(f"{k}={c[k]!r} not allowed for target triton: expected one of {list(allowed)}")
    for k, v in PROBLEM[c["weights"]].items():
        c.setdefault(k, v)
    for k in ("n", "k", "m"):
        if not isinstance(c[k], int) or c[k] < 0:
            raise SpecError(f"{k}={c[k]!r} must be a non-negative integer")
    if c["k"] % BLOCK[c["weights"]]:
        raise SpecError(f"k must be a multiple of {BLOCK[c['weights']]} ({c['weights']} block)")
    c.setdefault("kernel", f"{c['weights']}_{c['op']}_triton")
    return c


def load(path):
    with open(path) as fh:
        return parse(fh.read())


def configs(spec, tune):
    """Every legal config of the spec's tune space (the spec itself if there is none) (src/komp/spec.py:68-75)."""
    names = list(tune)
    for combo in itertools.product(*(tune[k] for k in names)) if names else [()]:
        try:
            yield resolve(spec, dict(zip(names, combo)))
        except SpecError:
            continue


def label(c):
    return f"mode={c['mode']} block_n={c['block_n']} nb={c['nb']} num_warps={c['num_warps']}"

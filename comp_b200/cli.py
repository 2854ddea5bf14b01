"""comp_b200 command line: the spec routing of COMP's CLI (src/komp/cli.py), on the B200 backend.

    python -m comp_b200 check  SPEC [k=v ...]   validate a `target triton` spec (and its tune space)
    python -m comp_b200 verify SPEC [k=v ...]   every config of the spec on the GPU vs exact references
    python -m comp_b200 verify --all            the full GPU self-check set (dp4a, both GEMVs, both variants)
    python -m comp_b200 verify --all --json [--hbm-gbs G]
                                                the same as JSON lines, each GEMV also timed (us, GB/s, and the
                                                fraction of G, or of $COMP_B200_HBM_GBS, when one is given)

`kurn check|verify SPEC` routes here for specs with `target triton` through comp_b200.kurn_ext. COMP's `gen` and
`mix` (PTX/SASS generation and inspection) have no counterpart: this backend ships its own compiled library.
Exit codes as COMP's: 0 ok, 1 check failures, 2 usage or spec error.
"""

import sys

USAGE = __doc__


def _spec(args):
    from . import spec

    path = next((a for a in args if not a.startswith("-") and "=" not in a), None)
    if path is None:
        raise spec.SpecError("no spec file given")
    base, tune = spec.load(path)
    single, lists = spec.parse_overrides([a for a in args if "=" in a and not a.startswith("-")])
    base.update(single)
    tune.update(lists)
    return spec, base, tune


def cmd_check(args):
    from . import spec as _s

    try:
        spec, base, tune = _spec(args)
        c = spec.resolve(base)
        n = len(list(spec.configs(base, tune)))
    except (_s.SpecError, OSError) as e:
        print(f"comp_b200 check: {e}", file=sys.stderr)
        return 2
    print(f"ok {c['kernel']}: {c['weights']} {c['op']} target triton {c['arch']} {spec.label(c)}; "
          f"tune space: {n} legal configs")
    return 0


def cmd_verify(args):
    from . import spec as _s
    from . import verify

    if "--all" in args:
        peak = args[args.index("--hbm-gbs") + 1] if "--hbm-gbs" in args[:-1] else None
        try:
            peak = verify.hbm_peak(peak)
        except ValueError as e:
            print(f"comp_b200 verify: {e}", file=sys.stderr)
            return 2
        return 1 if verify.run_all(as_json="--json" in args, peak=peak) else 0
    try:
        spec, base, tune = _spec(args)
        spec.resolve(base)
        cfgs = list(spec.configs(base, tune))
    except (_s.SpecError, OSError) as e:
        print(f"comp_b200 verify: {e}", file=sys.stderr)
        return 2
    fails = 0
    ok = verify.check_dp4a()
    fails += not ok
    print(f"{'ok  ' if ok else 'FAIL'} dp4a.s32.s32 on the GPU == its definition")
    for c in cfgs:
        mode = spec.MODE[c["mode"]]
        for seed, extreme in ((1, False), (2, True)):
            r = verify.check_gemv(c["weights"], c["n"], c["k"], c["m"], seed, extreme, mode)
            fails += not r["ok"]
            print(verify.line(r, mode, spec.label(c)) + (" extreme" if extreme else "") + "  [sm_100a]")
    print(f"{fails} failures")
    return 1 if fails else 0


COMMANDS = {"check": cmd_check, "verify": cmd_verify}


def main(argv=None):
    argv = list(sys.argv[1:] if argv is None else argv)
    if not argv or argv[0] not in COMMANDS:
        print(USAGE)
        return 0 if argv and argv[0] in ("-h", "--help") else 2
    return COMMANDS[argv[0]](argv[1:])


def spec_command(cmd, argv):
    """Entry for kurn.hooks.TARGET_BACKENDS["triton"] (the role of komp.cli.spec_command, src/komp/cli.py:195-200)."""
    if cmd not in ("check", "verify"):
        print(f"kurn {cmd}: not available for target triton on comp_b200 (supports check, verify)", file=sys.stderr)
        return 2
    return main([cmd, *argv])

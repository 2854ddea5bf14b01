"""KURN spec routing of the B200 backend, as the reference tests it (tests/test_komp.py:43-66): the CLI checks a
`target triton` spec and its tune space, rejects bad specs with exit 2 and the offending key on stderr, and the KURN
hook (comp_b200.kurn_ext, the role of kurn/src/kurn/ext/komp.py) routes `kurn check` on such a spec here. KURN itself
is not installed: a stub `kurn.hooks` module stands in for it. The GPU test runs `verify SPEC` over the tune space."""

import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
FIX = os.path.join(ROOT, "tests", "fixtures")
Q4 = os.path.join(FIX, "q4_0_gemv.kurn")
TQ2 = os.path.join(FIX, "tq2_0_gemv.kurn")


def run(*args, env=None):
    e = dict(os.environ if env is None else env)
    e["PYTHONPATH"] = ROOT + os.pathsep + e.get("PYTHONPATH", "")
    return subprocess.run([sys.executable, *args], capture_output=True, text=True, env=e, cwd=ROOT, timeout=600)


@pytest.mark.parametrize("spec,n_cfg", [(Q4, 8), (TQ2, 8)])
def test_check_accepts_spec_and_counts_tune_space(spec, n_cfg):
    r = run("-m", "comp_b200", "check", spec)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "target triton" in r.stdout and f"tune space: {n_cfg} legal configs" in r.stdout, r.stdout


def test_check_overrides():
    r = run("-m", "comp_b200", "check", Q4, "block_n=32", "nb=4,8,16")
    assert r.returncode == 0, r.stdout + r.stderr
    assert "block_n=32" in r.stdout and "tune space: 12 legal configs" in r.stdout, r.stdout


@pytest.mark.parametrize("old,new,key", [
    ("block_n    64", "block_n    33", "block_n"),       # the reference's own bad-spec case
    ("weights    q4_0", "weights    q5_1", "weights"),
    ("k          416", "k          400", "k"),           # not a whole number of 32-value blocks
    ("target     triton", "target     cuda", "target"),
    ("num_warps  4", "num_warps  4\nwarps      8", "warps"),  # unknown key
])
def test_bad_spec_rejected(tmp_path, old, new, key):
    text = open(Q4).read()
    assert old in text
    p = tmp_path / "bad.kurn"
    p.write_text(text.replace(old, new))
    r = run("-m", "comp_b200", "check", str(p))
    assert r.returncode == 2 and key in r.stderr, r.stdout + r.stderr


def test_missing_spec_file_is_a_usage_error(tmp_path):
    r = run("-m", "comp_b200", "check", str(tmp_path / "absent.kurn"))
    assert r.returncode == 2


def test_unknown_command_prints_usage():
    r = run("-m", "comp_b200", "mix")
    assert r.returncode == 2 and "check" in r.stdout


def _stub_kurn(tmp_path):
    pkg = tmp_path / "kurn"
    pkg.mkdir()
    (pkg / "__init__.py").write_text("")
    (pkg / "hooks.py").write_text("TARGET_BACKENDS = {}\n")
    env = dict(os.environ)
    env["PYTHONPATH"] = str(tmp_path)
    return env


def test_kurn_routes_target_triton(tmp_path):
    """Importing the hook inside a KURN install registers TARGET_BACKENDS["triton"]; `kurn check SPEC` then runs
    this backend's check."""
    env = _stub_kurn(tmp_path)
    code = ("import sys; from kurn import hooks; import comp_b200.kurn_ext; "
            f"sys.exit(hooks.TARGET_BACKENDS['triton']('check', [{Q4!r}]))")
    r = run("-c", code, env=env)
    assert r.returncode == 0 and "target triton" in r.stdout, r.stdout + r.stderr


def test_kurn_hook_refuses_commands_it_lacks(tmp_path):
    env = _stub_kurn(tmp_path)
    code = ("import sys; from kurn import hooks; import comp_b200.kurn_ext; "
            f"sys.exit(hooks.TARGET_BACKENDS['triton']('gen', [{Q4!r}]))")
    r = run("-c", code, env=env)
    assert r.returncode == 2 and "gen" in r.stderr, r.stdout + r.stderr


def test_kurn_hook_reports_a_missing_backend(tmp_path):
    """Without an importable comp_b200.cli the hook says how to get it and exits 2, as COMP's hook does."""
    env = _stub_kurn(tmp_path)
    code = ("import sys; from kurn import hooks; import comp_b200.kurn_ext; sys.modules['comp_b200.cli'] = None; "
            f"sys.exit(hooks.TARGET_BACKENDS['triton']('check', [{Q4!r}]))")
    r = run("-c", code, env=env)
    assert r.returncode == 2 and "comp_b200" in r.stderr, r.stdout + r.stderr


def test_register_into_a_hooks_object():
    from comp_b200 import kurn_ext

    class Hooks:
        TARGET_BACKENDS = {}

    kurn_ext.register(Hooks)
    assert Hooks.TARGET_BACKENDS["triton"] is kurn_ext._spec_command


@pytest.mark.gpu
@pytest.mark.parametrize("spec", [Q4, TQ2])
def test_spec_tune_space_verifies(spec):
    r = run("-m", "comp_b200", "verify", spec)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.strip().endswith("0 failures")
    assert "MISMATCH" not in r.stdout and "DIFFERS" not in r.stdout


@pytest.mark.gpu
def test_verify_all():
    r = run("-m", "comp_b200", "verify", "--all")
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.strip().endswith("0 failures")
    assert "decode q4_0" in r.stdout and "decode tq2_0" in r.stdout

"""KURN routing hook: `kurn check|verify SPEC` on a spec whose target is triton runs comp_b200.

Same shape as COMP's hook (kurn/src/kurn/ext/komp.py:10-19): comp_b200.cli is imported lazily, and a failed import
reports how to install it (exit 2) instead of raising. `register(hooks)` installs the hook into a KURN `hooks`
module (`hooks.TARGET_BACKENDS["triton"]`); importing this module inside a KURN install registers it directly.
"""

import sys


def _spec_command(cmd, argv):
    try:
        from comp_b200.cli import spec_command
    except ImportError as e:
        print(f"kurn {cmd}: target triton needs the comp_b200 package (build it with python -m comp_b200.build; {e})",
              file=sys.stderr)
        return 2
    return spec_command(cmd, argv)


def register(hooks):
    hooks.TARGET_BACKENDS["triton"] = _spec_command
    return hooks


try:  # inside KURN: register on import, as kurn/ext/komp.py does
    from kurn import hooks as _hooks  # type: ignore[import-not-found]
except ImportError:
    _hooks = None
else:
    register(_hooks)

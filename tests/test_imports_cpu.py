"""Every module of the package imports on its own, whichever is imported first
(a fresh set of kore_b200 modules per import catches circular imports that a
lucky import order would hide). Runs in a child process so the registries of
the test session are left alone."""
import subprocess
import sys

SCRIPT = r"""
import importlib, pkgutil, sys
import kore_b200
names = [m.name for m in pkgutil.walk_packages(kore_b200.__path__, "kore_b200.") if m.name != "kore_b200._C"]
bad = []
for n in names:
    for k in [k for k in sys.modules if k == "kore_b200" or k.startswith("kore_b200.")]:
        del sys.modules[k]
    try:
        importlib.import_module(n)
    except ImportError as e:
        if "libc10" in str(e) or "_C" in str(e).split()[-1:]:
            continue                     # the compiled extension needs torch's libraries first
        bad.append(f"{n}: {e!r}"[:200])
    except Exception as e:  # noqa: BLE001
        bad.append(f"{n}: {e!r}"[:200])
print(len(names))
print("\n".join(bad))
sys.exit(1 if bad else 0)
"""


def test_every_module_imports_first():
    r = subprocess.run([sys.executable, "-c", SCRIPT], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert int(r.stdout.split()[0]) > 100

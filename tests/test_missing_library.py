"""Without libkvcache.so the package fails loudly: importing the binding, the
matmul_module shim or the paged pool raises an ImportError that names the build
command, as the reference's actionable ImportError does when its extension is
missing (tests/test_cpu_only.py:81-101); the reference's own kv_cache.py, which
imports matmul_module, turns that into its ImportError.  There is no CPU
fallback to reach.
Each case runs in a fresh interpreter with KVC_LIB_PATH pointing at a file
that does not exist."""

from __future__ import annotations

import os
import subprocess
import sys

import pytest

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
PKG = os.path.join(ROOT, "gfx1150-inference_b200")


@pytest.mark.parametrize("module", ["kvcache_ffi", "matmul_module", "paged"])
def test_import_without_library_raises_actionable_error(module, tmp_path):
    code = (
        "import sys\n"
        f"sys.path.insert(0, {PKG!r})\n"
        "try:\n"
        f"    import {module}\n"
        "except ImportError as exc:\n"
        "    print('IMPORTERROR', exc)\n"
        "    sys.exit(3)\n"
        "print('IMPORTED')\n"
    )
    env = dict(os.environ, KVC_LIB_PATH=str(tmp_path / "no_such_libkvcache.so"),
               PYTHONDONTWRITEBYTECODE="1")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                       timeout=240)
    assert r.returncode == 3, r.stdout + r.stderr
    assert "build_lib.py" in r.stdout, r.stdout

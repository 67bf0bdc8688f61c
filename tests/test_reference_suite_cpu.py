"""The reference's own CPU test files, run unmodified against this package.

``nano_train_b200.compat.pytest_plugin`` answers the reference's ``import src.*`` with this
package's modules (``compat/src_alias.py`` maps each module), so the reference's tests exercise
this framework's public API: runtime engine and contracts, layers, models, MoE, ZeRO, pipeline,
precision, trainer hooks and the example scripts' wiring. The reference tree is found through
``$NTB_REFERENCE_PATH`` or ``reference_path`` in ``BASELINE.json``; without it the test skips.

Excluded: ``tests/test_model_info.py``. It imports the reference's private analytics helpers
(``_eta_tc``, ``_render_appendix_derivations``, ``_resolve_roofline_axis_limits`` and more), which
this package's analytic model (``utils/model_info.py``, a different design with the same public
``dump_model_info``) does not reproduce.
"""
import json
import os
import re
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EXCLUDED = ("test_model_info.py",)


def _reference_tests():
    cands = [os.environ.get("NTB_REFERENCE_PATH")]
    try:
        with open(os.path.join(ROOT, "BASELINE.json")) as f:
            cands.append(json.load(f).get("reference_path"))
    except (OSError, ValueError):
        pass
    for c in cands:
        if c and os.path.isdir(os.path.join(c, "tests")) and os.path.isdir(os.path.join(c, "src")):
            return os.path.join(c, "tests")
    return None


@pytest.mark.slow
def test_reference_suite_passes_against_this_package(tmp_path):
    tests = _reference_tests()
    if tests is None:
        pytest.skip("reference tree not available")
    cmd = [sys.executable, "-m", "pytest", "-q", "-p", "nano_train_b200.compat.pytest_plugin", "-p",
           "no:cacheprovider", tests] + [f"--ignore={os.path.join(tests, e)}" for e in EXCLUDED]
    env = dict(os.environ, PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""),
               PYTHONDONTWRITEBYTECODE="1", OMP_NUM_THREADS="1")
    p = subprocess.run(cmd, cwd=str(tmp_path), env=env, capture_output=True, text=True, timeout=1500)
    tail = p.stdout[-4000:] + p.stderr[-2000:]
    m = re.search(r"(\d+) passed", p.stdout)
    assert p.returncode == 0 and m is not None, tail
    assert int(m.group(1)) >= 198, tail
    assert "failed" not in p.stdout.splitlines()[-1], tail

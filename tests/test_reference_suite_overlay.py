"""The reference's own test suite, run against this build's modules (CPU).

A copy of the reference package gets this build's ``layers.py``,
``cache.py``, ``parallel.py``, ``ggml.py``, ``arch/``, ``_C.py``,
``fused_blocks.py``, ``quants/rtn.py`` and ``libvoodoo_b200.so`` put over its
own; the reference's ``tests/`` then run unchanged, and must give the same
passed / failed / skipped / error counts as an untouched copy run the same
way in the same environment.  The reference's trainer and CLI must import
from the overlaid tree.

The reference checkout is found through ``reference_path`` in BASELINE.json;
where it is absent (the GPU box) the test skips.  Both runs use copies, so
the checkout itself is only read.
"""

from __future__ import annotations

import json
import os
import re
import shutil
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "voodoo-dyn-quant_b200" / "voodoo_quant"
OVERLAY = ["layers.py", "cache.py", "parallel.py", "ggml.py", "_C.py", "fused_blocks.py", "libvoodoo_b200.so",
           "arch/__init__.py", "arch/base.py", "arch/llama.py", "arch/qwen.py", "arch/lfm2.py", "quants/rtn.py"]


def _reference() -> Path | None:
    try:
        path = json.loads((ROOT / "BASELINE.json").read_text()).get("reference_path")
    except (OSError, ValueError):
        return None
    if not path:
        return None
    p = Path(path)
    return p if (p / "voodoo_quant").is_dir() and (p / "tests").is_dir() else None


def _counts(tree: Path) -> tuple[dict, str]:
    env = dict(os.environ, HF_HUB_OFFLINE="1", TRANSFORMERS_OFFLINE="1", PYTHONDONTWRITEBYTECODE="1")
    env.pop("PYTHONPATH", None)
    r = subprocess.run([sys.executable, "-m", "pytest", "tests", "-p", "no:cacheprovider", "--tb=no", "-o",
                        "addopts="], cwd=tree, env=env, capture_output=True, text=True, timeout=900)
    tail = (r.stdout + r.stderr).strip().splitlines()[-1] if (r.stdout + r.stderr).strip() else ""
    counts = {k: 0 for k in ("passed", "failed", "skipped", "error")}
    for n, kind in re.findall(r"(\d+) (passed|failed|skipped|errors?)", tail):
        counts["error" if kind.startswith("error") else kind] = int(n)
    return counts, tail


def test_reference_suite_passes_the_same_over_this_build(tmp_path):
    ref = _reference()
    if ref is None:
        pytest.skip("the reference checkout is not present here")
    if not (PKG / "libvoodoo_b200.so").exists():
        pytest.skip("libvoodoo_b200.so not built")
    ignore = shutil.ignore_patterns(".git", "__pycache__", ".pytest_cache", ".cache")
    plain, over = tmp_path / "plain", tmp_path / "overlay"
    shutil.copytree(ref, plain, ignore=ignore)
    shutil.copytree(ref, over, ignore=ignore)
    for rel in OVERLAY:
        shutil.copy2(PKG / rel, over / "voodoo_quant" / rel)

    base, base_tail = _counts(plain)
    ours, ours_tail = _counts(over)
    assert base["passed"] > 0, base_tail
    assert ours == base, (ours_tail, base_tail)

    env = dict(os.environ, PYTHONDONTWRITEBYTECODE="1")
    env.pop("PYTHONPATH", None)
    # the reference's trainer and CLI import over this build's layers (which the
    # static-shape switch, absent from the reference, identifies)
    r = subprocess.run([sys.executable, "-c", "import voodoo_quant.training.trainer, voodoo_quant.cli, "
                        "voodoo_quant.layers as L; assert hasattr(L, 'set_static_shapes'); print(L.__file__)"],
                       cwd=over, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert str(over) in r.stdout

"""Install the reference's own Python modules into ``oracle/_ref/`` (test and baseline infrastructure).

The reference (qianghua-rl/910b_e2e_accleration_by_codex) is plain Python with no build system, so
``pip install <reference>`` refuses it ("neither setup.py nor pyproject.toml").  This recipe copies
its ``src/`` to a scratch directory, adds a minimal pyproject.toml that names the modules of the
GDN path as top-level py-modules, and lets pip install them (offline, no dependencies) into
``oracle/_ref/``.  That directory is git-ignored but travels with working-tree snapshots, so
``bench.py``'s CPU baseline and ``--impl reference`` arm can import and time the reference's own
``fast_chunk_gated_delta_rule_v2`` where the reference sources themselves are absent.

    python oracle/install_ref.py --reference <reference checkout>

Nothing here is product code: only bench.py's CPU legs and the tests import ``oracle/_ref``.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
TARGET = os.path.join(HERE, "_ref")
# the modules on the GDN path (imports between them included)
MODULES = ("gdn_chunk_fast", "gdn_chunk_fast2", "recurrent_single_step", "cb_engine", "cb_tp",
           "shift_conv_update", "exact_gated_norm")

PYPROJECT = """[build-system]
requires = ["setuptools"]
build-backend = "setuptools.build_meta"

[project]
name = "qianghua-gdn-reference"
version = "0.0.0"

[tool.setuptools]
package-dir = {{"" = "src"}}
py-modules = [{mods}]
"""


def install(reference: str) -> str:
    src = os.path.join(reference, "src")
    present = [m for m in MODULES if os.path.exists(os.path.join(src, m + ".py"))]
    if "gdn_chunk_fast2" not in present:
        raise SystemExit(f"{src} has no gdn_chunk_fast2.py: not the reference checkout")
    with tempfile.TemporaryDirectory(prefix="gdn_ref_") as tmp:
        os.makedirs(os.path.join(tmp, "src"))
        for m in present:
            shutil.copy2(os.path.join(src, m + ".py"), os.path.join(tmp, "src", m + ".py"))
        with open(os.path.join(tmp, "pyproject.toml"), "w") as f:
            f.write(PYPROJECT.format(mods=", ".join(f'"{m}"' for m in present)))
        if os.path.isdir(TARGET):
            shutil.rmtree(TARGET)
        cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--no-deps",
               "--target", TARGET, tmp]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise SystemExit(f"pip install failed:\n{r.stdout}\n{r.stderr}")
    return TARGET


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="the reference checkout (holds src/)")
    print(install(ap.parse_args().reference))

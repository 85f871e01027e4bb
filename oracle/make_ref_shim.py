"""Test infrastructure: materialise an importable copy of the reference DSL.

The reference (pdum.dsl / pdum.tl) targets Python >= 3.14 and uses exactly two
3.14-only syntax forms; this interpreter is 3.12.  This script copies the two
source trees (``packages/dsl/src`` and ``packages/tensorlib/src``) into the
git-ignored ``baseline/_ref/`` and rewrites those forms mechanically:

* PEP 758 ``except A, B:``  ->  ``except (A, B):``
  (``pdum/dsl/capture.py:67``, ``pdum/tl/buffer.py:82``, ``pdum/tl/producer.py:94,102``)
* PEP 750 ``from string.templatelib import Template``  ->  a local stub class
  (``pdum/tl/units.py:26``; only t-string unit literals use it, and nothing on
  the attention / row-reduction path does).

Nothing else is changed.  The reference's own GPU columns
(``conformance/triton_zoo.py``: the hand-written Triton flash kernel) are
copied unchanged to ``baseline/_ref/conformance/`` so the bench can time them
as labelled bars.  The copy is used only to (a) regenerate the golden
fixtures under ``tests/golden/`` with the reference's own ``run_region``,
(b) run the tests that drive the reference's ``plan_region`` into this
package's lowering and (c) time the reference's columns beside ours.  Usage: ``python oracle/make_ref_shim.py [REFERENCE_ROOT]``.
"""

from __future__ import annotations

import re
import json
import os
import shutil
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]
DEST = REPO / "baseline" / "_ref"
_EXCEPT = re.compile(r"^(\s*)except ([A-Za-z_][\w.]*(?:, [A-Za-z_][\w.]*)+):", re.M)


def shim_text(text: str) -> str:
    text = _EXCEPT.sub(lambda m: f"{m.group(1)}except ({m.group(2)}):", text)
    return text.replace(
        "from string.templatelib import Template",
        "class Template:  # py3.12 stand-in for PEP 750's string.templatelib.Template\n    pass",
    )


def reference_root() -> Path | None:
    """Where the reference checkout is mounted: $PDUM_DSL_REFERENCE, else the
    ``reference_path`` that BASELINE.json records; None when neither names an
    existing directory (e.g. on a GPU box, which only uses the prebuilt copy)."""
    env = os.environ.get("PDUM_DSL_REFERENCE")
    cand = env
    if cand is None:
        bj = Path(__file__).resolve().parents[1] / "BASELINE.json"
        if bj.exists():
            cand = json.loads(bj.read_text()).get("reference_path")
    if cand and Path(cand).is_dir():
        return Path(cand)
    return None


def make(ref_root: Path) -> Path:
    for pkg in ("dsl", "tensorlib"):
        src = ref_root / "packages" / pkg / "src"
        dst = DEST / "packages" / pkg / "src"
        if dst.exists():
            shutil.rmtree(dst)
        shutil.copytree(src, dst, ignore=shutil.ignore_patterns("__pycache__"))
        for f in dst.rglob("*.py"):
            t = f.read_text()
            s = shim_text(t)
            if s != t:
                f.write_text(s)
    conf = DEST / "conformance"
    conf.mkdir(parents=True, exist_ok=True)
    for name in ("triton_zoo.py",):
        shutil.copy2(ref_root / "conformance" / name, conf / name)
    return DEST


def ref_paths() -> list[str]:
    return [str(DEST / "packages" / p / "src") for p in ("dsl", "tensorlib")]


def ensure_importable() -> bool:
    """Put the shimmed copy on sys.path; False when it has not been made."""
    paths = ref_paths()
    if not all(Path(p).is_dir() for p in paths):
        return False
    for p in paths:
        if p not in sys.path:
            sys.path.insert(0, p)
    return True


if __name__ == "__main__":
    root = Path(sys.argv[1]) if len(sys.argv) > 1 else reference_root()
    if root is None:
        sys.exit("usage: make_ref_shim.py <reference checkout> (or set PDUM_DSL_REFERENCE)")
    print(make(root))

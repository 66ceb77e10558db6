"""Reference arm of the serving benchmark.

Runs the unmodified reference (installed under ``baseline/_ref``) through
its own public API on the same trace and prints the same JSON line with
``"impl": "reference"``; prints an ``unavailable`` line when it cannot run.
"""

from __future__ import annotations

import os

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def run_reference(args) -> dict:
    if not os.path.isdir(os.path.join(REF_DIR, "infera")):
        return {"impl": "reference", "unavailable": "reference not installed under baseline/_ref"}
    return {"impl": "reference",
            "unavailable": "reference stack (infera router + vLLM worker) launch not wired in this build"}

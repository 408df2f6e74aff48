"""Where the reference checkout lies (TEST INFRASTRUCTURE ONLY).

The reference sources are only needed to build oracle/_ref and to read the
reference headers in layout tests; the GPU box never has them.  Lookup
order: the QWANTO_REFERENCE environment variable, the ``reference_path``
that BASELINE.json names, then ``baseline/_ref`` inside this repository.
Returns None when none of them holds the reference's ``c/`` tree.
"""
from __future__ import annotations

import json
import os

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def reference_root() -> str | None:
    cands = []
    env = os.environ.get("QWANTO_REFERENCE")
    if env:
        cands.append(env)
    try:
        with open(os.path.join(ROOT, "BASELINE.json")) as f:
            p = json.load(f).get("reference_path")
        if p:
            cands.append(p)
    except (OSError, ValueError):
        pass
    cands.append(os.path.join(ROOT, "baseline", "_ref"))
    for c in cands:
        if os.path.isfile(os.path.join(c, "c", "qwanto_turboquant.h")):
            return c
    return None


def reference_c() -> str | None:
    r = reference_root()
    return None if r is None else os.path.join(r, "c")

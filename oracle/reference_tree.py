"""Where the reference project's source tree is, for the steps that build or
run the reference itself (oracle/build_ref.sh, tests/golden/make_golden.py).

TEST INFRASTRUCTURE ONLY.  The location comes from the environment variable
WLQ_REFERENCE_TREE; unset, a directory named ``reference`` beside this
repository's root is tried.  None when neither holds the reference's
csrc/gemv_kernel.cu: the callers then skip the reference steps (GPU boxes
carry only the prebuilt files).
"""
from __future__ import annotations

import os
from typing import Optional

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def locate() -> Optional[str]:
    cands = []
    env = os.environ.get("WLQ_REFERENCE_TREE")
    if env:
        cands.append(env)
    cands.append(os.path.join(os.path.dirname(os.path.realpath(ROOT)), "reference"))
    for c in cands:
        if os.path.isfile(os.path.join(c, "csrc", "gemv_kernel.cu")):
            return c
    return None

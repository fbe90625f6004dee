"""Shared helpers of the test suite (paths, fixtures loading, torch device setup)."""
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")


def golden(name):
    with np.load(os.path.join(GOLDEN, name)) as z:
        return {k: z[k] for k in z.files}


def ensure_built():
    """Builds the in-tree library if sources are newer (nvcc, no GPU needed)."""
    import build  # ultimate-anime-videoplayer_b200/build.py
    return build.build()

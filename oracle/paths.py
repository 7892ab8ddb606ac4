"""Where the reference's source tree is (TEST INFRASTRUCTURE).

The oracle recipe (oracle/Makefile) holds the one default location; the
environment variable CARL_REFERENCE_DIR overrides it.  The tree exists only
where the oracles are built; on a machine without it the prebuilt files under
oracle/_ref/ are used and the tests that read the reference's sources skip.
"""

from __future__ import annotations

import functools
import os
import subprocess
from pathlib import Path

ORACLE = Path(__file__).resolve().parent


@functools.lru_cache(maxsize=1)
def reference_dir() -> Path:
    env = os.environ.get("CARL_REFERENCE_DIR")
    if env:
        return Path(env)
    try:
        out = subprocess.run(["make", "-s", "-C", str(ORACLE), "print-ref"], capture_output=True, text=True,
                             check=True).stdout.strip().splitlines()
        return Path(out[-1]) if out else Path("/nonexistent")
    except (OSError, subprocess.CalledProcessError):
        return Path("/nonexistent")


def reference_present() -> bool:
    return (reference_dir() / "src" / "Kernels.cu").exists()

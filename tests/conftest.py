"""Shared pytest configuration.

Markers:
  gpu   needs a CUDA device (runs the staged sm_100a tick kernels and the env
        kernels); everything else runs on CPU and covers the oracle, the host
        build of the product physics, the arena build, the C ABI library's
        exports and the multi-process host logic.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
TESTS = ROOT / "tests"
for p in (str(ROOT), str(TESTS)):
    if p not in sys.path:
        sys.path.insert(0, p)

from oracle import paths as _oracle_paths  # noqa: E402

REFERENCE = _oracle_paths.reference_dir()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


def _cuda_available() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _cuda_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def oracle_built() -> Path:
    """oracle/_ref/ built from the reference sources (here) or prebuilt (GPU box)."""
    ref = ROOT / "oracle" / "_ref"
    need = [ref / "libcarlref_cpu.so", ref / "libcarlref_ka.so", ref / "arena.obj"]
    if not all(p.exists() for p in need):
        if not _oracle_paths.reference_present():
            pytest.skip("oracle not built and the reference tree is absent")
        subprocess.run(["make", "-C", str(ROOT / "oracle"), "cpu", "arena"], check=True, capture_output=True)
    os.environ.setdefault("CARL_ARENA_OBJ", str(ref / "arena.obj"))
    return ref


@pytest.fixture(scope="session")
def arena_path(oracle_built) -> Path:
    return oracle_built / "arena.obj"

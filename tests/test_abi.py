"""The C ABI library: it loads, exports every entry point include/carlb.h
declares, and validates its arguments before touching a device."""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from carl_b200 import _build, capi

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "carlb.h"


@pytest.fixture(scope="module")
def lib():
    _build.build()
    return capi.load()


def declared_functions() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    text = re.sub(r"//[^\n]*", "", text)
    names = re.findall(r"\b(carlb_[a-z0-9_]+)\s*\(", text)
    return sorted(set(names))


def exported_symbols(path: Path) -> set[str]:
    out = subprocess.run(["nm", "-D", "--defined-only", str(path)], check=True, capture_output=True, text=True).stdout
    return {line.split()[-1] for line in out.splitlines() if line.strip()}


def test_header_declares_the_boundary():
    names = declared_functions()
    for required in ["carlb_create", "carlb_destroy", "carlb_env_step", "carlb_ticks", "carlb_reset",
                     "carlb_apply_reset_state", "carlb_set_ball", "carlb_set_car", "carlb_set_match_state",
                     "carlb_reset_boost_pads", "carlb_get_buffer", "carlb_stream", "carlb_last_error",
                     "carlb_read_field", "carlb_write_field"]:
        assert required in names


def test_library_exports_every_declared_symbol(lib):
    exported = exported_symbols(capi.library_path())
    missing = [n for n in declared_functions() if n not in exported]
    assert not missing, missing


def test_only_carlb_symbols_are_public(lib):
    exported = exported_symbols(capi.library_path())
    ours = {s for s in exported if s.startswith("carlb_")}
    assert ours == set(declared_functions())


def _create(lib, **kw):
    base = dict(n_sim=4, n_blue=1, n_orange=1, seed=0, frameskip=1, invert_orange=1, normalize=0,
                previous_controls=0, device=0, compat_flags=0, sim_offset=0)
    base.update(kw)
    cfg = capi.Config(*[base[f] for f, _ in capi.Config._fields_])
    h = ctypes.c_void_p()
    st = lib.carlb_create(ctypes.byref(cfg), ctypes.byref(h))
    return st, h, lib.carlb_last_error(None).decode()


@pytest.mark.parametrize("kw, needle", [
    (dict(n_sim=0), "n_sim"),
    (dict(n_blue=-1), "team"),
    (dict(n_blue=0, n_orange=0), "team"),
    (dict(n_blue=5), "at most 4"),
    (dict(frameskip=0), "frameskip"),
    (dict(sim_offset=-3), "sim_offset"),
])
def test_create_rejects_bad_config(lib, kw, needle):
    st, h, msg = _create(lib, **kw)
    assert st == capi.ERR_VALUE and not h.value
    assert needle in msg


def test_null_handles_fail_cleanly(lib):
    assert lib.carlb_ticks(None, 0, None, 1) == capi.ERR_VALUE
    assert lib.carlb_env_step(None, 0, None) == capi.ERR_VALUE
    assert lib.carlb_reset(None) == capi.ERR_VALUE
    assert lib.carlb_destroy(None) == capi.OK
    assert lib.carlb_create(None, None) == capi.ERR_VALUE


def test_action_mask_validates_before_launch(lib):
    """carlb_action_mask checks its arguments before any device work (no GPU needed)."""
    err = lambda: lib.carlb_last_error(None).decode()  # noqa: E731
    assert lib.carlb_action_mask(None, 0, 200, 0, None, None) == capi.OK  # nothing to do
    assert lib.carlb_action_mask(None, -1, 200, 0, None, None) == capi.ERR_VALUE
    assert "non-negative" in err()
    assert lib.carlb_action_mask(None, 4, 200, 0, None, None) == capi.ERR_VALUE
    assert "null" in err()
    assert lib.carlb_action_mask(16, 4, 200, 0, 18, None) == capi.ERR_VALUE
    assert "aligned" in err()
    assert lib.carlb_action_mask(16, 4, 36, 0, 16, None) == capi.ERR_VALUE
    assert "obs_dim" in err()
    # With previous controls the ego fields sit 8 values further from the end.
    assert lib.carlb_action_mask(16, 4, 44, 1, 16, None) == capi.ERR_VALUE


def test_create_without_a_device_reports_cuda_error(lib):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a device is present")
    st, h, msg = _create(lib)
    assert st == capi.ERR_CUDA and not h.value
    assert msg


def test_field_and_buffer_enums_match_the_header():
    text = HEADER.read_text()
    fields = [f for f in re.findall(r"\bCARLB_F_([A-Z0-9_]+)\s*=\s*(\d+)", text) if f[0] != "COUNT"]
    assert [n for n, _ in sorted(fields, key=lambda x: int(x[1]))] == capi.FIELDS
    bufs = [b for b in re.findall(r"\bCARLB_BUF_([A-Z_]+)\s*=\s*(\d+)", text) if b[0] != "COUNT"]
    assert len(bufs) == 12 and sorted(int(v) for _, v in bufs) == list(range(12))
    assert re.search(r"CARLB_SOURCE_LAGGED_LATERAL_FRICTION\s+(\d+)", text).group(1) == str(
        capi.SOURCE_LAGGED_LATERAL_FRICTION)

"""The C-ABI library loads without a GPU and exports every symbol the header declares."""

from __future__ import annotations

import re

import pytest

from fused_hoad import _native


def declared_functions() -> list[str]:
    text = _native.HEADER.read_text()
    return sorted(set(re.findall(r"\b(fhb_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_entry_points() -> None:
    names = declared_functions()
    for required in ("fhb_forward", "fhb_backward", "fhb_backward_workspace_bytes",
                     "fhb_poisson_step_gradients", "fhb_adam_step"):
        assert required in names


@pytest.mark.parametrize("name", declared_functions())
def test_library_exports_declared_symbol(name: str) -> None:
    lib = _native.library()
    assert hasattr(lib, name), f"{name} declared in the header but not exported"


def test_python_signatures_cover_the_header() -> None:
    assert set(declared_functions()) == set(_native._SIGNATURES)


def test_no_compute_without_gpu_and_clear_status_strings() -> None:
    lib = _native.library()
    assert lib.fhb_parameter_count() == 12737
    assert _native.status_string(0) == "ok"
    assert "sm_100" in _native.status_string(4)
    # argument validation happens before any device work
    assert lib.fhb_forward(None, None, None, None, 4, 9, None) == 1  # bad version
    assert lib.fhb_forward(None, None, None, None, -1, 2, None) == 1  # negative size
    assert lib.fhb_forward(None, None, None, None, 0, 2, None) == 0   # empty batch: no-op

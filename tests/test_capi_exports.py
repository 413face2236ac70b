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


def test_noalloc_backward_rejects_bad_arguments_before_any_device_work() -> None:
    """The workspace-free backward checks sizes, missing pointers and 4-byte alignment before
    it touches the device, so these calls return their codes on a host with no GPU."""
    lib = _native.library()
    good = 4096  # an aligned stand-in address: never dereferenced, the checks return first
    bad = 4098
    args = dict(coords=good, params=good, grad_u=good, grad_lap=good, grad_params=good,
                grad_coords=good)

    def call(n: int, **override) -> int:
        a = {**args, **override}
        return lib.fhb_backward_noalloc(a["coords"], a["params"], a["grad_u"], a["grad_lap"],
                                        a["grad_params"], a["grad_coords"], n, None)

    assert call(-1) == 1                      # negative size
    assert call(8, params=None) == 1          # no parameters
    assert call(8, grad_params=None) == 1     # nowhere to write the gradient
    assert call(8, coords=None) == 1          # points missing for a non-empty batch
    assert call(8, grad_lap=None) == 1        # upstream Laplacian gradient missing
    for name in args:                         # every pointer's alignment is checked
        assert call(8, **{name: bad}) == 2, name


def test_biharmonic_entry_validates_before_device_work() -> None:
    lib = _native.library()
    good, bad = 4096, 4098  # stand-in addresses, never dereferenced
    assert lib.fhb_forward_biharmonic(good, good, good, good, good, -1, None) == 1
    assert lib.fhb_forward_biharmonic(None, None, None, None, None, 0, None) == 0
    assert lib.fhb_forward_biharmonic(good, good, good, None, good, 8, None) == 1
    assert lib.fhb_forward_biharmonic(good, good, good, good, bad, 8, None) == 2

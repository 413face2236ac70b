"""Access to the compiled sm_100a extension (``fused_hoad._C``).

Mirrors the reference's ``src/fused_hoad/_extension.py:8-65``: same function names,
arguments, defaults and return shapes, so code written against the reference's Python API
runs unchanged. There is no CPU or PyTorch fallback: if the extension is missing, every
call raises.
"""

from __future__ import annotations

from types import ModuleType

from torch import Tensor

BUILD_HINT = (
    "The fused_hoad CUDA extension is not built. Build it in-tree with "
    "`python expanded-gpu-optimization_b200/build.py` (nvcc for sm_100a); the kernels need "
    "a B200 (sm_100) GPU to run."
)


def load_extension() -> ModuleType:
    """Return the compiled extension or raise an actionable error."""
    try:
        from fused_hoad import _C
    except ImportError as exc:
        raise RuntimeError(BUILD_HINT) from exc
    return _C


def extension_available() -> bool:
    """Return whether the compiled extension can be imported."""
    try:
        load_extension()
    except RuntimeError:
        return False
    return True


def fused_forward_laplacian(
    coordinates: Tensor, parameters: Tensor, version: int = 2, activation: str = "tanh"
) -> tuple[Tensor, Tensor]:
    """Evaluate the fixed MLP and its input Laplacian: ``(u [N,1], lap [N,1])``.

    ``version`` 0, 1, 2: the FP32 CUDA-core kernel with 32-, 128- and 64-point tiles (2 is
    the default, as in the reference). 3: the 3xFP16 tcgen05/TMEM tensor-core kernel; 4, 5:
    the 3xTF32 one; both hold the FP32 tolerance (the reference's single-TF32 v3-v5 did
    not). ``activation`` is ``"tanh"`` (the reference kernels') or ``"silu"`` (the other jet
    of the reference's PyTorch forward-Laplacian backend; versions 3-5 then run 3xTF32).
    """
    output, laplacian = load_extension().fused_forward_laplacian(
        coordinates, parameters, version, activation
    )
    return output, laplacian


def fused_forward_biharmonic(
    coordinates: Tensor, parameters: Tensor
) -> tuple[Tensor, Tensor, Tensor]:
    """``(u, lap, bilap)``, each ``[N, 1]``: the tanh MLP, its input Laplacian and its
    biharmonic (the Laplacian of the Laplacian), from one FP32 CUDA-core kernel that carries
    a nine-component jet per neuron. Not part of the reference's extension (it computes the
    biharmonic only by nested autograd)."""
    u, lap, bilap = load_extension().fused_forward_biharmonic(coordinates, parameters)
    return u, lap, bilap


def fused_forward_laplacian_backward(
    coordinates: Tensor,
    parameters: Tensor,
    grad_output: Tensor,
    grad_laplacian: Tensor,
    version: int = 6,
    activation: str = "tanh",
) -> tuple[Tensor, Tensor]:
    """Return ``(grad_parameters [12737], grad_coordinates [N,2])``.

    Version 6 (the default) runs the tensor-core adjoint kernel, 1..5 the FP32 CUDA-core one;
    both reduce in a fixed order, so the gradients are bitwise reproducible. SiLU runs the
    FP32 kernel for every version.
    """
    grad_parameters, grad_coordinates = load_extension().fused_forward_laplacian_backward(
        coordinates,
        parameters,
        grad_output.reshape(-1).contiguous(),
        grad_laplacian.reshape(-1).contiguous(),
        version,
        activation,
    )
    return grad_parameters, grad_coordinates


def fused_forward_laplacian_host(
    coordinates: Tensor,
    parameters: Tensor,
    version: int = 3,
    output: Tensor | None = None,
    laplacian: Tensor | None = None,
    activation: str = "tanh",
) -> tuple[Tensor, Tensor]:
    """``(u, lap)`` for points in pinned host memory, without staging copies.

    Pinned host memory is device-addressable, so the kernel reads the points and writes the
    results over the host link while it computes. The results are pinned host tensors,
    valid once the current CUDA stream of ``parameters``' device has completed.
    """
    u, lap = load_extension().fused_forward_laplacian_host(
        coordinates, parameters, version, output, laplacian, activation
    )
    return u, lap


# Bits of the device status word (include/fused_hoad_b200.h FHB_STATUS_*).
STATUS_STAGE_TIMEOUT = 0x1
STATUS_MMA_TIMEOUT = 0x2
STATUS_PEER_TIMEOUT = 0x4


def read_device_status(device: int) -> int:
    """Read and clear device ``device``'s status word (synchronises that device).

    Kernels whose bounded waits give up set bits here instead of hanging or faulting:
    ``STATUS_STAGE_TIMEOUT`` (parameter staging), ``STATUS_MMA_TIMEOUT`` (tensor-core
    pipeline), ``STATUS_PEER_TIMEOUT`` (a peer rank's gradient never arrived). Zero means
    every wait since the last read completed.
    """
    return int(load_extension().read_device_status(int(device)))

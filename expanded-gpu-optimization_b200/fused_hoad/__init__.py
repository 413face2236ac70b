"""fused_hoad on B200: the forward-Laplacian hot path of the fixed 2->64x4->1 tanh MLP.

Drop-in for the reference package's fused path: ``fused_hoad._C`` keeps the
torch.utils.cpp_extension op contract (``fused_forward_laplacian``,
``fused_forward_laplacian_backward``), the flat 12,737-float parameter ABI, the autograd
glue and the ``fused_cuda*`` backend names, on hand-written sm_100a kernels. There is no
CPU or PyTorch fallback: calls raise if the extension is missing.
"""

from fused_hoad._extension import (
    extension_available,
    fused_forward_biharmonic,
    fused_forward_laplacian,
    fused_forward_laplacian_backward,
    fused_forward_laplacian_host,
    load_extension,
    read_device_status,
)
from fused_hoad.backends import BACKENDS, FIXED_CONTRACT_BACKENDS, get_backend
from fused_hoad.backends.fused import FusedForwardLaplacian, fused_laplacian
from fused_hoad.distributed import PeerExchange, shard_range
from fused_hoad.parameters import (
    POISSON_PARAMETER_COUNT,
    POISSON_PARAMETER_LAYOUT,
    bind_model_to_flat,
    pack_poisson_parameters,
    unpack_poisson_parameters,
)
from fused_hoad.problem import (
    DEFAULT_POISSON_MLP,
    MLPConfig,
    build_mlp,
    manufactured_solution,
    manufactured_source,
    uniform_points,
)
from fused_hoad.training import PoissonTrainer, cuda_graph_step

__all__ = [
    "BACKENDS",
    "DEFAULT_POISSON_MLP",
    "FIXED_CONTRACT_BACKENDS",
    "FusedForwardLaplacian",
    "MLPConfig",
    "POISSON_PARAMETER_COUNT",
    "POISSON_PARAMETER_LAYOUT",
    "PeerExchange",
    "PoissonTrainer",
    "bind_model_to_flat",
    "build_mlp",
    "cuda_graph_step",
    "extension_available",
    "fused_forward_biharmonic",
    "fused_forward_laplacian",
    "fused_forward_laplacian_backward",
    "fused_forward_laplacian_host",
    "fused_laplacian",
    "get_backend",
    "load_extension",
    "manufactured_solution",
    "manufactured_source",
    "pack_poisson_parameters",
    "read_device_status",
    "shard_range",
    "uniform_points",
    "unpack_poisson_parameters",
]
__version__ = "0.1.0"

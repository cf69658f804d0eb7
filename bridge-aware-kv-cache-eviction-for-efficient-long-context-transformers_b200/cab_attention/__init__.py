"""CAB-Attention prefill path on B200 (sm_100a).

Public surface (the reference's import paths, ``README.md:77,117``):
``from cab_attention import CABAttention``;
``from cab_attention.coarse_predictor import CoarseCurvaturePredictor``;
``cab_attention.kernels.coarsening``, ``cab_attention.kernels.frc_kernel`` and
``cab_attention.kernels.sparse_attention`` for the individual stages;
``cab_attention.prefill_from_host`` for the whole path over page-locked host tensors;
``torch.ops.cab.*`` (registered on import, ``cab_attention.ops``) for the stages as PyTorch
operators with fake implementations. Every op runs the sm_100a kernels of
``libcab_b200.so`` through its C ABI (``include/cab_capi.h``).
"""

__version__ = "1.0.0"

from .cab_attention import CABAttention  # noqa: E402
from .coarse_predictor import CoarseCurvaturePredictor  # noqa: E402
from .host_prefill import prefill_from_host  # noqa: E402
from . import ops  # noqa: E402,F401  (registers torch.ops.cab.*)

__all__ = ["CABAttention", "CoarseCurvaturePredictor", "prefill_from_host"]

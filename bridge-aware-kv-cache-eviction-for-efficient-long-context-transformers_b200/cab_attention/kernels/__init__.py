"""Stage-level ops of the CAB prefill path (each backed by one C-ABI entry point)."""

from .coarsening import coarsen_max_l2, coarsen_qk_max_l2, coarsen_qk_max_l2_pytorch  # noqa: F401
from .frc_kernel import (block_max_pool, compute_block_frc, generate_block_mask,  # noqa: F401
                         keep_count, topk_blocks, visualize_frc_statistics)
from .sparse_attention import block_sparse_attention  # noqa: F401
from .frc_triton import compute_frc, compute_frc_pytorch, compute_frc_triton  # noqa: F401
from .flash_attention_accumulate import (flash_attention_forward,  # noqa: F401
                                         flash_attention_with_cumulative_scores)

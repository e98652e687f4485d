"""strata_mlx_b200: strata-mlx's quantized-expert hot path (the MoE matmuls straight from GGUF blocks, with the
router, top-k and combine around them) rebuilt for the B200.

    strata_mlx_b200.blocks   the call surface of strata_mlx/blocks.py
    strata_mlx_b200.fused    the router / top_k / moe_combine of strata_mlx/fused.py, and the decode block
    strata_mlx_b200.ep       the block expert-parallel over GPUs: pair outputs stored into the token owner's
                             memory over NVLink (peer stores), or NCCL all-gather + all-reduce
    strata_mlx_b200.paged    experts within a device-memory budget, read from the GGUF file as routes ask
                             (strata_mlx/paged.py)
    include/strata_cuda.h    the C ABI of libstrata_cuda.so underneath

The package is importable without a GPU; the kernels need one (sm_100a).
"""

from ._lib import check_device_errors, load  # noqa: F401

__all__ = ["blocks", "fused", "check_device_errors", "load"]

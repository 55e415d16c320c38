"""B200-native (sm_100a) FP8 block-scaled MoE hot path of GLM-5.3-Flash.

Drop-in counterpart of the reference operator layer (``glm53_flash_mlx.fp8``,
``.packed``, ``.grouped_fp8``, ``.ownership``, ``.abi`` and the FP32 router of
``.patch``) over PyTorch tensors and hand-written CUDA behind a C ABI
(``include/glm53_b200.h``).
"""

from .abi import (  # noqa: F401
    GROUPED_KERNEL_ABI,
    GROUPED_MEASURED_CROSSOVER_ROUTES,
    GROUPED_MIN_ROUTES,
    KERNEL_ABI_VERSION,
    PACKED_DECODE_KERNEL_ABI,
    PACKED_EXPERT_BANK_ABI,
)
from .checkpoint import (  # noqa: F401
    CheckpointIndex,
    load_packed_bank,
    load_packed_moe,
    load_router,
    load_shared_expert,
)
from .fp8 import BlockFP8Linear, DirectFP8Expert, DirectFP8MoE, block_fp8_linear  # noqa: F401
from .grouped_fp8 import (  # noqa: F401
    SortedGroupedFP8MoE,
    activate_gate_up,
    build_grouped_tile_plan,
    build_route_plan,
    grouped_fp8_linear,
    grouped_moe,
    restore_and_reduce,
)
from .packed import PackedFP8ExpertBank, PackedFP8MoE, packed_decode_moe  # noqa: F401
from .router import Float32Gate, router_topk  # noqa: F401
from .hyper_connection import FFNBoundary, HyperConnection, RMSNorm, hc_expand, rms_norm  # noqa: F401
from .dsa_output import DSAOutputProjection, head_major_to_rows  # noqa: F401

"""Revisioned identities of the B200 kernels and the reference's constants.

Counterpart of glm53_flash_mlx/abi.py:3-15.  The B200 kernel ABI strings name
the numerics that change results (decode table, accumulation, rounding) so
that any cache keyed on them is invalidated when those change.
"""

# Kept from the reference (glm53_flash_mlx/abi.py:5-6): the measured decode /
# grouped crossover and the grouped-path threshold in routes.
GROUPED_MEASURED_CROSSOVER_ROUTES = 16
GROUPED_MIN_ROUTES = 256

KERNEL_ABI_VERSION = "glm53-b200-fp8-v1-e4m3lut480-block128-gemv-f32-tc-bf16-scalefold"
GROUPED_KERNEL_ABI = "glm53-b200-grouped-fp8-v1-sorted-routes-tile128-bf16mma-swiglu-epilogue"
PACKED_EXPERT_BANK_ABI = "glm53-packed-expert-bank-v2-gate-up-output-major-row-contiguous"
PACKED_DECODE_KERNEL_ABI = (
    "glm53-b200-packed-selected8-fp8-v1"
    "-exact-bf16-swiglu"
    "-fp32-slot-ordered-reduction"
    "-shared-as-ninth-slot"
)
ROUTER_ABI = "glm53-b200-router-fp32-v1-sigmoid-bias-topk-desc-lowid"

"""B200-native NVFP4 block-scaled grouped GEMM.

Public API:
  custom_kernel(data) / solve(data)   harness entry points (submission.py:788-891)
  grouped_gemm(...)                   explicit grouped launch (blocked scales)
  GroupedGemmPlan(...).run()          the same launch prepared once, run repeatedly
  sf_to_blocked / plain_to_blocked    scale-factor layout conversion
  quantize / global_scale_for         NVFP4 activation quantiser (bf16/fp16 -> A operand)
  moe                                 MoE block: route, dispatch+quantise, gated GEMM, down GEMM, combine
  workloads                           seeded synthetic benchmark problems
  expert_parallel                     expert sharding + output all-gather
"""
from . import _native, expert_parallel, layout, moe, quantize as quantize_module, workloads
from ._native import Nvfp4Error, load_library
from .interface import (GroupedGemmPlan, check_device_errors, custom_kernel, grouped_gemm,
                        grouped_gemm_segments, input_t, output_t, solve)
from .layout import (blocked_as_reordered, blocked_sf_bytes, blocked_to_plain, plain_to_blocked,
                     sf_to_blocked)
from .quantize import global_scale_for, quantize

__all__ = [
    "GroupedGemmPlan", "Nvfp4Error", "blocked_as_reordered", "blocked_sf_bytes", "blocked_to_plain",
    "check_device_errors", "custom_kernel", "expert_parallel", "global_scale_for", "grouped_gemm",
    "grouped_gemm_segments",
    "input_t", "moe", "quantize",
    "layout", "load_library", "output_t", "plain_to_blocked", "sf_to_blocked", "solve",
    "workloads",
]

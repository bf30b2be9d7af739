"""spec_ep: a Blackwell-native (sm_100a) MoE expert-parallel runtime.

Public entry points:
  * ``spec_ep.rbd`` - redundancy-bypassing dispatch/combine API over torch.distributed
    (the reference-compatible plan/dispatch/combine functions).
  * ``spec_ep.parallel`` - fused expert-parallel dispatch/combine over NVLink P2P,
    the placement planner and the two-stage hierarchical path.
  * ``spec_ep.models`` - Qwen3-MoE-shaped decoder built on the fused ops.
"""
__version__ = "0.1.0"

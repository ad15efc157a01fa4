"""Multi-GPU execution on one node: process groups, a symmetric peer-memory heap with
bounded-wait flag barriers, the P2P all-reduce, and expert-parallel MoE whose token
dispatch and combine are fused with the grouped GEMMs (NCCL versions kept as the
baseline)."""
from .groups import init_distributed, rank_info

__all__ = ["init_distributed", "rank_info"]

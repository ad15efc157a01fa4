"""Expert placement across tiers: GPU-resident layers, a hot-expert pool per layer,
the streamed prefill ring, and the C++ CPU expert engine for everything else."""
from .policy import load_pin_table, plan_swap, save_pin_table, table_from_counts

__all__ = ["load_pin_table", "plan_swap", "save_pin_table", "table_from_counts", "TieredExperts", "plan"]


def __getattr__(name):
    if name == "TieredExperts":
        from .executor import TieredExperts
        return TieredExperts
    if name == "plan":
        from .planner import plan
        return plan
    raise AttributeError(name)

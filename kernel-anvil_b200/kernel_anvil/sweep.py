"""Guided config sweep: candidate launch configs from a bottleneck report.

The reference builds Triton candidates per classification (kernel_anvil/sweep.py:7-81);
here the candidates are the MMVQ launch knobs themselves -- {"nwarps", "rows_per_block"}
-- so the sweep tunes the production kernel.  Runner scripts with other knobs can pass
their own ``param_space``.  The cartesian product is taken in key order, the baseline is
put first when given, and the list is capped at ``max_configs`` (same policy as the
reference).  ``launch_overhead`` yields no candidates: such kernels need fusion, not tuning.
"""
from __future__ import annotations

from itertools import product

from kernel_anvil.analyze import BottleneckReport

GRID_NWARPS = (1, 2, 4, 8)
GRID_RPB = (1, 2, 4)

PARAM_SPACES: dict[str, dict[str, list] | None] = {
    "bandwidth_bound": {"nwarps": [2, 4, 8], "rows_per_block": [1, 2, 4, 8]},
    "occupancy_limited_regs": {"nwarps": [1, 2, 4], "rows_per_block": [1, 2]},
    "occupancy_limited_smem": {"nwarps": [1, 2, 4, 8], "rows_per_block": [1, 2]},
    "register_spill": {"nwarps": [1, 2], "rows_per_block": [1]},
    "compute_bound": {"nwarps": [4, 8], "rows_per_block": [1, 2, 4]},
    "launch_overhead": None,
}


def _get_param_space(classification: str) -> dict[str, list] | None:
    return PARAM_SPACES.get(classification)


def generate_configs(report: BottleneckReport, baseline_config: dict | None = None,
                     max_configs: int = 20, param_space: dict[str, list] | None = None) -> list[dict]:
    space = param_space if param_space is not None else _get_param_space(report.classification)
    if space is None:
        return []
    keys = list(space)
    configs = [dict(zip(keys, combo)) for combo in product(*space.values())]
    if baseline_config is not None and baseline_config not in configs:
        configs.insert(0, baseline_config)
    return configs[:max_configs]


def grid_configs(nwarps=GRID_NWARPS, rpb=GRID_RPB) -> list[dict]:
    """The autoforge grid (kernel_anvil/autoforge.py:254-257): every nwarps x rows_per_block."""
    return [{"nwarps": nw, "rows_per_block": r} for nw in nwarps for r in rpb]

"""Bottleneck classification from kernel profile metrics.

Same decision order as the reference (kernel_anvil/analyze.py:29-131) -- spills, then
register-limited occupancy, then shared-memory-limited occupancy, then bandwidth bound
(> 60% of peak), then launch overhead, else compute bound -- with NVIDIA resources
(registers and shared memory instead of VGPRs and LDS) and recommendations phrased in
the MMVQ knobs (nwarps, rows_per_block).  When ncu DRAM counters are present, achieved
bandwidth is taken from them instead of algorithmic bytes.
"""
from __future__ import annotations

from dataclasses import dataclass, field

from kernel_anvil.specs import GpuSpec

LAUNCH_US = 5.0  # below this a B200 kernel is dominated by launch and ramp


@dataclass
class ProfileMetrics:
    duration_ns: float
    regs_per_thread: int = 0
    smem_bytes: int = 0
    spill_bytes: int = 0          # local memory per thread (register spills)
    bandwidth_gbs: float = 0.0
    occupancy_pct: float = 0.0
    limiting_factor: str = "unknown"
    threads_per_block: int = 128
    dram_bytes: int | None = None  # ncu dram__bytes_read.sum + dram__bytes_write.sum

    # reference field names
    @property
    def vgpr_count(self) -> int:
        return self.regs_per_thread

    @property
    def lds_bytes(self) -> int:
        return self.smem_bytes

    @property
    def scratch_bytes(self) -> int:
        return self.spill_bytes

    @property
    def threads_per_wg(self) -> int:
        return self.threads_per_block


@dataclass
class BottleneckReport:
    classification: str
    severity: float
    limiting_factor: str
    directions: list[str] = field(default_factory=list)


def classify(metrics: ProfileMetrics, gpu_spec: GpuSpec) -> BottleneckReport:
    if metrics.spill_bytes > 0:
        return BottleneckReport("register_spill", 1.0, "local_memory", [
            "Lower rows_per_block (fewer accumulators per thread)",
            "Lower ncols per launch or split the batch",
            "Check -Xptxas -v for the spilling instantiation",
        ])
    occ, factor = metrics.occupancy_pct, metrics.limiting_factor
    if metrics.regs_per_thread > 0 or metrics.smem_bytes > 0:
        occ, factor = gpu_spec.occupancy(metrics.regs_per_thread, metrics.smem_bytes,
                                         metrics.threads_per_block)
    if occ < 50.0 and factor == "regs":
        return BottleneckReport("occupancy_limited_regs", 1.0 - occ / 50.0, "regs", [
            "Lower rows_per_block to cut per-thread accumulators",
            "Lower nwarps so more CTAs fit per SM",
        ])
    if occ < 50.0 and factor == "smem":
        return BottleneckReport("occupancy_limited_smem", 1.0 - occ / 50.0, "smem", [
            "Lower rows_per_block (smaller weight tiles per stage)",
            "Fewer activation columns per launch",
        ])
    bw = metrics.bandwidth_gbs
    if metrics.dram_bytes and metrics.duration_ns > 0:
        bw = metrics.dram_bytes / metrics.duration_ns
    ratio = bw / gpu_spec.peak_bandwidth_gbs if gpu_spec.peak_bandwidth_gbs > 0 else 0.0
    if ratio > 0.6:
        return BottleneckReport("bandwidth_bound", min(1.0, (ratio - 0.6) / 0.4), "memory_bandwidth", [
            "Raise rows_per_block or nwarps to keep more weight bytes in flight",
            "Fuse consumers of the same activation (gate+up) to share its staging",
            "Chain GEMVs under programmatic dependent launch to hide ramp and tail",
        ])
    if metrics.duration_ns < LAUNCH_US * 1000:
        return BottleneckReport("launch_overhead", 0.5, "launch", [
            "Capture the chain in a CUDA graph with programmatic dependent launch",
            "Fuse with adjacent kernels (quantize prologue, gate+up)",
        ])
    return BottleneckReport("compute_bound", 0.2, "compute", [
        "Raise nwarps for more issue slots",
        "Use the tensor-core path for batched columns",
    ])

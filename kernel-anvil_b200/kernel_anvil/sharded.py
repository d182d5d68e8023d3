"""Row-sharded GEMV chain across GPUs: each rank multiplies its row slice of every matrix
and the fp32 output slices are all-gathered over NVLink with NCCL after every GEMV.

Rows of a GEMV are independent and a GGUF block never spans rows, so the shards are exact
(chains.shard_rows).  The all-gather is the one exchange step: the next layer needs the
whole output vector.  One step is recorded eagerly and captured, NCCL included, into a
torch CUDA graph by the caller.
"""
from __future__ import annotations

import torch

from kernel_anvil import mmvq as ops


class ShardedStep:
    """One token of a DeviceChain built with world > 1, plus per-GEMV all-gathers."""

    def __init__(self, dc, dist, group=None):
        self.dc, self.dist, self.group = dc, dist, group
        self.full = []
        for gm, y, (r0, r1) in zip(dc.spec.gemvs, dc.outputs, dc.rows):
            if gm.nrows % dc.world:
                raise ValueError(f"{gm.name}: {gm.nrows} rows do not split evenly over {dc.world} ranks")
            self.full.append(torch.empty(dc.world * y.numel(), dtype=torch.float32, device=y.device))

    def eager(self) -> None:
        dc = self.dc
        seen: set[str] = set()
        for gm, W, y, full, (r0, r1) in zip(dc.spec.gemvs, dc.weights, dc.outputs, self.full, dc.rows):
            if gm.input not in seen:
                ops.quantize_q8_1(dc.x[gm.input], out=dc.xq[gm.input], pdl=True)
                seen.add(gm.input)
            ops.mmvq(W, gm.qt, dc.xq[gm.input], nrows=r1 - r0, K=gm.K, ncols=dc.ncols, out=y, pdl=True)
            self.dist.all_gather_into_tensor(full, y.view(-1), group=self.group)

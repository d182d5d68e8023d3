"""Oracle check of a persistent chain's outputs (a test helper, not a test module).

Each GEMV is checked on its own: its input is rebuilt on the host from what the GPU
actually produced (the fixed fp32 vector, or the gathered output of the producer GEMV,
quantised with the oracle's chained-input rule), and its output rows are compared with the
oracle's float64 result within the y tolerance.  Errors therefore do not compound along the
chain, and a wrong exchange (a missing or stale row) shows up as a NaN or a mismatch."""
from __future__ import annotations

import numpy as np

from kernel_anvil.chains import spec_index
from oracle import oracle

Y_TOL = 1e-3  # max |y - y_ref| / max |y_ref|


def chain_inputs_q8_1(dc, outs: dict[int, np.ndarray]) -> dict[str, tuple]:
    """(blocks, column scales or None) of every activation of the chain as the oracle computes
    them from the GPU's own fixed inputs and outputs."""
    spec = dc.spec
    xq = {}
    for act in spec.inputs:
        src = spec.sources.get(act) if dc.dataflow else None
        if src is None:
            xq[act] = (oracle.quantize_q8_1(dc.x[act].cpu().numpy()), None)
        else:
            xq[act] = oracle.quantize_q8_1_chained(outs[dc.pidx[spec_index(spec, src[1])]])
    return xq


def check_chain(dc, rows_only: bool = True) -> float:
    """Checks every GEMV of a persistent DeviceChain (this rank's rows); returns the worst
    normalised error."""
    spec = dc.spec
    outs = {j: dc.pchain.output(j).cpu().numpy() for j in range(dc.pchain.n_gemv)}
    for j, o in outs.items():
        assert not np.isnan(o).any(), f"chain GEMV {j}: values missing (stale or unwritten words)"
    xq = chain_inputs_q8_1(dc, outs)
    worst = 0.0
    for i, gm in enumerate(spec.gemvs):
        j = dc.pidx[i]
        item = dc._items[j]
        if item[0] != i:
            continue  # the up half of a gate/up pair
        r0, r1 = dc.rows[i]
        W = dc.weights[i].cpu().numpy()
        blocks, scale = xq[gm.input]
        if len(item) == 2:
            W2 = dc.weights[i + 1].cpu().numpy()
            ref = (oracle.mmvq_glu(gm.qt, W, W2, blocks, r1 - r0, gm.K) if scale is None else
                   oracle.mmvq_glu_chained(gm.qt, W, W2, blocks, scale, r1 - r0, gm.K))
        else:
            ref = (oracle.mmvq(gm.qt, W, blocks, r1 - r0, gm.K, dc.ncols) if scale is None else
                   oracle.mmvq_chained(gm.qt, W, blocks, scale, r1 - r0, gm.K, dc.ncols))
        got = outs[j][:, r0:r1]
        err = oracle.max_rel_err(got, ref)
        assert err <= Y_TOL, f"{gm.name} ({gm.qt} {gm.nrows}x{gm.K}): error {err}"
        worst = max(worst, err)
    return worst

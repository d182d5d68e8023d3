"""Runner script (setup / run / reference / DATA_BYTES / BASELINE_CONFIG) for one Q4_K MMVQ
GEMV of 28672 x 8192 (a Llama-3-70B ffn_gate / ffn_up shape, 132 MB of weights: long enough
to be bandwidth-bound even as a cold, serialised launch under ncu).  Records
tests/golden/ncu_mmvq_q4k_28672x8192.csv with:

  ncu --metrics gpu__time_duration.sum,dram__bytes_read.sum,dram__bytes_write.sum \\
      --clock-control none --csv -k regex:mmvq -c 3 \\
      python -m kernel_anvil.profile --run-runner tests/golden/runner_mmvq_q4k_28672x8192.py \\
      --launches 3
"""
import torch

from kernel_anvil import mmvq as ops
from kernel_anvil.quants import gemv_bytes, make_weights_device

N, K = 28672, 8192
DATA_BYTES = gemv_bytes("Q4_K", N, K)
BASELINE_CONFIG = {"quant": "Q4_K", "n": N, "k": K, "nwarps": 0, "rows_per_block": 0}


def setup():
    W = make_weights_device("Q4_K", N, K, seed=5)
    g = torch.Generator(device="cuda")
    g.manual_seed(6)
    x = torch.randn((1, K), generator=g, device="cuda")
    return {"W": W, "xq": ops.quantize_q8_1(x), "y": torch.empty((1, N), device="cuda")}


def run(inputs, quant="Q4_K", n=N, k=K, nwarps=0, rows_per_block=0, **_):
    return ops.mmvq(inputs["W"], quant, inputs["xq"], ncols=1, nwarps=nwarps,
                    rows_per_block=rows_per_block, out=inputs["y"])


def reference(inputs):
    return ops.mmvq(inputs["W"], "Q4_K", inputs["xq"], ncols=1, nwarps=4, rows_per_block=1)

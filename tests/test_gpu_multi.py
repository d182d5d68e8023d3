"""Row-sharded persistent chain on 2 GPUs: every rank writes its output rows into every
rank's buffer (CUDA IPC peer stores) and the group barriers count the CTAs of both ranks.
The gathered outputs must equal each rank's own single-GEMV results, concatenated.

Runs as two spawned processes, one per GPU (NCCL only for set-up and the check); skipped
with fewer than two GPUs."""
import os
import socket
from datetime import timedelta

import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    import sys
    from pathlib import Path

    repo = Path(__file__).resolve().parent.parent
    for p in (repo / "kernel-anvil_b200", repo):
        sys.path.insert(0, str(p))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    from kernel_anvil import mmvq as ops
    from kernel_anvil.chains import DeviceChain, get_chain
    from kernel_anvil.pchain import take_status

    ok = True
    try:
        spec = get_chain("qwen3_8b").head(14)
        dc = DeviceChain(spec, rank=rank, world=world, executor="persistent", dist=dist)
        for _ in range(3):  # three tokens: the cross-rank barrier epochs advance
            dc.launch()
        torch.cuda.synchronize()
        dist.barrier()
        ok &= take_status() == 0
        for i, gm in enumerate(spec.gemvs):
            rpb, _ = dc.pchain.gemv_shape(i)
            r0, r1 = dc.rows[i]
            local = ops.mmvq(dc.weights[i], gm.qt, ops.quantize_q8_1(dc.x[gm.input]), nrows=r1 - r0,
                             K=gm.K, rows_per_block=rpb).view(-1)
            parts = [torch.empty(gm.nrows // world, device="cuda") for _ in range(world)]
            dist.all_gather(parts, local.contiguous())
            want = torch.cat(parts)
            got = dc.outputs[i].view(-1)
            if not torch.allclose(got, want, rtol=1e-5, atol=1e-5 * float(want.abs().max())):
                ok = False
        dist.barrier()
        dc.close()
    finally:
        Path(out_dir, f"rank{rank}.txt").write_text("ok" if ok else "fail")
        dist.destroy_process_group()


def test_sharded_persistent_chain_two_gpus(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.start_processes(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    assert [(tmp_path / f"rank{r}.txt").read_text() for r in range(2)] == ["ok", "ok"]

"""Row-sharded persistent chain on 2 GPUs: every rank writes its output rows, as flagged
words, into every rank's buffer (CUDA IPC peer stores), and each chained group reads the
gathered output of its producer as the words arrive.

Checks, on every rank: the gathered outputs of every GEMV hold no stale or missing value;
this rank's rows of every GEMV match the oracle computed from the gathered input (the
fixed vector, or the producer's gathered output under the chained-input rule); and the
gathered vectors are identical on both ranks (checksums exchanged once).  Every rank takes
the same collective steps whatever its local checks find.  Runs as two spawned processes,
one per GPU (NCCL with NVLS off, only for set-up and the comparison); skipped with fewer
than two GPUs."""
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


def _worker(rank, world, port, out_dir, spec_name, ngemv):
    import hashlib
    import sys
    from pathlib import Path

    repo = Path(__file__).resolve().parent.parent
    for p in (repo / "kernel-anvil_b200", repo, repo / "tests"):
        sys.path.insert(0, str(p))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    from chain_oracle import check_chain
    from kernel_anvil.chains import DeviceChain, get_chain
    from kernel_anvil.pchain import take_status

    status, sums, dc = "ok", [], None
    try:
        spec = get_chain(spec_name).head(ngemv)
        dc = DeviceChain(spec, rank=rank, world=world, executor="persistent", dist=dist, seed=0)
        for _ in range(3):  # three tokens: epochs 1..3, both output parities
            dc.launch()
        torch.cuda.synchronize()
        st = take_status()
        if st:
            status = f"device status {st}"
        sums = [hashlib.sha1(dc.pchain.output(j).cpu().numpy().tobytes()).hexdigest()
                for j in range(dc.pchain.n_gemv)]
        try:
            worst = check_chain(dc)
            if status == "ok":
                status = f"ok {worst:.2e}"
        except AssertionError as e:
            status = f"fail: {e}"
    except Exception as e:  # noqa: BLE001 -- reported, and the collectives below still run
        status = f"error: {type(e).__name__}: {e}"
    finally:
        got = [None] * world
        dist.all_gather_object(got, sums)
        if status.startswith("ok") and any(g != sums for g in got):
            status = "fail: gathered outputs differ between ranks"
        dist.barrier()
        if dc is not None:
            dc.close()
        Path(out_dir, f"rank{rank}.txt").write_text(status)
        dist.destroy_process_group()


@pytest.mark.timeout(600)
@pytest.mark.parametrize("spec_name,ngemv", [("qwen3_8b", 15), ("llama3_70b", 8)])
def test_sharded_dataflow_chain_two_gpus(tmp_path, spec_name, ngemv):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.start_processes(_worker, args=(2, _free_port(), str(tmp_path), spec_name, ngemv), nprocs=2,
                       join=True, start_method="spawn")
    res = [(tmp_path / f"rank{r}.txt").read_text() for r in range(2)]
    assert all(r.startswith("ok") for r in res), res

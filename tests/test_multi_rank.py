"""Row-sharded GEMV over world_size 2 (gloo on CPU): every rank computes its row slice with
the oracle, the slices are all-gathered, and the gathered vector equals the one-rank result
bit for bit (rows are independent and a block never spans rows).  Also covers the shard
partition itself and a rank that fails before the gather."""
import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from kernel_anvil.chains import get_chain, shard_rows


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, qt, nrows, K, fail_rank, out_dir):
    import sys
    from pathlib import Path

    repo = Path(__file__).resolve().parent.parent
    for p in (repo / "kernel-anvil_b200", repo):
        sys.path.insert(0, str(p))
    import torch

    from kernel_anvil.chains import shard_rows as shard
    from kernel_anvil.quants import make_activation, make_weights
    from oracle import oracle

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    try:
        W = make_weights(qt, nrows, K, seed=3)   # every rank draws the same matrix
        xq = oracle.quantize_q8_1(make_activation(K, seed=4))
        r0, r1 = shard(nrows, rank, world)
        if rank == fail_rank:
            raise RuntimeError("rank failed before its gather")
        y = oracle.mmvq(qt, W[r0:r1], xq, r1 - r0, K)
        # uneven shards: gather padded slices, then cut each to its own length
        pad = -(-nrows // world)
        buf = torch.zeros(pad, dtype=torch.float32)
        buf[: r1 - r0] = torch.from_numpy(np.ascontiguousarray(y, dtype=np.float32).reshape(-1))
        parts = [torch.zeros(pad, dtype=torch.float32) for _ in range(world)]
        dist.all_gather(parts, buf)
        full = np.concatenate([parts[r][: shard(nrows, r, world)[1] - shard(nrows, r, world)[0]].numpy()
                               for r in range(world)])
        np.save(os.path.join(out_dir, f"rank{rank}.npy"), full)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("qt,nrows,K", [("Q4_K", 96, 512), ("Q6_K", 77, 256), ("Q8_0", 130, 64)])
def test_row_sharded_allgather_matches_single_rank(tmp_path, qt, nrows, K):
    from kernel_anvil.quants import make_activation, make_weights
    from oracle import oracle

    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), qt, nrows, K, -1, str(tmp_path)),
                       nprocs=world, join=True, start_method="spawn")
    W = make_weights(qt, nrows, K, seed=3)
    ref = oracle.mmvq(qt, W, oracle.quantize_q8_1(make_activation(K, seed=4)), nrows, K).reshape(-1)
    for r in range(world):
        got = np.load(tmp_path / f"rank{r}.npy")
        assert np.array_equal(got, ref.astype(np.float32))


def test_rank_failure_is_reported(tmp_path):
    """Rank 1 raises before the gather: the launcher reports the failure; rank 0's gather
    ends with an error through the process-group timeout instead of waiting forever."""
    with pytest.raises(Exception):
        mp.start_processes(_worker, args=(2, _free_port(), "Q8_0", 64, 64, 1, str(tmp_path)),
                           nprocs=2, join=True, start_method="spawn")
    assert not (tmp_path / "rank1.npy").exists()


@pytest.mark.parametrize("world", [2, 3, 4, 8])
def test_shard_rows_partition(world):
    for nrows in (1, 7, 128, 1024, 151936, 28672):
        spans = [shard_rows(nrows, r, world) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == nrows
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
        sizes = [b - a for a, b in spans]
        assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("name", ["qwen3_8b", "llama3_70b"])
def test_chain_rows_split_evenly_over_8(name):
    """The sharded bench splits every matrix of these chains evenly at 2, 4 and 8 ranks."""
    for g in get_chain(name).gemvs:
        for world in (2, 4, 8):
            assert g.nrows % world == 0, (g.name, world)


@pytest.mark.parametrize("name,pairs", [("qwen3_8b", 36), ("llama3_70b", 80), ("qwen3_0_6b", 28),
                                        ("qwen35_27b", 0)])
def test_gate_up_pairs_found(name, pairs):
    """Every decoder layer's ffn_gate/ffn_up pair is recognised for the gate/up launch
    (16-byte rows: Q4_K always, Q8_0 at K = 1024), and nothing else is."""
    from kernel_anvil.chains import is_gate_up

    g = get_chain(name).gemvs
    found = [i for i in range(len(g) - 1) if is_gate_up(g[i:i + 2])]
    assert len(found) == pairs
    assert all(g[i].name.endswith("ffn_gate") for i in found)
    assert not is_gate_up(g[:2]) and not is_gate_up(g[:3])

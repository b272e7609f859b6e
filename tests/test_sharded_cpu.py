"""Column sharding on CPU ranks (gloo, world size 2 and 3): shard ranges, gather layout, failures.

Each rank computes its rows of the projection with the CPU oracle, the ranks
all-gather the padded slices rank-major ([G][M][ceil(N/G)], what NCCL's
all-gather produces on the GPU), and the same index permutation the GPU
`gather_permute_kernel` applies must rebuild the full [M, N] output exactly.
"""
import os
import socket

import numpy as np
import pytest


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def permute_rank_major(gathered: np.ndarray, G: int, M: int, Ns: int, N: int) -> np.ndarray:
    """[G*M*Ns] rank-major -> [M, N]; column n lives in rank n // Ns at offset n % Ns."""
    src = gathered.reshape(G, M, Ns)
    out = np.empty((M, N), dtype=gathered.dtype)
    n = np.arange(N)
    out[:, :] = src[n // Ns, :, n % Ns].T
    return out


def _worker(rank, world, port, M, N, K, q_path, result_path):
    import torch
    import torch.distributed as dist

    from oracle import Oracle
    import vvllm_b200 as v

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    data = np.load(q_path)
    q, s, b, x = data["q"], data["s"], data["b"], data["x"]
    r0, rows = v.shard_range(N, world, rank)
    per = -(-N // world)
    local = np.zeros((M, per), np.float32)  # padded slot, as on the GPU
    if rows:
        local[:, :rows] = Oracle().linear_q8(x, np.ascontiguousarray(q[r0:r0 + rows]), s[r0:r0 + rows],
                                             b[r0:r0 + rows])
    gathered = [torch.zeros(M * per) for _ in range(world)]
    dist.all_gather(gathered, torch.from_numpy(local.ravel().copy()))
    full = permute_rank_major(torch.cat(gathered).numpy(), world, M, per, N)
    if rank == 0:
        np.save(result_path, full)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,M,N,K", [(2, 1, 4736, 896), (2, 3, 1001, 576), (3, 2, 10, 64), (3, 1, 2, 32)])
def test_sharded_gather_matches_full(tmp_path, oracle, world, M, N, K):
    import torch.multiprocessing as mp

    from tests._util import make_bias, make_weight, make_x

    q, s = oracle.quantize_per_channel(make_weight(N, K, 31 + N))
    b = make_bias(N, 32)
    x = make_x(M, K, 33)
    qp = str(tmp_path / "in.npz")
    np.savez(qp, q=q, s=s, b=b, x=x)
    rp = str(tmp_path / "out.npy")
    mp.start_processes(_worker, args=(world, _free_port(), M, N, K, qp, rp), nprocs=world, join=True,
                       start_method="spawn")
    full = np.load(rp)
    ref = oracle.linear_q8(x, q, s, b)
    assert np.array_equal(full.view(np.uint32), ref.view(np.uint32))  # same arithmetic per element


def _failing_worker(rank, world, port, result_path):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    if rank == 1:
        dist.destroy_process_group()
        os._exit(3)  # a rank that leaves between steps without joining the collective
    t = torch.zeros(4)
    try:
        dist.all_reduce(t)
        outcome = "completed"
    except Exception as e:  # the surviving rank learns of it through the collective's timeout/error
        outcome = "error: " + type(e).__name__
    with open(result_path, "w") as f:
        f.write(outcome)
    os._exit(0)


def test_rank_failure_is_reported_not_hung(tmp_path):
    """Failure detection on the host: a rank exits between steps; the other rank's next
    collective fails within the process-group timeout instead of hanging."""
    import torch.multiprocessing as mp

    rp = str(tmp_path / "outcome.txt")
    ctx = mp.start_processes(_failing_worker, args=(2, _free_port(), rp), nprocs=2, join=False,
                             start_method="spawn")
    for p in ctx.processes:
        p.join(timeout=120)
        assert not p.is_alive()
    with open(rp) as f:
        assert f.read().startswith("error")


def test_shard_range_matches_gather_layout():
    import vvllm_b200 as v

    for N, G in [(152064, 8), (37888, 4), (3584, 2), (10, 4), (7, 3), (1, 2)]:
        per = -(-N // G)
        seen = []
        for r in range(G):
            r0, rows = v.shard_range(N, G, r)
            assert r0 == min(r * per, N)
            seen.extend(range(r0, r0 + rows))
        assert seen == list(range(N))

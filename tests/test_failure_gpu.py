"""Failure paths that must end with an error status, never a hung GPU or process.

* The bounded wait of the gathered calls (a rank's outputs of the previous call must have
  landed) runs out on one GPU: the counts it watches are a device buffer nothing advances, as
  if a peer never finished.  Checked in all three places the wait runs (the standalone wait
  kernel, inside the digit GEMV, inside its prep kernel): the error word reports it, clearing
  it resets the library's state, and the next ordinary call is correct against the oracle.
* A communicator whose second rank never joins: b200q8_comm_init returns B200Q8_ERR_TIMEOUT at
  its deadline (in a child process, so a stuck NCCL could never hold the test session).
* Two GPUs: rank 1 skips a gathered call (a rank that left between steps); rank 0's wait runs
  out, and after both ranks rebuild the communicator a gathered call is correct again.

No test here faults, traps or hangs a GPU: every wait it makes run out is bounded in-kernel.
"""
import os
import socket
import subprocess
import sys
import textwrap

import numpy as np
import pytest

from tests._util import TOL_F16, make_weight, make_x, rowwise_normwise_err

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SHIFT = 20  # each finished gathered call adds 2^20 to a rank's completion count


def _inputs(cuda, oracle, N, K, seed):
    import torch

    q, s = oracle.quantize_per_channel(make_weight(N, K, seed))
    x = make_x(1, K, seed + 1).astype(np.float16)
    return (q, s, x, torch.from_numpy(q).to(cuda), torch.from_numpy(s).to(cuda),
            torch.from_numpy(x).to(cuda))


def _reference(oracle, q, s, x):
    return oracle.linear_q8(x.astype(np.float32), q, s, None)


@pytest.mark.parametrize("n", [2, 8])
def test_standalone_wait_runs_out_and_reports(cuda, n):
    import torch

    import vvllm_b200 as v

    assert v.kernel_error(clear=True) == 0
    # this rank (the last slot) has finished one call; nothing ever advances the others
    counts = torch.zeros(n, dtype=torch.int64, device=cuda)
    counts[n - 1] = 1 << SHIFT
    v.diag_peer_wait(counts, n - 1, timeout_s=0.05, where=0)
    torch.cuda.synchronize()  # returns: the kernel gave up after 50 ms
    assert v.kernel_error(clear=False) & 2
    v.kernel_error(clear=True)
    assert v.kernel_error(clear=False) == 0
    counts.fill_(1 << SHIFT)  # every rank's call 1 has landed: no error
    v.diag_peer_wait(counts, n - 1, timeout_s=0.05, where=0)
    torch.cuda.synchronize()
    assert v.kernel_error() == 0


@pytest.mark.parametrize("where,N,K", [(1, 1000, 896), (2, 1000, 896), (2, 3584, 18944)])
def test_wait_inside_gemv_runs_out_then_recovers(cuda, oracle, where, N, K):
    import torch

    import vvllm_b200 as v

    assert v.kernel_error(clear=True) == 0
    q, s, x, qt, st, xt = _inputs(cuda, oracle, N, K, 1300 + where)
    counts = torch.zeros(2, dtype=torch.int64, device=cuda)
    counts[0] = 3 << SHIFT  # this rank (slot 0) has finished three calls, its peer none
    out = torch.zeros((1, N), dtype=torch.float16, device=cuda)
    v.diag_peer_wait(counts, 0, timeout_s=0.05, where=where, out=out, x=xt, w=qt, scales=st)
    torch.cuda.synchronize()
    code = v.kernel_error(clear=False)
    assert code & 2, code  # the peer wait ran out ...
    if where == 1:
        assert code & 1, code  # ... and the GEMV gave up (its outputs are invalid)
    v.kernel_error(clear=True)  # also resets the split-tile counters a give-up may leave set
    assert v.kernel_error(clear=False) == 0
    # the context is usable and the library's state is clean: an ordinary call is correct
    y = torch.empty((1, N), dtype=torch.float16, device=cuda)
    v.linear_q8_ex(y, xt, qt, st, algo=v.ALGO_TC_I8)
    torch.cuda.synchronize()
    assert v.kernel_error() == 0
    ref = _reference(oracle, q, s, x)
    assert rowwise_normwise_err(y.float().cpu().numpy(), ref) <= TOL_F16
    # the same wait with the counts reached: the GEMV behind it is the ordinary kernel's result
    counts[1] = (3 << SHIFT) + 5  # the peer's three calls have landed (and part of a fourth)
    out.zero_()
    v.diag_peer_wait(counts, 0, timeout_s=0.05, where=where, out=out, x=xt, w=qt, scales=st)
    torch.cuda.synchronize()
    assert v.kernel_error() == 0
    np.testing.assert_array_equal(out.cpu().numpy(), y.cpu().numpy())


_INIT_CHILD = textwrap.dedent("""
    import json, sys, time
    sys.path.insert(0, {root!r})
    import vvllm_b200 as v
    uid = v.Comm.unique_id()
    t0 = time.monotonic()
    try:
        v.Comm(0, 2, 0, uid, timeout_s={deadline})  # rank 1 never joins
        status = 0
    except v.B200Q8Error as e:
        status = e.status
    print(json.dumps({{"status": status, "elapsed": time.monotonic() - t0}}))
""")


def test_comm_init_deadline_when_a_rank_never_joins(cuda):
    import json

    deadline = 3.0
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", CUDA_VISIBLE_DEVICES=os.environ.get("CUDA_VISIBLE_DEVICES", "0"))
    r = subprocess.run([sys.executable, "-c", _INIT_CHILD.format(root=ROOT, deadline=deadline)], env=env,
                       capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr[-2000:]
    res = json.loads(r.stdout.strip().splitlines()[-1])
    assert res["status"] == -5, res  # B200Q8_ERR_TIMEOUT
    assert deadline <= res["elapsed"] < deadline + 30, res


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _missing_rank_worker(rank, world, port, path):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    import vvllm_b200 as v

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    data = np.load(os.path.join(path, "case.npz"))
    N = data["q"].shape[0]
    results = {}
    for attempt in range(2):
        uid = [v.Comm.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        comm = v.Comm(rank, world, rank, uid[0], timeout_s=60.0)
        r0, rows = v.shard_range(N, world, rank)
        qt = torch.from_numpy(np.ascontiguousarray(data["q"][r0:r0 + rows])).to(dev)
        st = torch.from_numpy(data["s"][r0:r0 + rows].copy()).to(dev)
        xt = torch.from_numpy(data["x"]).to(dev)
        sym = comm.sym_alloc(N * 2)
        out = sym.view(torch.float16).view(1, N)
        if attempt == 0:
            # One call on both ranks first: the first gathered call sets up the completion counts,
            # a collective step every rank must take.
            v.linear_q8_sharded_p2p(comm, out, xt, qt, st, None, N)
            torch.cuda.synchronize()
            dist.barrier()
            # Then rank 1 leaves a step: it makes no call, so its part never arrives on rank 0.
            if rank == 0:
                v.linear_q8_sharded_p2p(comm, out, xt, qt, st, None, N)
                torch.cuda.synchronize()  # the wait kernel gives up after its 2 s limit
            results[f"err{attempt}"] = v.kernel_error(clear=True)
        else:
            v.linear_q8_sharded_p2p(comm, out, xt, qt, st, None, N)
            torch.cuda.synchronize()
            results[f"err{attempt}"] = v.kernel_error(clear=True)
            results["out"] = out.float().cpu().numpy()
        dist.barrier()  # every rank is between steps, no kernel of either in flight
        del out
        comm.sym_free(sym)
        del sym
        comm.destroy()
    np.savez(os.path.join(path, f"rank{rank}.npz"), **results)
    dist.barrier()
    dist.destroy_process_group()


def test_gathered_call_with_a_missing_rank(tmp_path, oracle):
    import torch
    import torch.multiprocessing as mp

    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    os.environ["NCCL_NVLS_ENABLE"] = "0"  # no NVLink multicast object a leaving rank could be bound to
    N, K = 2048, 896
    q, s = oracle.quantize_per_channel(make_weight(N, K, 1400))
    x = make_x(1, K, 1401).astype(np.float16)
    np.savez(tmp_path / "case.npz", q=q, s=s, x=x)
    mp.start_processes(_missing_rank_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    r = [np.load(tmp_path / f"rank{i}.npz") for i in range(2)]
    assert r[0]["err0"] & 2, int(r[0]["err0"])  # rank 0's wait for rank 1 ran out
    assert int(r[1]["err0"]) == 0
    ref = oracle.linear_q8(x.astype(np.float32), q, s, None)
    for i in range(2):
        assert int(r[i]["err1"]) == 0
        assert rowwise_normwise_err(r[i]["out"], ref) <= TOL_F16

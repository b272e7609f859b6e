"""Column-sharded linear_q8 over 2, 4 and 8 GPUs (each world size runs where that many GPUs exist).

Each rank owns rows [r*ceil(N/G), ...) of the weight (b200q8_shard_range) and must end with the
full [M, N] output, gathered by NCCL (b200q8_linear_q8_sharded) or by the GEMV's own stores into
every rank's buffer (b200q8_linear_q8_sharded_p2p).  The gathered outputs must equal, bit for
bit, each shard computed on one GPU by the kernel the gathered call runs per shard (up to 4
tokens the local dispatch's choice, b200q8_linear_q8 on the shard's rows; more tokens the int8
digit GEMV), so the same sums in the same order, and the CPU oracle on a row sample within the
fp16 tolerance.
"""
import os
import socket

import numpy as np
import pytest

from tests._util import TOL_F16, make_weight, make_x, rowwise_normwise_err, sample_rows

pytestmark = pytest.mark.gpu

CASES = [
    # M, N, K
    (1, 37888, 3584),   # 7B gate/up: direct in-place all-gather
    (4, 1001, 896),     # ragged shards + rank-major permute
    (1, 3584, 18944),   # 7B down: long K, split tiles on every rank
    (8, 4736, 3584),    # several tokens
]


CHAIN = [
    # N1 (= K2), K1, N2, tokens.  The second call waits for the first one's gathered output inside
    # its GEMV (few tokens, rows up to 4096, or longer rows of small weights) or in its prep kernel
    # (more than 4 tokens, or long rows of large weights).
    (2048, 896, 640, 1),
    (6144, 896, 1000, 1),
    (3072, 896, 640, 5),
]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _sharded_ref(v, torch, dev, q, s, x, N, world, odt):
    """Every shard's rows computed on this GPU by the kernel the gathered call runs for them,
    assembled into [M, N]."""
    M = x.shape[0]
    algo = v.ALGO_AUTO if M <= 4 else v.ALGO_TC_I8
    out = torch.empty((M, N), dtype=odt, device=dev)
    qd, sd = torch.from_numpy(q).to(dev), torch.from_numpy(s).to(dev)
    for r in range(world):
        r0, rows = v.shard_range(N, world, r)
        if rows == 0:
            continue
        part = torch.empty((M, rows), dtype=odt, device=dev)
        v.linear_q8_ex(part, x, qd[r0:r0 + rows], sd[r0:r0 + rows], algo=algo)
        out[:, r0:r0 + rows] = part
    return out


def _worker(rank, world, port, path):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    import vvllm_b200 as v

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    uid = [v.Comm.unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    comm = v.Comm(rank, world, rank, uid[0], timeout_s=60.0)
    results = {}
    for ci, (M, N, K) in enumerate(CASES):
        data = np.load(os.path.join(path, f"case{ci}.npz"))
        q, s, x = data["q"], data["s"], data["x"]
        r0, rows = v.shard_range(N, world, rank)
        qt = torch.from_numpy(np.ascontiguousarray(q[r0:r0 + rows])).to(dev)
        st = torch.from_numpy(s[r0:r0 + rows].copy()).to(dev)
        xt = torch.from_numpy(x).to(dev).half()
        per = -(-N // world)
        out = torch.zeros((M, N), dtype=torch.float16, device=dev)
        gather = None if (M == 1 and N % world == 0) else torch.zeros(world * M * per, dtype=torch.float16,
                                                                          device=dev)
        for _ in range(2):  # twice: the second call must not depend on leftovers of the first
            v.linear_q8_sharded(comm, out, xt, qt, st, None, N, gather=gather)
        torch.cuda.synchronize()
        results[f"out{ci}"] = out.float().cpu().numpy()
        # The gather fused into the GEMV (peer stores + flags), double-buffered in one
        # symmetric allocation; the third call reuses buffer 0 with the same inputs.
        for odt in (torch.float16, torch.float32):
            eb = 2 if odt == torch.float16 else 4
            sym = comm.sym_alloc(2 * M * N * eb)
            bufs = [sym[i * M * N * eb:(i + 1) * M * N * eb].view(odt).view(M, N) for i in range(2)]
            xin = xt if odt == torch.float16 else xt.float()
            for it in range(3):
                v.linear_q8_sharded_p2p(comm, bufs[it % 2], xin, qt, st, None, N)
            torch.cuda.synchronize()
            tag = "h" if odt == torch.float16 else "f"
            results[f"p2p{tag}{ci}_0"] = bufs[0].float().cpu().numpy()
            results[f"p2p{tag}{ci}_1"] = bufs[1].float().cpu().numpy()
            del bufs
            comm.sym_free(sym)
            del sym
        if rank == 0:  # every shard on one GPU, on the kernel the gathered call runs per shard
            full = _sharded_ref(v, torch, dev, q, s, xt, N, world, torch.float16)
            fullf = _sharded_ref(v, torch, dev, q, s, xt.float(), N, world, torch.float32)
            torch.cuda.synchronize()
            results[f"full{ci}"] = full.float().cpu().numpy()
            results[f"fullf{ci}"] = fullf.cpu().numpy()
    # Chained gathered calls with deferred waits: y2 = W2 . gather(W1 . x); the second call reads
    # the first one's gathered output, waiting for it inside its GEMV or in its prep kernel; then
    # Comm.wait().
    for ci, (N1, K1, N2, M) in enumerate(CHAIN):
        data = np.load(os.path.join(path, f"chain{ci}.npz"))
        r1 = v.shard_range(N1, world, rank)
        r2 = v.shard_range(N2, world, rank)
        q1 = torch.from_numpy(np.ascontiguousarray(data["q1"][r1[0]:r1[0] + r1[1]])).to(dev)
        s1 = torch.from_numpy(data["s1"][r1[0]:r1[0] + r1[1]].copy()).to(dev)
        q2 = torch.from_numpy(np.ascontiguousarray(data["q2"][r2[0]:r2[0] + r2[1]])).to(dev)
        s2 = torch.from_numpy(data["s2"][r2[0]:r2[0] + r2[1]].copy()).to(dev)
        x = torch.from_numpy(data["x"]).to(dev).half()
        b1 = -(-M * N1 * 2 // 256) * 256
        sym = comm.sym_alloc(b1 + M * N2 * 2)
        y1 = sym[:M * N1 * 2].view(torch.float16).view(M, N1)
        y2 = sym[b1:b1 + M * N2 * 2].view(torch.float16).view(M, N2)
        for _ in range(3):
            v.linear_q8_sharded_p2p(comm, y1, x, q1, s1, None, N1, defer_wait=True)
            v.linear_q8_sharded_p2p(comm, y2, y1, q2, s2, None, N2, defer_wait=True)
            comm.wait()
        torch.cuda.synchronize()
        results[f"chain{ci}"] = y2.float().cpu().numpy()
        if rank == 0:
            f1 = _sharded_ref(v, torch, dev, data["q1"], data["s1"], x, N1, world, torch.float16)
            f2 = _sharded_ref(v, torch, dev, data["q2"], data["s2"], f1, N2, world, torch.float16)
            torch.cuda.synchronize()
            results[f"chainref{ci}"] = f2.float().cpu().numpy()
        del y1, y2
        comm.sym_free(sym)
        del sym
    assert v.kernel_error() == 0
    np.savez(os.path.join(path, f"rank{rank}.npz"), **results)
    dist.barrier()
    comm.destroy()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded(tmp_path, oracle, world):
    import torch
    import torch.multiprocessing as mp

    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    for ci, (M, N, K) in enumerate(CASES):
        q, s = oracle.quantize_per_channel(make_weight(N, K, 900 + ci))
        x = make_x(M, K, 910 + ci).astype(np.float16).astype(np.float32)
        np.savez(tmp_path / f"case{ci}.npz", q=q, s=s, x=x)
    for ci, (N1, K1, N2, M) in enumerate(CHAIN):
        q1, s1 = oracle.quantize_per_channel(make_weight(N1, K1, 950 + ci))
        q2, s2 = oracle.quantize_per_channel(make_weight(N2, N1, 960 + ci))
        x = make_x(M, K1, 970 + ci).astype(np.float16).astype(np.float32)
        np.savez(tmp_path / f"chain{ci}.npz", q1=q1, s1=s1, q2=q2, s2=s2, x=x)
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    r = [np.load(tmp_path / f"rank{i}.npz") for i in range(world)]
    for ci, (M, N, K) in enumerate(CASES):
        full = r[0][f"full{ci}"]
        for i in range(world):
            got = r[i][f"out{ci}"]
            assert rowwise_normwise_err(got, full) <= TOL_F16, (ci, i)
            # The fused gather runs the local dispatch's kernel per shard: bit-identical.
            for b in (0, 1):
                np.testing.assert_array_equal(r[i][f"p2ph{ci}_{b}"], full, err_msg=f"case {ci} rank {i} buf {b}")
                np.testing.assert_array_equal(r[i][f"p2pf{ci}_{b}"], r[0][f"fullf{ci}"],
                                              err_msg=f"case {ci} rank {i} buf {b} f32")
        data = np.load(tmp_path / f"case{ci}.npz")
        rows = sample_rows(N, 64)
        ref = oracle.linear_q8(data["x"], data["q"][rows], data["s"][rows], None)
        assert rowwise_normwise_err(r[1][f"out{ci}"][:, rows], ref) <= TOL_F16, ci
    for ci in range(len(CHAIN)):
        for i in range(world):  # deferred-wait chain: bit-identical to the shards computed on one GPU
            np.testing.assert_array_equal(r[i][f"chain{ci}"], r[0][f"chainref{ci}"], err_msg=f"chain {ci} rank {i}")

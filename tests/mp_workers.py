"""Bodies of the multi-process tests (run in spawned child processes).

Every worker joins a gloo process group on 127.0.0.1 with a short timeout,
reports through a multiprocessing queue as (rank, ok, detail), and never
raises out of the process.
"""

from __future__ import annotations

import datetime
import os
import sys
import traceback
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent
for p in (str(ROOT), str(ROOT / "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)

SOFTMAX = "0 input 0\n1 softmax 0 1\n"
RELU_LOGISTIC = "0 input 0\n1 relu 0\n2 logistic 1\n"
# H = logistic(X @ W1 + b1); P = softmax(H @ W2 + b2, 1) -- config 5's graph.
MLP = ("0 input 0\n1 input 1\n2 input 2\n3 input 3\n4 input 4\n5 matmul 0 1\n"
       "6 broadcast 2 {m},{h}\n7 add 5 6\n8 logistic 7\n9 matmul 8 3\n"
       "10 broadcast 4 {m},{d}\n11 add 9 10\n12 softmax 11 1\n")


def _gloo(rank: int, world: int, port: int, seconds: int = 60):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=seconds))
    return dist


def _mlp_inputs(rows: int, d: int, h: int, seed: int):
    rng = np.random.default_rng(seed)
    x = rng.normal(0, 1, (rows, d)).astype(np.float32)
    w1 = rng.normal(0, 1 / np.sqrt(d), (d, h)).astype(np.float32)
    b1 = rng.uniform(-0.1, 0.1, h).astype(np.float32)
    w2 = rng.normal(0, 1 / np.sqrt(h), (h, d)).astype(np.float32)
    b2 = rng.uniform(-0.1, 0.1, d).astype(np.float32)
    return [x, w1, b1, w2, b2]


def gloo_row_shard_worker(rank: int, world: int, port: int, q) -> None:
    """Each rank evaluates its row block of three row-local graphs with the
    host oracle; the blocks, gathered over gloo, must equal the whole graph
    bit for bit (the property the GPU row sharding relies on)."""
    try:
        from porch_b200 import api
        import graphs

        dist = _gloo(rank, world, port)
        rng = np.random.default_rng(7)
        cases = []
        x = rng.normal(0, 2, (1001, 257)).astype(np.float32)
        cases.append(("softmax", SOFTMAX, [x], 1001))
        cases.append(("relu_logistic", RELU_LOGISTIC, [x], 1001))
        ins = _mlp_inputs(203, 48, 80, 11)
        cases.append(("mlp", MLP.format(m="{m}", h=80, d=48), ins, 203))
        details = []
        for name, program, inputs, rows in cases:
            b, e = api.row_block(rows, rank, world)
            local = [np.ascontiguousarray(inputs[0][b:e])] + inputs[1:]
            text = program.replace("{m}", str(e - b))
            block = graphs.evaluate_oracle(text, local, threads=1)
            blocks = [None] * world
            dist.all_gather_object(blocks, block)
            if rank == 0:
                whole = graphs.evaluate_oracle(program.replace("{m}", str(rows)), inputs, threads=1)
                got = np.concatenate(blocks, axis=0)
                same = got.shape == whole.shape and np.array_equal(
                    got.view(np.uint32), whole.view(np.uint32))
                details.append((name, bool(same), [blk.shape[0] for blk in blocks]))
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, all(d[1] for d in details) if rank == 0 else True, details))
    except Exception:
        q.put((rank, False, traceback.format_exc()))


def gloo_bench_helpers_worker(rank: int, world: int, port: int, q) -> None:
    """bench.py's multi-rank plumbing on gloo: process group from the
    torchrun environment, max over ranks, per-rank row blocks of the inputs."""
    try:
        os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank),
                          MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        import bench
        from porch_b200 import api

        r, w, local, dist = bench.dist_setup(world)
        assert (r, w, local) == (rank, world, rank)
        slowest = bench.max_over_ranks(dist, 1.0 + rank)
        # A small stand-in for config 3's input, partitioned as the bench does.
        bench.CONFIGS["c3a_softmax"] = ([([1001, 64], "normal", 0, 2)], 2 * 1001 * 64 * 4, "hbm")
        arrays = bench.make_host_inputs(api, "c3a_softmax", rank, world)
        full = np.empty(1001 * 64, dtype=np.float32)
        api.fill_synthetic(full, bench.SEED, "normal", 0, 2)
        full = full.reshape(1001, 64)
        b, e = api.row_block(1001, rank, world)
        ok_rows = np.array_equal(arrays[0], full[b:e])
        sizes = [None] * world
        dist.all_gather_object(sizes, arrays[0].shape[0])
        bench.barrier(dist)
        dist.destroy_process_group()
        ok = slowest == float(world) and ok_rows and sum(sizes) == 1001
        q.put((rank, ok, {"max": slowest, "rows": sizes}))
    except Exception:
        q.put((rank, False, traceback.format_exc()))


def gpu_allgather_worker(rank: int, world: int, port: int, q) -> None:
    """Row-sharded realisation on one GPU per rank, gathered by NCCL, equals
    the whole graph realised on one GPU (bit for bit: every row runs the same
    arithmetic whatever the row count); uneven blocks use Send/Recv."""
    try:
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        from porch_b200 import api

        dist = _gloo(rank, world, port)
        uid = [api.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        comm = api.Communicator(world, uid[0], rank, rank, timeout_s=60.0)
        details = []
        rng = np.random.default_rng(5)
        cases = [("softmax_uneven", rng.normal(0, 2, (1001, 257)).astype(np.float32), None),
                 ("relu_logistic_equal", rng.normal(0, 2, (1024, 4096)).astype(np.float32), None),
                 ("mlp_equal", None, _mlp_inputs(512, 2048, 256, 9))]
        for name, x, mlp in cases:
            if mlp is None:
                rows = x.shape[0]
                b, e = api.row_block(rows, rank, world)
                xs = api.tensor(list(x[b:e].shape), np.ascontiguousarray(x[b:e]), device=rank)
                expr = api.softmax(xs, 1) if name.startswith("softmax") else api.logistic(api.relu(xs))
                whole_expr = None
                if rank == 0:
                    xw = api.tensor(list(x.shape), x, device=0)
                    whole_expr = (api.softmax(xw, 1) if name.startswith("softmax")
                                  else api.logistic(api.relu(xw)))
            else:
                rows = mlp[0].shape[0]
                b, e = api.row_block(rows, rank, world)

                def graph(x_rows, dev):
                    t = {"x": api.tensor(list(x_rows.shape), x_rows, device=dev)}
                    for k, arr in zip(("w1", "b1", "w2", "b2"), mlp[1:]):
                        t[k] = api.tensor(list(arr.shape), arr, device=dev)
                    return api.config_graph("c5_mlp", t)

                expr = graph(np.ascontiguousarray(mlp[0][b:e]), rank)
                whole_expr = graph(mlp[0], 0) if rank == 0 else None
            shard = api.materialize(expr)
            gathered = comm.allgather_rows(shard, rows)
            got = gathered.cpu().reshape(gathered.shape())
            # The asynchronous gather, read back at once: the host read is
            # ordered after it by events alone; then the bounded wait.
            late = comm.allgather_rows(shard, rows, wait=False)
            got_async = late.cpu().reshape(late.shape())
            comm.wait()
            same_async = np.array_equal(got.view(np.uint32), got_async.view(np.uint32))
            if rank == 0:
                want = api.materialize(whole_expr).cpu().reshape(rows, -1)
                same = np.array_equal(got.view(np.uint32), want.view(np.uint32))
                details.append((name, bool(same and same_async)))
            else:
                details.append((name, got.shape[0] == rows and same_async))
        comm.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, all(d[1] for d in details), details))
    except Exception:
        q.put((rank, False, traceback.format_exc()))


def gpu_missing_peer_worker(rank: int, world: int, port: int, q) -> None:
    """Rank 1 leaves between steps (it never joins the gather, and has no
    collective in flight); rank 0's gather must end with an error after its
    communicator's short timeout instead of hanging, and the process must
    stay usable (a later materialize on the same GPU succeeds)."""
    try:
        import time

        os.environ["NCCL_NVLS_ENABLE"] = "0"
        from porch_b200 import api

        dist = _gloo(rank, world, port, seconds=120)
        uid = [api.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        comm = api.Communicator(world, uid[0], rank, rank, timeout_s=60.0)
        dist.barrier()
        if rank == 0:
            comm.set_timeout(2.0)
            x = api.tensor([4, 8], np.ones(32, dtype=np.float32), device=0)
            t0 = time.monotonic()
            err = None
            try:
                comm.allgather_rows(api.materialize(api.relu(x)), 8)
            except RuntimeError as exc:
                err = str(exc)
            waited = time.monotonic() - t0
            y = api.materialize(api.relu(x) + 1.0).cpu()
            ok = err is not None and waited < 30.0 and float(np.asarray(y).reshape(-1)[0]) == 2.0
            detail = {"error": err, "waited_s": round(waited, 2)}
        else:
            ok, detail = True, "left without joining the gather"
        dist.barrier()  # rank 1 leaves only after rank 0 has seen the error
        comm.abort()
        comm.close()
        dist.destroy_process_group()
        q.put((rank, ok, detail))
    except Exception:
        q.put((rank, False, traceback.format_exc()))

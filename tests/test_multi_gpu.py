"""Row sharding across GPUs (one process per GPU) and its host plumbing.

CPU: the block partition, argument checks, and world_size-2 gloo runs of
(a) the row-shard decomposition of configs 3 and 5 against the whole graph
on the host oracle and (b) bench.py's multi-rank helpers.
GPU (two devices; skipped with a reason on a one-GPU box): the NCCL row
gather against the whole graph realised on one GPU, and a peer that never
joins a gather ending in a bounded error.
"""

import multiprocessing as mp
import socket

import pytest

import mp_workers


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(target, world: int, timeout: float = 240.0):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, ok, detail = q.get(timeout=timeout)
            results[rank] = (ok, detail)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
                p.join(timeout=10)
        for rank in sorted(results):
            print(f"rank {rank}: ok={results[rank][0]}\n{results[rank][1]}")
        print("exit codes:", [p.exitcode for p in procs])
    return results


@pytest.mark.parametrize("rows,n", [(0, 1), (1, 4), (7, 2), (65536, 8), (1001, 3), (16384, 8)])
def test_row_block_partition_covers_rows_contiguously(api, rows, n):
    blocks = [api.row_block(rows, r, n) for r in range(n)]
    assert blocks[0][0] == 0 and blocks[-1][1] == rows
    for (b0, e0), (b1, _) in zip(blocks, blocks[1:]):
        assert e0 == b1
    sizes = [e - b for b, e in blocks]
    assert max(sizes) - min(sizes) <= 1
    assert sizes == sorted(sizes, reverse=True)


def test_row_block_rejects_bad_ranks(api):
    for rows, rank, n in [(10, 2, 2), (10, -1, 2), (10, 0, 0), (-1, 0, 1)]:
        with pytest.raises(ValueError):
            api.row_block(rows, rank, n)


def test_communicator_rejects_bad_arguments_before_any_device_work(api):
    with pytest.raises(ValueError):
        api.Communicator(2, b"\0" * 127, 0, 0)
    for nranks, rank, timeout in [(0, 0, 1.0), (2, 2, 1.0), (2, -1, 1.0), (2, 0, 0.0)]:
        with pytest.raises(ValueError):
            api.Communicator(nranks, b"\0" * 128, rank, 0, timeout_s=timeout)


def test_gloo_two_ranks_row_blocks_equal_whole_graph(api, oracle_lib):
    results = _run(mp_workers.gloo_row_shard_worker, 2)
    assert all(ok for ok, _ in results.values()), results
    names = [d[0] for d in results[0][1]]
    assert names == ["softmax", "relu_logistic", "mlp"]
    assert results[0][1][0][2] == [501, 500]


def test_gloo_two_ranks_bench_helpers(api):
    results = _run(mp_workers.gloo_bench_helpers_worker, 2)
    assert all(ok for ok, _ in results.values()), results
    assert results[0][1]["rows"] == [501, 500]


def _need_two_gpus(api):
    n = api.device_count()
    if n < 2:
        pytest.skip(f"needs 2 GPUs, this box shows {n}")


@pytest.mark.gpu
def test_nccl_row_gather_equals_whole_graph_on_one_gpu(gpu):
    _need_two_gpus(gpu)
    results = _run(mp_workers.gpu_allgather_worker, 2, timeout=600)
    assert all(ok for ok, _ in results.values()), results


@pytest.mark.gpu
def test_missing_peer_ends_gather_with_bounded_error(gpu):
    _need_two_gpus(gpu)
    results = _run(mp_workers.gpu_missing_peer_worker, 2, timeout=300)
    assert all(ok for ok, _ in results.values()), results
    assert results[0][1]["error"]

"""Benchmark: porch lazy-graph hot path on B200.

Headline workload: config 5 of the baseline, the two-layer MLP realised as
one lazy graph P = softmax(logistic(X@W1 + b1)@W2 + b2, 1) with
X [16384,4096], W1 [4096,16384], W2 [16384,4096] in fp32 (tcgen05 3xTF32
GEMMs with fused epilogues), metric "fp32 matmul TFLOP/s". The same run
times every other configuration of the baseline and reports each under
"extra" with its own value, roofline, e2e and cpu_baseline: config 1
((a+b)*2-1), config 2 (slice/transpose/bias/concat), configs 3a/3b (softmax,
logistic(relu)) and config 4 (relu(A@B + bias)); --no-extra skips them and
--workload picks another headline.

Multi-GPU (python -m torch.distributed.run ... bench.py --gpus N): config 5
splits X's rows across ranks in contiguous blocks (W1, W2 replicated, strong
scaling); each rank realises its block on its own GPU and P is gathered
whole on every rank with one ncclAllGather over NVLink per step (porch_b200
Communicator.allgather_rows), inside the timed region. Configs 3a/3b are
reported row-sharded too (no exchange: no consumer needs them whole); the
single-GPU configs 1, 2 and 4 are reported at N=1 only. torch.distributed
(gloo) carries only barriers and the max-over-ranks timing.

--impl reference runs the reference's own implementation of the path
(oracle/_ref/ref_runner: AkhilSamavedam/porch compiled from its sources,
NVRTC JIT on the same GPU) on rank 0 and prints the same metric for the same
workloads. It has no multi-GPU path: its one-GPU number is the baseline at
every N.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

SEED = 20261201
CONFIGS = {
    # name: (inputs [(shape, dist, a, b)], algorithmic bytes or flops, bound)
    "c1_elementwise": ([([1 << 24], "uniform", -1, 1), ([1 << 24], "uniform", -1, 1)],
                       12 * (1 << 24), "hbm"),
    "c2_view": ([([8192, 8192], "normal", 0, 1), ([4096], "uniform", -0.5, 0.5),
                 ([6144, 4096], "normal", 0, 1)],
                4096 * 6144 * 4 + 6144 * 4096 * 4 + 4096 * 4 + 12288 * 4096 * 4, "hbm"),
    "c3a_softmax": ([([65536, 4096], "normal", 0, 2)], 2 * 65536 * 4096 * 4, "hbm"),
    "c3b_relu_logistic": ([([65536, 4096], "normal", 0, 2)], 2 * 65536 * 4096 * 4, "hbm"),
    "c4_matmul": ([([8192, 8192], "uniform", -1 / 90.50966799187808, 1 / 90.50966799187808),
                   ([8192, 8192], "uniform", -1 / 90.50966799187808, 1 / 90.50966799187808),
                   ([8192], "uniform", -0.1, 0.1)], 2 * 8192 ** 3, "tensor"),
    "c5_mlp": ([([16384, 4096], "normal", 0, 1), ([4096, 16384], "normal", 0, 1 / 64),
                ([16384], "uniform", -0.1, 0.1), ([16384, 4096], "normal", 0, 1 / 128),
                ([4096], "uniform", -0.1, 0.1)], 4 * 16384 * 4096 * 16384, "tensor"),
}
ROW_SHARDED = {"c3a_softmax", "c3b_relu_logistic", "c5_mlp"}
# Row-sharded workloads whose output a consumer needs whole (gathered by NCCL).
GATHERED = {"c5_mlp"}
KEYS = {
    "c1_elementwise": ["a", "b"], "c2_view": ["x", "bias", "y"], "c3a_softmax": ["x"],
    "c3b_relu_logistic": ["x"], "c4_matmul": ["a", "b", "bias"],
    "c5_mlp": ["x", "w1", "b1", "w2", "b2"],
}
# Activations of the GEMM configurations: in a serving loop a data loader
# writes each new batch through the tensor's device pointer, so the bench
# hands their pointers out (tensor::device_data()) and their 3xTF32 split
# runs every step; the weights (c4's B, c5's W1 and W2) are realised once and
# keep their split from the first step on.
ACTIVATIONS = {"c4_matmul": ["a"], "c5_mlp": ["x"]}
# Kernel family whose launches the roofline line describes.
DOMINANT = {"c1_elementwise": "pb_elem", "c2_view": "pb_elem", "c3a_softmax": "pb_softmax",
            "c3b_relu_logistic": "pb_elem", "c4_matmul": "pb_gemm_tc", "c5_mlp": "pb_gemm_tc"}


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self._t.join(timeout=2)
        return False

    def mark(self) -> int:
        return len(self.lines)

    def hold_load(self, work, count: int, since: int | None = None, limit_s: float = 5.0) -> None:
        """Runs `work` (the benchmark's own steps) until `count` samples have
        arrived after `since`, so that a timed region shorter than the
        sampling period is bracketed by samples taken under the same load."""
        if self.proc is None:
            return
        base = self.mark() if since is None else since
        t0 = time.perf_counter()
        while self.mark() < base + count and time.perf_counter() - t0 < limit_s:
            work()

    def summary(self, lo: int = 0, hi: int | None = None) -> dict | None:
        rows = []
        for ln in self.lines[lo:hi]:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        if not rows:
            return None
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for _, _, flags in rows:
            for n, f in zip(names, flags):
                if f.lower().startswith("active"):
                    reasons.add(n)
        loaded = [r[0] for r in rows]
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": sorted(reasons), "samples": len(rows),
                "window": "samples from the last one before to the first one after the timed "
                          "region, the same steps running throughout"}


def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=180))
        return rank, world, local, dist
    return 0, 1, 0, None


def max_over_ranks(dist, value: float) -> float:
    if dist is None:
        return value
    import torch

    t = torch.tensor([value], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(dist):
    if dist is not None:
        dist.barrier()


def make_host_inputs(api, workload: str, rank: int, world: int):
    specs, _, _ = CONFIGS[workload]
    arrays = []
    for i, (shape, dist_name, a, b) in enumerate(specs):
        shape = list(shape)
        arr = np.empty(int(np.prod(shape)), dtype=np.float32)
        api.fill_synthetic(arr, SEED + i, dist_name, a, b)
        arr = arr.reshape(shape)
        if workload in ROW_SHARDED and world > 1 and i == 0:
            begin, end = api.row_block(shape[0], rank, world)
            arr = np.ascontiguousarray(arr[begin:end])
        arrays.append(arr)
    return arrays


def cpu_baseline(workload: str, arrays, seconds: float = 10.0) -> dict:
    """The host oracle on a bounded sample of the same workload."""
    from oracle.graph import Program

    threads = os.cpu_count() or 1
    P = Program(threads=threads)
    if workload == "c2_view":
        # A row band of the output: rows [0, R) of the transposed slice and
        # rows [0, R) of Y -> 2R output rows; bytes scale accordingly. At
        # R = 6144 the band is the whole output.
        R = 6144
        x, bias, y = arrays
        xs = np.ascontiguousarray(x[:, 1024:1024 + R])
        X = P.tensor(list(xs.shape), xs)
        B = P.tensor([4096], bias)
        Y = P.tensor([R, 4096], np.ascontiguousarray(y[:R]))
        node = P.concat(P.transpose(X[0::2, 0:R]) + P.broadcast_to(B, [R, 4096]), Y, 0)
        nbytes = (R * 4096 * 4) * 2 + 4096 * 4 + (2 * R * 4096 * 4)
        sample = f"output rows 0..{R} and {6144}..{6144 + R} (2*{R} of 12288 rows)"
    elif workload == "c1_elementwise":
        n = 1 << 22
        a, b = (P.tensor([n], arr[:n]) for arr in arrays)
        node = (a + b) * 2.0 - 1.0
        nbytes = 12 * n
        sample = f"first {n} of {1 << 24} elements"
    elif workload in ("c3a_softmax", "c3b_relu_logistic"):
        rows = 2048
        xs = np.ascontiguousarray(arrays[0][:rows])
        X = P.tensor(list(xs.shape), xs)
        node = P.softmax(X, 1) if workload == "c3a_softmax" else P.logistic(P.relu(X))
        nbytes = 2 * xs.size * 4
        sample = f"{rows} of {arrays[0].shape[0]} rows"
    else:
        rows = 16
        a = np.ascontiguousarray(arrays[0][:rows])
        A = P.tensor(list(a.shape), a)
        if workload == "c4_matmul":
            Bm = P.tensor(list(arrays[1].shape), arrays[1])
            Bi = P.tensor([arrays[2].shape[0]], arrays[2])
            node = P.relu(P.matmul(A, Bm) + P.broadcast_to(Bi, [rows, arrays[1].shape[1]]))
            nbytes = 2 * rows * arrays[0].shape[1] * arrays[1].shape[1]
        else:
            W1 = P.tensor(list(arrays[1].shape), arrays[1])
            B1 = P.tensor([arrays[2].shape[0]], arrays[2])
            W2 = P.tensor(list(arrays[3].shape), arrays[3])
            B2 = P.tensor([arrays[4].shape[0]], arrays[4])
            h = P.logistic(P.matmul(A, W1) + P.broadcast_to(B1, [rows, arrays[1].shape[1]]))
            node = P.softmax(P.matmul(h, W2) + P.broadcast_to(B2, [rows, arrays[3].shape[1]]), 1)
            nbytes = 4 * rows * arrays[1].shape[0] * arrays[1].shape[1]
        sample = f"{rows} output rows"
    # The sample is evaluated again and again (the oracle keeps no results
    # between evaluations) until about `seconds` of host work are timed.
    reps = 0
    t0 = time.perf_counter()
    while True:
        P.evaluate(node)
        reps += 1
        dt = time.perf_counter() - t0
        if dt >= seconds or dt / reps * (reps + 1) > 3 * seconds:
            break
    unit = "GFLOP/s" if CONFIGS[workload][2] == "tensor" else "GB/s"
    value = nbytes * reps / dt / 1e9
    return {"value": round(value, 3), "unit": unit, "cores": threads, "kind": "port",
            "sample": f"{sample}, evaluated {reps} times", "seconds": round(dt, 3)}


def shape_of(workload: str, key: str) -> list:
    return CONFIGS[workload][0][KEYS[workload].index(key)][0]


def _config_keys(workload: str, world: int) -> dict:
    specs = CONFIGS[workload][0]
    return {"workload": workload,
            "shapes": {k: s for k, (s, *_) in zip(KEYS[workload], specs)},
            "parallelism": (f"row-shard x{world}" if workload in ROW_SHARDED and world > 1
                            else (f"replicas x{world}" if world > 1 else "single GPU")),
            # Both arms: each step's inputs together exceed the 126 MB L2
            # (this arm also rotates two input sets, `setup`).
            "l2": "inputs larger than L2"}


def measure(api, workload: str, args, rank, world, local, dist, cpu_seconds: float | None,
            two_threads: bool) -> dict:
    """Times `args.steps` steps of `workload` after `args.warmup` warm-up
    steps on this rank's GPU (max over ranks), then the same steps with
    events around every launch (roofline), then end to end through the
    C-ABI from pinned host memory; returns the record."""
    specs, work, bound = CONFIGS[workload]
    keys = KEYS[workload]
    device = local
    arrays = make_host_inputs(api, workload, rank, world)
    work_rank = work
    if workload in ROW_SHARDED and world > 1:
        work_rank = work // world
    # Device-resident input sets, rotated so each step reads memory the
    # previous step did not (every set is larger than the 126 MB L2).
    n_sets = 2
    sets = []
    for s in range(n_sets):
        sets.append({k: api.tensor(list(a.shape), a, device=device) for k, a in zip(keys, arrays)})
    for t in sets:
        for k in ACTIVATIONS.get(workload, []):
            t[k].device_data()
    graphs = [api.config_graph(workload, t) for t in sets]
    # The tensor-core GEMM form the plan chose (the plan's own description).
    plan_text = api.describe(graphs[0])
    gemm_form = None
    if "pb_gemm_tc_" in plan_text:
        gemm_form = ("CTA pairs: tcgen05.mma.cta_group::2, 256x256 tiles on 2-CTA clusters, 32-wide k-blocks"
                     if "CTA pairs" in plan_text else "one CTA per 128x256 tile, 16-wide k-blocks")

    # Config 5 gathers its output P whole on every rank (one ncclAllGather
    # over NVLink per step); configs 3a/3b keep their row blocks where they
    # are, since no consumer of the benchmark needs them whole.
    comm = None
    total_rows = CONFIGS[workload][0][0][0][0]
    if workload in GATHERED and world > 1:
        # NVLink multicast (NVLS) is left off unless the caller asks for it:
        # the gather is a plain all-gather, and a rank that dies while bound
        # to a multicast object can fault the other ranks' GPUs.
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        uid = [api.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        comm = api.Communicator(world, uid[0], rank, device, timeout_s=120.0)

    def step(i, gather=True):
        out = api.materialize(graphs[i % n_sets])
        if comm is not None and gather:
            # On the communicator's stream: step i's gather overlaps step
            # i+1's GEMMs; comm.wait() closes every timed region.
            out = comm.allgather_rows(out, total_rows, wait=False)
        return out

    def run_steps(n, outs, gather=True):
        # At most three results alive at once, in warm-up and timing alike,
        # so the timed steps see the allocator state warm-up left behind.
        for i in range(n):
            outs.append(step(i, gather))
            if len(outs) > 2:
                outs.pop(0)

    # Warm-up (first call lowers + compiles; later calls hit the plan cache).
    outs = []
    run_steps(max(3, args.warmup), outs)
    if comm is not None:
        comm.wait()
    api.device_synchronize(device)

    def load():
        # Runs a rank-dependent number of times: no collective inside.
        run_steps(4, outs, gather=False)
        api.device_synchronize(device)

    with ClockSampler(device) as clocks:
        clocks.hold_load(load, 2)
        api.host_profile_enable(True)
        api.host_profile_read()  # clear
        barrier(dist)
        api.device_synchronize(device)
        launches0 = api.launch_count()
        lo = clocks.mark()
        # The timed region: K steps with nothing of the profiler between the
        # kernels (events around every launch would sit in the gaps).
        with api.DeviceTimer(device) as timer:
            run_steps(args.steps, outs)
            if comm is not None:
                comm.wait()  # the last gather is inside the timed region
        api.device_synchronize(device)
        launches = api.launch_count() - launches0
        host = api.host_profile_read()
        api.host_profile_enable(False)
        # The same K steps again with CUDA events around every launch on the
        # launching stream: per-kernel durations for the roofline.
        api.profile_enable(True)
        api.profile_read()  # clear
        barrier(dist)
        run_steps(args.steps, outs)
        if comm is not None:
            comm.wait()
        api.device_synchronize(device)
        prof = api.profile_read()
        api.profile_enable(False)
        clocks.hold_load(load, 1, since=clocks.mark())
        clock_summary = clocks.summary(max(0, lo - 1), clocks.mark())
    barrier(dist)
    ms_rank = timer.ms / args.steps
    ms = max_over_ranks(dist, ms_rank)
    total_work = work_rank * world
    unit = "GB/s" if bound == "hbm" else "TFLOP/s"
    scale = 1e9 if bound == "hbm" else 1e12
    value = total_work / (ms * 1e-3) / scale

    # Roofline of the dominant kernel family from live per-launch events.
    fam = DOMINANT[workload]
    k_launches = sum(n for name, (n, _) in prof.items() if name.startswith(fam))
    k_ms = sum(t for name, (_, t) in prof.items() if name.startswith(fam))
    pk = peaks()
    roofline = None
    if k_launches:
        per_launch_ms = k_ms / k_launches
        per_launch_work = work_rank / max(1, k_launches // args.steps)
        achieved = per_launch_work / (per_launch_ms * 1e-3) / scale
        if bound == "hbm":
            peak, basis = pk["hbm_gbs"], f"hbm_gbs ({pk['source']}): STREAM-style copy"
        else:
            # fp32 work on the 3xTF32 path: TF32 MMAs run at half the bf16
            # rate and each fp32 product costs three of them (hi*hi, hi*lo,
            # lo*hi), so the tensor-pipe ceiling in useful fp32 flop/s is
            # the measured bf16 figure / 6.
            peak = round(pk["bf16_tflops"] / 6.0, 2)
            basis = f"bf16_tflops ({pk['source']}) / 6: TF32 = bf16 / 2, three TF32 MMAs per fp32 product"
        traffic = None
        tfile = ROOT / "profiles" / "ncu_traffic.json"
        if tfile.exists():
            traffic = json.loads(tfile.read_text()).get(workload)
        roofline = {"bound": bound, "achieved": round(achieved, 2), "peak": peak,
                    "unit": unit, "frac": round(achieved / peak, 4), "traffic": traffic,
                    "peak_source": pk["source"], "peak_basis": basis, "kernel": fam,
                    "how": "CUDA events around every launch over a second pass of the same K steps "
                           "(the timed region itself runs without them)",
                    "kernel_ms": round(per_launch_ms, 5)}
        if launches == args.steps and k_launches == args.steps:
            # One launch per step: the timed region is that kernel back to
            # back on its stream, so its average launch duration there is
            # the step time (each launch overlapping the previous one's tail
            # through programmatic launch); `frac` keeps the isolated figure.
            in_stream = work_rank / (ms_rank * 1e-3) / scale
            roofline["kernel_ms_in_stream"] = round(ms_rank, 5)
            roofline["frac_in_stream"] = round(in_stream / peak, 4)
        if bound == "tensor" and pk.get("bf16_tflops_sustained"):
            # Context: the same ceiling from the power-capped figure (bf16
            # GEMMs back to back for seconds); `frac` keeps the burst one.
            sustained = round(pk["bf16_tflops_sustained"] / 6.0, 2)
            roofline["peak_sustained"] = sustained
            roofline["frac_sustained"] = round(achieved / sustained, 4)

    # End to end through the C-ABI with host buffers in pinned memory.
    pinned = [api.PinnedBuffer(a.size) for a in arrays]
    for pb, a in zip(pinned, arrays):
        pb.array[:] = a.reshape(-1)
    out_count = int(np.prod(step(0).shape()))
    if comm is not None:
        comm.wait()
    out_buf = api.PinnedBuffer(out_count)
    h2d = sum(a.size * 4 for a in arrays)
    d2h = out_count * 4

    def e2e_step(out=out_buf):
        # Uploads enqueued in graph order on the upload stream; each launch
        # waits only for the inputs it reads, so later inputs' copies
        # overlap earlier kernels (config 5: W2 uploads under GEMM1).
        ts = {k: api.tensor_from_pointer(list(a.shape), pb.address, a.size, device=device, asynchronous=True)
              for k, a, pb in zip(keys, arrays, pinned)}
        t = api.materialize(api.config_graph(workload, ts))
        if comm is not None:
            t = comm.allgather_rows(t, total_rows)
        t.cpu(out.array)

    bw = api.copy_bandwidth(device)
    e2e_steps = max(1, min(args.steps, 10))
    for _ in range(2):
        e2e_step()
    barrier(dist)
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    api.device_synchronize(device)
    e2e_ms_rank = (time.perf_counter() - t0) * 1e3 / e2e_steps
    e2e_ms = max_over_ranks(dist, e2e_ms_rank)
    e2e_value = total_work / (e2e_ms * 1e-3) / scale

    # The same steps from two host threads (each has its own stream, so one
    # step's host->device copies overlap the other's device->host read).
    # Skipped when a step holds a collective: threads would interleave the
    # ranks' collectives in different orders.
    e2e_threads = None
    if comm is None and two_threads:
        n_threads = 2
        per_thread = max(1, e2e_steps // n_threads)
        t_bufs = [api.PinnedBuffer(out_count) for _ in range(n_threads)]
        errors = []

        start = threading.Barrier(n_threads + 1)
        done = threading.Barrier(n_threads + 1)

        def worker(j):
            # Streams and allocator caches are per thread: warm this thread's
            # own before the timed steps.
            try:
                for _ in range(2):
                    e2e_step(t_bufs[j])
            except Exception as exc:  # reported, not raised, from a thread
                errors.append(repr(exc))
            start.wait()
            try:
                for _ in range(per_thread):
                    e2e_step(t_bufs[j])
            except Exception as exc:
                errors.append(repr(exc))
            done.wait()

        threads = [threading.Thread(target=worker, args=(j,)) for j in range(n_threads)]
        for th in threads:
            th.start()
        barrier(dist)
        start.wait()
        t0 = time.perf_counter()
        done.wait()
        thr_ms = max_over_ranks(dist, (time.perf_counter() - t0) * 1e3 / (per_thread * n_threads))
        for th in threads:
            th.join()
        e2e_threads = {"threads": n_threads, "value": round(total_work / (thr_ms * 1e-3) / scale, 3),
                       "unit": unit, "ms_per_step": round(thr_ms, 4), "errors": errors or None}

    cpu = None
    if rank == 0 and world == 1 and cpu_seconds:
        try:
            cpu = cpu_baseline(workload, arrays, cpu_seconds)
        except Exception as exc:  # the baseline must not sink the bench line
            cpu = {"error": str(exc)}

    if comm is not None:
        outs.clear()
        comm.close()
    outs.clear()
    del graphs, sets
    config = _config_keys(workload, world)
    return {
        "metric": CONFIG_METRIC[workload], "value": round(value, 3), "unit": unit,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 5), "higher_is_better": True,
        "scaling": "strong" if workload in ROW_SHARDED else "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (seeded; distributions as the baseline config)",
        "config": config,
        "setup": {"l2": f"inputs rotated over {n_sets} device-resident sets, each larger than L2",
                  "gemm": gemm_form,
                  "weights": (f"{', '.join(k for k in KEYS[workload] if k not in ACTIVATIONS[workload] and k[0] in 'wb' and len(shape_of(workload, k)) == 2)} "
                              "realised once and keep their 3xTF32 split; the activations' device pointers are handed "
                              "out (as a data loader writing each batch would), so their split runs every step"
                              if workload in ACTIVATIONS else None),
                  "collective": (f"ncclAllGather of the output rows ({total_rows} rows whole on every "
                                 "rank) inside every step, on its own stream (overlapping the next "
                                 "step's GEMMs), all complete before the timed region ends"
                                 if comm is not None else None)},
        "e2e": {"value": round(e2e_value, 3), "unit": unit, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 4),
                "copy_bound": {"h2d_gbs": round(bw["h2d_gbs"], 2), "d2h_gbs": round(bw["d2h_gbs"], 2),
                               "ms": round((h2d / bw["h2d_gbs"] + d2h / bw["d2h_gbs"]) / 1e6, 4),
                               "frac": round((h2d / bw["h2d_gbs"] + d2h / bw["d2h_gbs"]) / 1e6 / e2e_ms, 4),
                               "how": "pinned 256 MiB H2D and D2H copies timed alone (best of 3)"},
                "two_threads": e2e_threads,
                "path": "pb_tensor_create_async from pinned host -> pb_materialize -> pb_tensor_read"
                        + (" (after pb_allgather_rows)" if comm is not None else "")},
        "gpu_launches": launches,
        "roofline": roofline,
        "cpu_baseline": cpu,
        "clocks": clock_summary,
        "kernels": {k: {"launches": n, "ms": round(t, 4)} for k, (n, t) in prof.items()},
        "host_us_per_materialize": {k: round(v, 2) for k, v in host.items()},
    }


# Reported beside the headline in the same run: single-GPU configurations at
# N = 1 only, the row-sharded ones at every N.
EXTRA_SINGLE = ["c1_elementwise", "c2_view", "c4_matmul"]
EXTRA_SHARDED = ["c3a_softmax", "c3b_relu_logistic"]


def run_ours(args, rank, world, local, dist):
    from porch_b200 import api

    line = measure(api, args.workload, args, rank, world, local, dist,
                   None if args.no_cpu_baseline else 10.0, two_threads=True)
    extra = {}
    if not args.no_extra:
        names = (EXTRA_SINGLE if world == 1 else []) + EXTRA_SHARDED
        for name in sorted(n for n in names if n != args.workload):
            api.empty_cache(local)
            r = measure(api, name, args, rank, world, local, dist,
                        None if args.no_cpu_baseline else 5.0, two_threads=False)
            extra[name] = {k: r[k] for k in ("metric", "value", "unit", "ms_per_step", "scaling", "config",
                                              "setup", "e2e", "gpu_launches", "roofline", "cpu_baseline",
                                              "clocks", "kernels")}
        api.empty_cache(local)
    if rank == 0:
        if extra:
            line["extra"] = extra
        print(json.dumps(line), flush=True)


CONFIG_METRIC = {
    "c1_elementwise": "fused-graph HBM GB/s (config 1: (a+b)*2-1, [2^24])",
    "c2_view": "fused-graph HBM GB/s (config 2: slice/transpose/bias/concat -> [12288,4096])",
    "c3a_softmax": "fused-graph HBM GB/s (config 3: softmax [65536,4096])",
    "c3b_relu_logistic": "fused-graph HBM GB/s (config 3: logistic(relu) [65536,4096])",
    "c4_matmul": "fp32 matmul TFLOP/s (config 4: relu(A@B+bias), 8192^3)",
    "c5_mlp": "fp32 matmul TFLOP/s (config 5: MLP 16384x4096x16384)",
}


def reference_record(workload: str, args, world: int) -> dict:
    """The reference's own implementation of `workload` (its NVRTC-JIT GPU
    path, one GPU) through oracle/_ref/ref_runner, with the same steps and
    warm-up as this library's arm."""
    specs, work, bound = CONFIGS[workload]
    exe = ROOT / "oracle" / "_ref" / "ref_runner"
    unit = "GB/s" if bound == "hbm" else "TFLOP/s"
    scale = 1e9 if bound == "hbm" else 1e12
    cmd = [str(exe), "bench", workload, str(args.steps), str(args.warmup), "e2e"]
    res = subprocess.run(cmd, capture_output=True, text=True, timeout=1800)
    if res.returncode != 0:
        raise RuntimeError(f"ref_runner failed: {res.stderr[-300:]}")
    r = json.loads(res.stdout.strip().splitlines()[-1])
    value = work / (r["warm_ms"] * 1e-3) / scale
    e2e_value = work / (r["e2e_ms"] * 1e-3) / scale
    # Kernel-only time of the reference's launches (ncu launch list,
    # committed under profiles/): its warm step also holds a module load per
    # launch and host-side zero fills.
    kernels = None
    kfile = ROOT / "profiles" / "ref_kernels.json"
    if kfile.exists():
        k = json.loads(kfile.read_text()).get(workload)
        if k:
            kernels = dict(k)
            kernels["value"] = round(work / (k["kernel_ms_per_step"] * 1e-3) / scale, 4)
            kernels["unit"] = unit
    config = _config_keys(workload, 1)
    return {
        "impl": "reference", "metric": CONFIG_METRIC[workload], "value": round(value, 4),
        "unit": unit, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(r["warm_ms"], 4), "higher_is_better": True,
        "scaling": "strong" if workload in ROW_SHARDED else "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (same seeds and generator as the porch_b200 arm)",
        "config": config,
        "setup": {"reference": "AkhilSamavedam/porch compiled from source",
                  "path": "materialize(expr) + synchronize() through the reference's C++ API "
                          "(NVRTC JIT, one GPU: the reference has no multi-GPU path)",
                  "staged": r.get("staged") if workload == "c5_mlp" else None},
        "e2e": {"value": round(e2e_value, 4), "unit": unit, "h2d_bytes_per_step": r["h2d_bytes"],
                "d2h_bytes_per_step": r["d2h_bytes"], "ms_per_step": round(r["e2e_ms"], 4)},
        "cpu_baseline": {"value": round(value, 4), "unit": unit, "cores": 1, "kind": "reference",
                         "sample": "the reference has no CPU implementation of the path; "
                                   "this is its own NVRTC-JIT GPU path, timed on the same box"},
        "kernel_only": kernels,
        "cold_ms": r["cold_ms"],
    }


def run_reference(args, rank, world, dist):
    if rank != 0:
        return
    exe = ROOT / "oracle" / "_ref" / "ref_runner"
    if not exe.exists():
        print(json.dumps({"impl": "reference", "unavailable":
                          "oracle/_ref/ref_runner was not built (reference sources absent)"}))
        return
    try:
        line = reference_record(args.workload, args, world)
    except RuntimeError as exc:
        print(json.dumps({"impl": "reference", "unavailable": str(exc)}))
        return
    if not args.no_extra and world == 1:
        extra = {}
        for name in sorted(EXTRA_SINGLE + EXTRA_SHARDED):
            if name == args.workload:
                continue
            try:
                r = reference_record(name, args, world)
                extra[name] = {k: r[k] for k in ("metric", "value", "unit", "ms_per_step", "config", "e2e",
                                                  "kernel_only", "cold_ms")}
            except RuntimeError as exc:
                extra[name] = {"unavailable": str(exc)}
        line["extra"] = extra
    print(json.dumps(line), flush=True)


def measure_tf32_peak() -> None:
    """cuBLAS TF32 GEMM throughput (torch.matmul, fp32 inputs with TF32
    allowed), 8192^3, best of 10 after warm-up: the tensor-pipe ceiling for
    one TF32 product. A 3xTF32 kernel's fp32-equivalent ceiling is a third."""
    import torch

    torch.backends.cuda.matmul.allow_tf32 = True
    n = 8192
    a = torch.randn(n, n, device="cuda")
    b = torch.randn(n, n, device="cuda")
    for _ in range(3):
        a @ b
    torch.cuda.synchronize()
    best = 1e9
    for _ in range(10):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        a @ b
        e.record()
        e.synchronize()
        best = min(best, s.elapsed_time(e))
    tf = 2 * n ** 3 / (best * 1e-3) / 1e12
    print(json.dumps({"tf32_tflops": round(tf, 1), "ms": round(best, 4),
                      "how": "torch.matmul fp32 8192^3 allow_tf32, best of 10"}))


def main():
    if "--measure-tf32-peak" in sys.argv:
        measure_tf32_peak()
        return
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="porch_b200", choices=["porch_b200", "reference"])
    ap.add_argument("--workload", default="c5_mlp", choices=sorted(CONFIGS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true",
                    help="time the headline workload only (not the other configurations)")
    args = ap.parse_args()
    rank, world, local, dist = dist_setup(args.gpus)
    try:
        if args.impl == "reference":
            run_reference(args, rank, world, dist)
        else:
            run_ours(args, rank, world, local, dist)
    finally:
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()

#!/usr/bin/env python
"""Codec benchmark on B200: the BASELINE configurations through the cuda_zlib API.

Headline workload (default, any N): config 4a, 65,536 independent files of
exactly 64 KiB (4 GiB) with the config-2 content mix (seed 4).  The files
are assigned to ranks by the LPT planner (cuda_zlib.sharding) from their
sizes and content kinds; each rank decodes its files' CPU-zlib level-6
streams with decompress_zlib_batch_checked and compresses its files at
chunk_bytes=32768 with compress_zlib_batch_padded, in calls within the batch
bounds (4096 and 4095 files of 64 KiB).  One step = every rank's share:
2 x 4 GiB of uncompressed bytes for the whole job.

  value    uncompressed GB/s (1e9 B/s), whole job: 2 x 4 GiB / the slowest
           rank's device time (CUDA events on the codec's stream), inputs
           resident in HBM and larger than L2 (L2 also flushed per step);
  e2e      the same step through the host-buffer counterparts of those calls
           (decompress_zlib_batch_checked_host, and
           compress_zlib_batch_packed_host, which returns the streams back
           to back; copies pipelined with the kernels) from inputs in pinned
           host memory to results in pinned host memory, copies inside the
           timed region (host wall clock, slowest rank);
  roofline the dominant kernel's algorithmic bytes (C + U of the calls it
           served) over its event-timed device time, against the measured
           HBM copy bandwidth (MEASURED_PEAKS.json);
  cpu_baseline  Python's zlib on a bounded sample of the same files:
           zlib.decompress of the level-6 streams and zlib.compress at level
           1, one file per task in a multiprocessing pool (fork, inputs
           inherited) over all host cores;
  configs  (N = 1 only) the same measurements for configs 0, 1, 2, 3 and 4b.

--impl reference times the reference's CPU path, which for this codec is
Python's zlib (the reference's own CPU baseline, benchmarks/benchmark.py:
126-169): the whole config-4a step (all 65,536 files, both directions) in a
multiprocessing pool over all host cores, rank 0 only.
"""
import argparse
import ctypes
import functools
import json
import multiprocessing
import os
import subprocess
import sys
import threading
import time
import zlib
from concurrent.futures import ThreadPoolExecutor

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "cuda-zlib_b200"))
sys.path.insert(0, ROOT)

import workloads  # noqa: E402

MIB = 1 << 20
CHUNK = 32768
FILE = 65536
FILES = 65536
CPU_LEVEL = 1  # CPU-side compression level of the baseline (zlib's fastest)

METRIC = "decompress & compress GB/s (uncompressed bytes)"
CONFIG = {"workload": "config4a: 65,536 files x 64 KiB (seed 4), config-2 content mix; "
                      "decode their zlib level-6 streams (decompress_zlib_batch_checked) and "
                      "compress at chunk_bytes=32768 (compress_zlib_batch_padded)",
          "files": FILES, "file_bytes": FILE, "chunk_bytes": CHUNK,
          "uncompressed_bytes_per_step": 2 * FILES * FILE,
          "parallelism": "files LPT-sharded over ranks",
          "l2": "inputs larger than L2; L2 also flushed between steps"}
# Estimated compressed fraction of each content kind (text, random, runs):
# the LPT weights, known to every rank without compressing anything.
KIND_RATIO = (0.36, 1.0, 0.05)


# ------------------------------------------------------------------ helpers
def measured_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as handle:
            return float(json.load(handle)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def committed_traffic(workload, kernel):
    """DRAM bytes per launch of `kernel` from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "kernel_traffic.json")
    try:
        with open(path) as handle:
            return json.load(handle).get(workload, {}).get(kernel)
    except (OSError, ValueError, AttributeError):
        return None


class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        # nvidia-smi numbers GPUs physically and ignores CUDA_VISIBLE_DEVICES:
        # query the GPU that the CUDA device index maps to (a physical index
        # or a UUID, both accepted by -i).
        visible = [v.strip() for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",")
                   if v.strip()]
        self.index = visible[index] if index < len(visible) else str(index)
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), "--query-gpu=" + self.QUERY,
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.5)  # nvidia-smi's first sample lands before the timed region
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [line for line in out.splitlines() if line.strip()]

    def summary(self):
        sms, maxes, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in getattr(self, "lines", []):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sms.append(float(parts[1]))
                maxes.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        if not sms:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": float(np.median(sms)), "sm_max_mhz": max(maxes),
                "reasons": sorted(reasons), "samples": len(sms)}


# ------------------------------------------------------------------ config 4a inputs
def plan_4a(world):
    """LPT plan of the config-4a files over `world` ranks (same on every rank)."""
    from cuda_zlib import sharding
    kinds, _ = workloads.config4a_kinds(FILES)
    weights = [FILE + int(FILE * KIND_RATIO[k]) for k in kinds.tolist()]
    return sharding.plan_files(weights, world)


def inputs_4a(indices):
    """(packed files, list of level-6 streams) of the given config-4a files."""
    packed, _ = workloads.config4a_files(indices)
    streams = workloads.zlib_files(packed, FILE, 6)
    return packed, streams


# ------------------------------------------------------------------ CPU baseline
# Inputs of the pool's tasks, set before the pool forks so that the workers
# inherit them instead of receiving pickles.
_CPU_INPUTS = {}


def _cpu_task(k):
    packed, streams = _CPU_INPUTS["files"], _CPU_INPUTS["streams"]
    n = len(zlib.decompress(streams[k]))
    n += len(zlib.compress(packed[k * FILE:(k + 1) * FILE], CPU_LEVEL))
    return n


def cpu_pool(packed, streams, processes):
    """A fork pool whose workers hold the files and streams (made before any
    CUDA call: a pool forked after CUDA initialisation can hang)."""
    _CPU_INPUTS["files"], _CPU_INPUTS["streams"] = packed, streams
    return multiprocessing.get_context("fork").Pool(processes)


def cpu_step(pool, count):
    """One pass of zlib.decompress + zlib.compress over files [0, count)."""
    start = time.perf_counter()
    pool.map(_cpu_task, range(count), chunksize=max(1, count // (8 * pool._processes)))
    return time.perf_counter() - start


def run_reference(args, rank, world):
    """The reference arm: Python's zlib on the whole config-4a step."""
    if rank != 0:
        return
    cores = os.cpu_count() or 1
    packed, streams = inputs_4a(range(FILES))
    pool = cpu_pool(packed, streams, cores)
    try:
        for _ in range(args.warmup):
            cpu_step(pool, FILES)
        times = [cpu_step(pool, FILES) for _ in range(args.steps)]
    finally:
        pool.close()
        pool.join()
    seconds = sum(times) / len(times)
    value = 2 * FILES * FILE / seconds / 1e9
    sample = ("whole config-4a step: zlib.decompress of all 65,536 level-6 streams and "
              "zlib.compress(level 1) of all 65,536 files, one file per task, "
              "multiprocessing pool (fork) of %d processes" % cores)
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(seconds * 1e3, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "u8", "data": "synthetic", "config": CONFIG,
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": cores,
                         "kind": "reference", "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0}}), flush=True)


# ------------------------------------------------------------------ GPU timing
class Timing:
    """Device-time steps with the library's per-kernel event totals."""

    NAMES = ("serial_inflate_kernel", "discover_kernel", "validate_kernel", "describe_kernel",
             "symbols_kernel", "expand_kernel", "resolve_kernel", "stage_resolve_kernel",
             "encode_chunks_kernel", "encode_pack_kernel")

    def __init__(self, torch, lib, device, flush):
        self.torch, self.lib, self.device, self.flush = torch, lib, device, flush
        lib.cuda_zlib_b200_profile.argtypes = [ctypes.c_int]
        lib.cuda_zlib_b200_profile_read.argtypes = [
            ctypes.c_char_p, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_uint64)]
        lib.cuda_zlib_b200_launches.restype = ctypes.c_uint64

    def run(self, step, steps, world, clocks=True):
        """Time `steps` calls of step(); returns (seconds, clock summary,
        launches, {kernel: (total ms, launches)})."""
        torch = self.torch
        stream = torch.cuda.current_stream(self.device)
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        self.lib.cuda_zlib_b200_profile(1)
        before = self.lib.cuda_zlib_b200_launches()
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        sampler = ClockSampler(self.device.index) if clocks else None
        if sampler:
            sampler.__enter__()
        try:
            for k in range(steps):
                self.flush.fill_(k & 255)
                starts[k].record(stream)
                step()
                ends[k].record(stream)
            torch.cuda.synchronize()
        finally:
            if sampler:
                sampler.__exit__(None, None, None)
        launched = self.lib.cuda_zlib_b200_launches() - before
        if world > 1:
            torch.distributed.barrier()
        kernels = {}
        for name in self.NAMES:
            total, count = ctypes.c_double(), ctypes.c_uint64()
            self.lib.cuda_zlib_b200_profile_read(name.encode(), ctypes.byref(total),
                                                 ctypes.byref(count))
            if count.value:
                kernels[name] = (total.value, count.value)
        self.lib.cuda_zlib_b200_profile(0)
        seconds = sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / 1e3
        return seconds, (sampler.summary() if sampler else None), launched, kernels


def max_over_ranks(torch, value, device, world):
    if world > 1:
        t = torch.tensor([value], dtype=torch.float64, device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        value = float(t.item())
    return value


DECODE_KERNELS = ("serial_inflate_kernel", "discover_kernel", "validate_kernel",
                  "describe_kernel", "symbols_kernel", "expand_kernel", "resolve_kernel",
                  "stage_resolve_kernel")


def roofline(workload, kernels, steps, decode_bytes, encode_bytes):
    """Dominant kernel's achieved GB/s: the algorithmic bytes (C + U) of the
    calls it served per step over its device time per step."""
    if not kernels:
        return None
    name, (total_ms, launches) = max(kernels.items(), key=lambda kv: kv[1][0])
    served = decode_bytes if name in DECODE_KERNELS else encode_bytes
    per_step_s = total_ms / steps / 1e3
    achieved = served / per_step_s / 1e9
    peak, kind = measured_peak()
    per_launch = served * steps / launches
    return {"bound": "hbm", "kernel": name, "achieved": round(achieved, 2), "peak": peak,
            "peak_kind": kind, "unit": "GB/s", "frac": round(achieved / peak, 5),
            "traffic": committed_traffic(workload, name),
            "algorithmic_bytes_per_launch": int(per_launch),
            "launch_ms": round(total_ms / launches, 4),
            "share_of_step": None}


def wall_steps(torch, step, warmup, steps):
    """Host wall-clock seconds per step (device synchronized around each)."""
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    times = []
    for _ in range(steps):
        torch.cuda.synchronize()
        start = time.perf_counter()
        step()
        torch.cuda.synchronize()
        times.append(time.perf_counter() - start)
    return sum(times) / len(times)


# ------------------------------------------------------------------ config 4a on the GPU
def groups_of(count, per):
    return [(a, min(a + per, count)) for a in range(0, count, per)]


def run_gpu(args, rank, world):
    plan = plan_4a(world)
    if args.profile_files:
        # A small case of the same kernels for ncu captures: not a bench line.
        plan = [p[:args.profile_files] for p in plan]
    mine = plan[rank]
    packed, streams = inputs_4a(mine)
    count = len(mine)
    cores = os.cpu_count() or 1
    sample_files = min(count, args.cpu_files)
    pool = None
    if world == 1 and not args.no_cpu:
        pool = cpu_pool(packed, streams, cores)

    import torch
    import cuda_zlib as codec
    from cuda_zlib import _native

    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)) % torch.cuda.device_count())
    device = torch.device("cuda", torch.cuda.current_device())
    codec.compile_kernels(device)
    lib = _native.library()
    flush = torch.empty(256 * MIB, dtype=torch.uint8, device=device)
    timing = Timing(torch, lib, device, flush)

    in_sizes = [len(s) for s in streams]
    z_packed = np.frombuffer(b"".join(streams), dtype=np.uint8)
    z_offsets = np.concatenate(([0], np.cumsum(in_sizes))).astype(np.int64)
    raw_dev = torch.from_numpy(packed).to(device)
    z_dev = torch.from_numpy(z_packed.copy()).to(device)
    decode_groups = groups_of(count, (1 << 28) // FILE)
    capacity = FILE + 5 * (FILE // CHUNK) + 6
    encode_groups = groups_of(count, (1 << 28) // capacity)
    results = {}

    def step():
        outs = []
        for a, b in decode_groups:
            outs.append(codec.decompress_zlib_batch_checked(
                z_dev[int(z_offsets[a]):int(z_offsets[b])], in_sizes[a:b], [FILE] * (b - a),
                device))
        for a, b in encode_groups:
            outs.append(codec.compress_zlib_batch_padded(
                raw_dev[a * FILE:b * FILE], [FILE] * (b - a), device, chunk_bytes=CHUNK))
        results["last"] = outs
        return outs

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    # Verify the last warm-up step: decoded files equal the sources; every
    # encoded stream decodes back to its file with the host's zlib.
    outs = results["last"]
    for (a, b), (out, meta) in zip(decode_groups, outs[:len(decode_groups)]):
        assert not meta.cpu().numpy().any()
        assert torch.equal(out, raw_dev[a * FILE:b * FILE])
    encoded = 0
    for (a, b), (slots, meta) in zip(encode_groups, outs[len(decode_groups):]):
        meta = meta.cpu().numpy()
        assert not meta[:, 1].any()
        host = slots.cpu().numpy()
        lengths = meta[:, 0].astype(np.int64)
        encoded += int(lengths.sum())
        ok = workloads.parallel_map(
            lambda k: zlib.decompress(host[k * capacity:k * capacity + lengths[k]].tobytes()) ==
            packed[(a + k) * FILE:(a + k + 1) * FILE].tobytes(), range(b - a))
        assert all(ok)
    results.clear()

    seconds, clocks, launched, kernels = timing.run(step, args.steps, world)
    seconds = max_over_ranks(torch, seconds, device, world)
    per_step = seconds / args.steps
    total_units = 2 * sum(len(p) for p in plan) * FILE
    value = total_units / per_step / 1e9
    my_u = count * FILE
    line_roofline = roofline("config4a", kernels, args.steps, my_u + int(z_offsets[-1]),
                             my_u + encoded)
    if line_roofline:
        name = line_roofline["kernel"]
        line_roofline["share_of_step"] = round(kernels[name][0] / args.steps / (per_step * 1e3), 4)

    # End to end through the host-buffer counterparts of the two packed
    # calls, inputs in pinned host memory, results in pinned host memory.
    e2e = None
    if not args.no_e2e:
        raw_pin = torch.from_numpy(packed).pin_memory().numpy()
        z_pin = torch.from_numpy(z_packed.copy()).pin_memory().numpy()
        sizes = np.full(count, FILE, dtype=np.int64)
        z_sizes = np.asarray(in_sizes, dtype=np.int64)
        box = {}
        side = ThreadPoolExecutor(max_workers=1)

        def e2e_step():
            # The previous step's results are released first, as a caller
            # reusing its result buffers would, so the pinned host memory of
            # the results comes from the allocator's cache rather than new
            # page locking.  The decode and the compression are independent
            # jobs, issued from two host threads as a caller with both would:
            # the decode's copies out and the compression's copies in then
            # share the host link's two directions while the kernels run.
            box.clear()
            decoded = side.submit(codec.decompress_zlib_batch_checked_host, z_pin, z_sizes,
                                  sizes, device)
            streams, emeta = codec.compress_zlib_batch_packed_host(raw_pin, sizes, device,
                                                                   chunk_bytes=CHUNK)
            out, meta = decoded.result()
            assert not meta.any() and not emeta[:, 1].any()
            box["result"] = (out, streams, emeta)

        e2e_seconds = wall_steps(torch, e2e_step, 1, args.e2e_steps)
        side.shutdown()
        out, streams, emeta = box["result"]
        assert np.array_equal(out, packed) and int(emeta[:, 0].sum()) == encoded
        assert streams.size == encoded
        e2e_seconds = max_over_ranks(torch, e2e_seconds, device, world)
        e2e = {"value": round(total_units / e2e_seconds / 1e9, 4), "unit": "GB/s",
               "h2d_bytes_per_step": int(z_offsets[-1]) + my_u,
               "d2h_bytes_per_step": my_u + encoded + 16 * count,
               "timer": "host wall clock, slowest rank",
               "calls": "decompress_zlib_batch_checked_host + compress_zlib_batch_packed_host, "
                        "issued from two host threads",
               "steps": args.e2e_steps}

    configs = None
    if world == 1 and not args.no_configs:
        configs = run_configs(args, torch, codec, device, timing)

    cpu = None
    if pool is not None:
        cpu_step(pool, min(sample_files, 1024))
        t = cpu_step(pool, sample_files)
        pool.close()
        pool.join()
        cpu = {"value": round(2 * sample_files * FILE / t / 1e9, 4), "unit": "GB/s",
               "cores": cores, "kind": "reference",
               "sample": "first %d of the 65,536 config-4a files: zlib.decompress of their "
                         "level-6 streams + zlib.compress(level 1), one file per task, "
                         "multiprocessing pool (fork) of %d processes" % (sample_files, cores)}
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": round(value, 4), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per_step * 1e3, 3),
        "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "u8", "data": "synthetic", "config": CONFIG,
        "compression_ratio_rank0": round(encoded / my_u, 5),
        "zlib6_ratio_rank0": round(int(z_offsets[-1]) / my_u, 5),
        "roofline": line_roofline,
        "kernels_ms_per_step": {k: round(v[0] / args.steps, 3) for k, v in kernels.items()},
        "e2e": e2e, "cpu_baseline": cpu, "clocks": clocks, "gpu_launches": launched,
        "configs": configs,
    }
    if args.profile_files:
        line["config"] = dict(CONFIG, profile_case_files_per_rank=args.profile_files)
        line["profile_case"] = "a small case for profiler captures, not a benchmark result"
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ configs 0-3, 4b (N = 1)
def _device_tensor(torch, array, device):
    return torch.from_numpy(np.ascontiguousarray(array)).to(device)


def _pinned(torch, data):
    array = np.frombuffer(data, dtype=np.uint8) if not isinstance(data, np.ndarray) else data
    return torch.from_numpy(np.ascontiguousarray(array)).pin_memory().numpy()


def measure_config(args, torch, timing, name, step, e2e_step, units, decode_bytes,
                   encode_bytes, extra):
    """Device and end-to-end throughput of one configuration's step."""
    steps, warmup = args.config_steps, args.config_warmup
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    seconds, _, launched, kernels = timing.run(step, steps, 1, clocks=False)
    per_step = seconds / steps
    result = {"value": round(units / per_step / 1e9, 4), "unit": "GB/s",
              "ms_per_step": round(per_step * 1e3, 3), "steps": steps, "warmup": warmup,
              "uncompressed_bytes_per_step": units, "gpu_launches": launched,
              "roofline": roofline(name, kernels, steps, decode_bytes, encode_bytes),
              "kernels_ms_per_step": {k: round(v[0] / steps, 3) for k, v in kernels.items()}}
    if result["roofline"]:
        k = result["roofline"]["kernel"]
        result["roofline"]["share_of_step"] = round(kernels[k][0] / steps / (per_step * 1e3), 4)
    if e2e_step is not None and not args.no_e2e:
        e2e_seconds = wall_steps(torch, e2e_step, 1, min(steps, 3))
        result["e2e"] = {"value": round(units / e2e_seconds / 1e9, 4), "unit": "GB/s",
                         "timer": "host wall clock"}
    result.update(extra)
    return result


def run_configs(args, torch, codec, device, timing):
    """Configs 0, 1, 2, 3 and 4b on this GPU, each verified before timing."""
    wanted = [c for c in args.configs.split(",") if c]
    out = {}
    # CPU-zlib streams of the large configs are made on host threads while
    # the smaller configs run on the GPU.
    pending = {}
    background = ThreadPoolExecutor(max_workers=4)
    # End to end, a batch config's decode and compression are independent
    # jobs, issued from two host threads as a caller with both would, so one
    # call's copies overlap the other's kernels.
    callers = ThreadPoolExecutor(max_workers=2)

    def concurrently(calls):
        for future in [callers.submit(*call) for call in calls]:
            future.result()
    if "3" in wanted:
        records = workloads.config3_records()
        raw3 = records.tobytes()
        pending["3l9"] = background.submit(workloads.zlib_stream, raw3, 9)
        pending["3fixed"] = background.submit(workloads.zlib_stream, raw3, 1, zlib.Z_FIXED)
    if "4b" in wanted:
        streams4b = workloads.config4b_streams()
        for key, raw in streams4b.items():
            pending["4b" + key] = background.submit(workloads.zlib_stream, raw.tobytes(), 6)

    def single(name, raws, payloads, chunks):
        """Decode every payload to its raw; compress every (raw, chunk)."""
        dev_payloads = [(_device_tensor(torch, np.frombuffer(p, dtype=np.uint8), device), n)
                        for p, n in payloads]
        dev_raws = [(_device_tensor(torch, r, device), c) for r, c in zip(raws, chunks)]

        def step():
            res = [codec.decompress_zlib_checked(p, n, device) for p, n in dev_payloads]
            res += [codec.compress_zlib_padded(r, device, chunk_bytes=c) for r, c in dev_raws]
            return res

        res = step()
        torch.cuda.synchronize()
        lengths = []
        for (p, n), (o, m) in zip(payloads, res[:len(payloads)]):
            assert [int(v) for v in m.cpu()] == [0, 0], name
        for r, (o, m) in zip(raws, res[len(payloads):]):
            length, status = (int(v) for v in m.cpu())
            assert status == 0, name
            assert zlib.decompress(o[:length].cpu().numpy().tobytes()) == r.tobytes(), name
            lengths.append(length)
        pin_payloads = [(_pinned(torch, p), n) for p, n in payloads]
        pin_raws = [(_pinned(torch, r), c) for r, c in zip(raws, chunks)]

        def e2e_step():
            # One call at a time: each single-stream call already overlaps its
            # own copies, and concurrent calls over 1 GiB streams measured
            # slower.
            for p, n in pin_payloads:
                codec.decompress_zlib_host(p, n, device)
            for r, c in pin_raws:
                codec.compress_zlib_host(r, device, chunk_bytes=c)

        units = sum(n for _, n in payloads) + sum(r.size for r in raws)
        decode_bytes = sum(len(p) + n for p, n in payloads)
        encode_bytes = sum(r.size for r in raws) + sum(lengths)
        return step, e2e_step, units, decode_bytes, encode_bytes, lengths

    if "0" in wanted:
        text = np.frombuffer(workloads.zipf_text(16 * MIB, 0), dtype=np.uint8)
        l6 = workloads.zlib_stream(text.tobytes(), 6)
        step, e2e, units, db, eb, lengths = single("config0", [text], [(l6, text.size)], [CHUNK])
        out["config0"] = measure_config(
            args, torch, timing, "config0", step, e2e, units, db, eb,
            {"workload": "16 MiB Zipf text (seed 0): decode its zlib level-6 stream, compress "
                         "at chunk_bytes=32768",
             "compression_ratio": round(lengths[0] / text.size, 5),
             "zlib6_ratio": round(len(l6) / text.size, 5)})
    if "1" in wanted:
        samples = np.frombuffer(workloads.config1_float32(), dtype=np.uint8)
        l1 = workloads.zlib_stream(samples.tobytes(), 1)
        l6 = workloads.zlib_stream(samples.tobytes(), 6)
        step, e2e, units, db, eb, lengths = single(
            "config1", [samples], [(l1, samples.size), (l6, samples.size)], [CHUNK])
        out["config1"] = measure_config(
            args, torch, timing, "config1", step, e2e, units, db, eb,
            {"workload": "64 MiB float32 random walk (seed 1): decode its zlib level-1 and "
                         "level-6 streams (to pinned host in e2e), compress at 32768",
             "compression_ratio": round(lengths[0] / samples.size, 5),
             "zlib1_ratio": round(len(l1) / samples.size, 5),
             "zlib6_ratio": round(len(l6) / samples.size, 5)})
    if "2" in wanted:
        files = workloads.config2_files()
        streams = workloads.parallel_map(lambda f: workloads.zlib_stream(f, 6), files)
        sizes, in_sizes = [len(f) for f in files], [len(s) for s in streams]
        raw_dev = _device_tensor(torch, np.frombuffer(b"".join(files), dtype=np.uint8), device)
        z_dev = _device_tensor(torch, np.frombuffer(b"".join(streams), dtype=np.uint8), device)

        def step2():
            return (codec.decompress_zlib_batch_checked(z_dev, in_sizes, sizes, device),
                    codec.compress_zlib_batch_padded(raw_dev, sizes, device, chunk_bytes=CHUNK))

        (out2, meta2), (slots2, emeta2) = step2()
        assert not meta2.cpu().numpy().any()
        assert torch.equal(out2, raw_dev)
        emeta2 = emeta2.cpu().numpy()
        assert not emeta2[:, 1].any()
        z_pin = _pinned(torch, np.frombuffer(b"".join(streams), dtype=np.uint8))
        r_pin = _pinned(torch, np.frombuffer(b"".join(files), dtype=np.uint8))

        def e2e2():
            concurrently([(codec.decompress_zlib_batch_checked_host, z_pin, in_sizes, sizes,
                           device),
                          (functools.partial(codec.compress_zlib_batch_packed_host,
                                             chunk_bytes=CHUNK), r_pin, sizes, device)])

        total = sum(sizes)
        out["config2"] = measure_config(
            args, torch, timing, "config2", step2, e2e2, 2 * total,
            total + sum(in_sizes), total + int(emeta2[:, 0].sum()),
            {"workload": "4096 files (seed 2), log-uniform 256 B-256 KiB, 1% empty, config-2 "
                         "mix: batch decode of their zlib level-6 streams, batch compress at "
                         "32768",
             "e2e_calls": "decompress_zlib_batch_checked_host + "
                          "compress_zlib_batch_packed_host, issued from two host threads",
             "compression_ratio": round(int(emeta2[:, 0].sum()) / total, 5),
             "zlib6_ratio": round(sum(in_sizes) / total, 5)})
    if "3" in wanted:
        l9, fixed = pending["3l9"].result(), pending["3fixed"].result()
        step, e2e, units, db, eb, lengths = single(
            "config3", [records, records], [(l9, records.size), (fixed, records.size)],
            [CHUNK, 262144])
        out["config3"] = measure_config(
            args, torch, timing, "config3", step, e2e, units, db, eb,
            {"workload": "1 GiB of 64-byte records (seed 3): decode its zlib level-9 and "
                         "level-1 Z_FIXED streams, compress at 32768 and 262144",
             "compression_ratio_32768": round(lengths[0] / records.size, 5),
             "compression_ratio_262144": round(lengths[1] / records.size, 5),
             "zlib9_ratio": round(len(l9) / records.size, 5),
             "zlib1_fixed_ratio": round(len(fixed) / records.size, 5)})
    if "4b" in wanted:
        keys = ("zeros", "random", "period")
        raws = [streams4b[k] for k in keys]
        payloads = [(pending["4b" + k].result(), streams4b[k].size) for k in keys]
        step, e2e, units, db, eb, lengths = single("config4b", raws, payloads, [65535] * 3)
        out["config4b"] = measure_config(
            args, torch, timing, "config4b", step, e2e, units, db, eb,
            {"workload": "three 256 MiB streams (seed 4): all-zero, uniform random, period-32768 "
                         "repeats; decode their zlib level-6 streams, compress at 65535",
             "compression_ratio": {k: round(n / (256 * MIB), 5) for k, n in zip(keys, lengths)},
             "zlib6_ratio": {k: round(len(p) / (256 * MIB), 5)
                             for k, (p, _) in zip(keys, payloads)}})
    background.shutdown()
    callers.shutdown()
    return out


# ------------------------------------------------------------------ main
def main():
    # Scratch kept by the codec's workspace pool between calls (the
    # reference's CUDA_ZLIB_WORKSPACE_RETENTION_BYTES, default 1 GiB): the
    # single-stream configs need several GiB of scratch per call, which a
    # 1 GiB release threshold would unmap and map again every step.  A
    # caller's own setting wins.
    os.environ.setdefault("CUDA_ZLIB_WORKSPACE_RETENTION_BYTES", str(32 << 30))
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=5)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", choices=["ours", "reference"], default="ours")
    parser.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    parser.add_argument("--no-e2e", action="store_true", help="skip the host-buffer legs")
    parser.add_argument("--no-configs", action="store_true",
                        help="skip the per-config sub-results (N = 1)")
    parser.add_argument("--configs", default="0,1,2,3,4b",
                        help="configs measured beside the headline at N = 1")
    parser.add_argument("--e2e-steps", type=int, default=3)
    parser.add_argument("--config-steps", type=int, default=3)
    parser.add_argument("--config-warmup", type=int, default=3)
    parser.add_argument("--cpu-files", type=int, default=8192,
                        help="config-4a files in the CPU baseline's bounded sample")
    parser.add_argument("--profile-files", type=int, default=0,
                        help="only this many config-4a files per rank: a small case for "
                             "profiler captures (its line is not a benchmark result)")
    args = parser.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if world > 1:
        import datetime
        import torch
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
    try:
        run_gpu(args, rank, world)
    finally:
        if world > 1:
            import torch
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()

#!/usr/bin/env python
"""Codec benchmark on B200: BASELINE config 1 through the cuda_zlib API.

Workload (one step, N=1): the 64 MiB float32 random walk of config 1
(16,777,216 samples, seed 1: x[i] = x[i-1] + N(0, 1e-3) plus
1e-2 * sin(2 pi 60 i / 4096)), compressed by CPU zlib at levels 1 and 6
outside the timed region.  A step decodes both streams
(decompress_zlib_checked) and compresses the array at chunk_bytes=32768
(compress_zlib_padded): 3 x 64 MiB of uncompressed bytes.

  value  = uncompressed GB/s (1e9 B/s) with inputs resident in HBM, timed
           with CUDA events on the codec's stream, L2 flushed between steps;
  e2e    = the same step through the host-buffer API (decompress_zlib_host
           and compress_zlib_host on inputs in pinned host memory), with the
           H2D copies of the inputs and the D2H copies of the results inside
           the timed region;
  roofline = the dominant kernel's algorithmic bytes (U + C per launch)
           over its event-timed device time, against the measured HBM copy
           bandwidth;
  cpu_baseline = the CPU oracle (the reference's algorithms restated in C)
           on a 16 MiB sample of the same data.

--gpus N > 1 runs one process per GPU (torchrun); single-stream decode has
no shard structure, so each rank runs an independent replica (weak scaling)
and value = all ranks' bytes / the slowest rank's time.
--impl reference times the reference's CPU path: the reference has no CPU
codec and its CUDA sources cannot be built here (generated from Python
strings, needs XLA FFI headers), so the arm runs the oracle port with all
host threads on the same workload.
"""
import argparse
import hashlib
import json
import os
import subprocess
import sys
import threading
import time
import zlib

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "cuda-zlib_b200"))

MIB = 1 << 20
CHUNK = 32768
L2_BYTES = 126 * MIB


# ------------------------------------------------------------------ data
def config1_float32(samples=16777216, seed=1):
    """Config 1: float32 LE random walk plus a 60-cycle-per-4096 sine."""
    rng = np.random.default_rng(seed)
    walk = np.cumsum(rng.normal(0.0, 1e-3, samples))
    i = np.arange(samples, dtype=np.float64)
    x = walk + 1e-2 * np.sin(2 * np.pi * 60 * i / 4096)
    return x.astype("<f4").tobytes()


def zlib_stream(raw, level, strategy=zlib.Z_DEFAULT_STRATEGY):
    c = zlib.compressobj(level, zlib.DEFLATED, zlib.MAX_WBITS, 8, strategy)
    return c.compress(raw) + c.flush()


def workload(size_mib=64):
    raw = config1_float32()[:size_mib * MIB]
    streams = {}

    def make(level):
        streams[level] = zlib_stream(raw, level)

    threads = [threading.Thread(target=make, args=(level,)) for level in (1, 6)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    return raw, streams[1], streams[6]


# ------------------------------------------------------------------ helpers
def measured_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as handle:
            return float(json.load(handle)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def committed_traffic(kernel):
    """DRAM bytes per launch of `kernel` from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "kernel_traffic.json")
    try:
        with open(path) as handle:
            return json.load(handle).get(kernel)
    except (OSError, ValueError):
        return None


class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), "--query-gpu=" + self.QUERY,
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
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


# ------------------------------------------------------------------ CPU side
def cpu_port(raw, l1, l6, threads):
    """One sample step of the oracle port: decode both streams (one thread
    each: a single stream is serial) and compress the array chunk-parallel."""
    from oracle import oracle
    import ctypes
    lib = oracle.lib()
    results = {}

    def decode(name, payload):
        out, status = oracle.inflate_serial(payload, len(raw))
        results[name] = status == 0 and out == raw

    src = np.frombuffer(raw, dtype=np.uint8)
    chunks = max(1, -(-len(raw) // CHUNK))
    slot = (CHUNK * 9 + 7) // 8 + 16
    slots = np.zeros(chunks * slot, dtype=np.uint8)
    sizes = np.zeros(chunks, dtype=np.uint32)
    per = -(-chunks // max(1, threads - 2))

    def encode(first):
        count = min(per, chunks - first)
        if count <= 0:
            return
        lib.oracle_compress_chunks(
            src.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)), len(raw), CHUNK, first, count,
            slots[first * slot:].ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)), slot,
            sizes[first:].ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)))

    workers = [threading.Thread(target=decode, args=("l1", l1)),
               threading.Thread(target=decode, args=("l6", l6))]
    workers += [threading.Thread(target=encode, args=(first,))
                for first in range(0, chunks, per)]
    start = time.perf_counter()
    for w in workers:
        w.start()
    for w in workers:
        w.join()
    elapsed = time.perf_counter() - start
    if not (results.get("l1") and results.get("l6")):
        raise RuntimeError("CPU oracle decode mismatch")
    return elapsed


def cpu_sample():
    """16 MiB of the config-1 data and its zlib streams (bounded CPU work)."""
    raw = config1_float32()[:16 * MIB]
    return raw, zlib_stream(raw, 1), zlib_stream(raw, 6)


def run_reference(args, rank, world):
    if rank != 0:
        return
    from oracle import oracle
    oracle.build()
    threads = os.cpu_count() or 1
    raw, l1, l6 = cpu_sample()
    for _ in range(args.warmup):
        cpu_port(raw, l1, l6, threads)
    times = [cpu_port(raw, l1, l6, threads) for _ in range(args.steps)]
    seconds = sum(times) / len(times)
    value = 3 * len(raw) / seconds / 1e9
    sample = ("16 MiB slice of config 1: zlib L1 + L6 decode (one thread per stream) and "
              "chunk-parallel compress at 32 KiB, oracle port")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(seconds * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u8", "data": "synthetic",
        "config": CONFIG,
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": threads,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU side
METRIC = ("decompress & compress GB/s (uncompressed bytes; zlib L1+L6 decode and "
          "chunk-32768 compress of config 1)")
CONFIG = {"workload": "config1: 64 MiB float32 random walk (seed 1); decode zlib L1 and L6 "
                      "streams, compress at chunk_bytes=32768",
          "uncompressed_bytes_per_step": 3 * 64 * MIB, "chunk_bytes": CHUNK,
          "l2": "flushed between steps (256 MiB write)"}


def run_gpu(args, rank, world):
    import torch
    import cuda_zlib as codec
    from cuda_zlib import _native
    import ctypes

    torch.cuda.set_device(rank % torch.cuda.device_count())
    device = torch.device("cuda", torch.cuda.current_device())
    codec.compile_kernels(device)
    raw, l1, l6 = workload(args.size_mib)
    U = len(raw)
    raw_dev = torch.frombuffer(bytearray(raw), dtype=torch.uint8).to(device)
    l1_dev = torch.frombuffer(bytearray(l1), dtype=torch.uint8).to(device)
    l6_dev = torch.frombuffer(bytearray(l6), dtype=torch.uint8).to(device)
    flush = torch.empty(256 * MIB, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)

    def step():
        o1, m1 = codec.decompress_zlib_checked(l1_dev, U, device)
        o6, m6 = codec.decompress_zlib_checked(l6_dev, U, device)
        c, mc = codec.compress_zlib_padded(raw_dev, device, chunk_bytes=CHUNK)
        return o1, m1, o6, m6, c, mc

    for _ in range(args.warmup):
        result = step()
    torch.cuda.synchronize()
    o1, m1, o6, m6, c, mc = result
    assert [int(v) for v in m1.cpu()] == [0, 0] and [int(v) for v in m6.cpu()] == [0, 0]
    assert o1.cpu().numpy().tobytes() == raw and o6.cpu().numpy().tobytes() == raw
    length, status = (int(v) for v in mc.cpu())
    assert status == 0
    stream_bytes = c[:length].cpu().numpy().tobytes()
    assert zlib.decompress(stream_bytes) == raw
    ratio = length / U

    lib = _native.library()
    lib.cuda_zlib_b200_profile.argtypes = [ctypes.c_int]
    lib.cuda_zlib_b200_profile_read.argtypes = [ctypes.c_char_p, ctypes.POINTER(ctypes.c_double),
                                                ctypes.POINTER(ctypes.c_uint64)]
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    lib.cuda_zlib_b200_launches.restype = ctypes.c_uint64
    lib.cuda_zlib_b200_profile(1)
    launches_before = lib.cuda_zlib_b200_launches()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler(device.index) as clocks:
        for k in range(args.steps):
            flush.fill_(k & 255)
            starts[k].record(stream)
            step()
            ends[k].record(stream)
        torch.cuda.synchronize()
    launched = lib.cuda_zlib_b200_launches() - launches_before
    if world > 1:
        torch.distributed.barrier()
    kernels = {}
    for name in ("serial_inflate_kernel", "discover_kernel", "describe_kernel", "emit_kernel",
                 "encode_chunks_kernel", "encode_pack_kernel"):
        total, launches = ctypes.c_double(), ctypes.c_uint64()
        lib.cuda_zlib_b200_profile_read(name.encode(), ctypes.byref(total), ctypes.byref(launches))
        if launches.value:
            kernels[name] = (total.value, launches.value)
    lib.cuda_zlib_b200_profile(0)
    seconds = sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / 1e3
    if world > 1:
        t = torch.tensor([seconds], dtype=torch.float64, device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        seconds = float(t.item())
    per_step = seconds / args.steps
    value = world * 3 * U / per_step / 1e9

    # Dominant kernel's roofline: algorithmic bytes (U + C per launch).
    algorithmic = {
        "serial_inflate_kernel": (U + len(l1), U + len(l6)),
        "emit_kernel": (U + len(l1), U + len(l6)),
        "describe_kernel": (len(l1), len(l6)),
        "encode_chunks_kernel": (U + length,),
        "encode_pack_kernel": (2 * length,),
        "discover_kernel": (len(l1), len(l6)),
    }
    name, (total_ms, launches) = max(kernels.items(), key=lambda kv: kv[1][0])
    per_launch = algorithmic.get(name, (U,))
    bytes_per_launch = sum(per_launch) / len(per_launch)
    achieved = bytes_per_launch / (total_ms / launches / 1e3) / 1e9
    peak, peak_kind = measured_peak()
    traffic = committed_traffic(name)

    # End to end through the host-buffer API.
    e2e_times = []
    if args.no_e2e:
        e2e_times.append(float("nan"))
    e2e_start = torch.cuda.Event(enable_timing=True)
    e2e_end = torch.cuda.Event(enable_timing=True)
    # Step inputs sit in pinned host memory (page-locked CPU tensors).
    l1_host = torch.frombuffer(bytearray(l1), dtype=torch.uint8).pin_memory()
    l6_host = torch.frombuffer(bytearray(l6), dtype=torch.uint8).pin_memory()
    raw_host = torch.frombuffer(bytearray(raw), dtype=torch.uint8).pin_memory()
    for k in range(0 if args.no_e2e else max(args.warmup, 1) + args.steps):
        flush.fill_(k & 255)
        torch.cuda.synchronize()
        e2e_start.record(stream)
        h1 = codec.decompress_zlib_host(l1_host, U, device)
        h6 = codec.decompress_zlib_host(l6_host, U, device)
        host_stream = codec.compress_zlib_host(raw_host, device, chunk_bytes=CHUNK)
        e2e_end.record(stream)
        torch.cuda.synchronize()
        if k >= max(args.warmup, 1):
            e2e_times.append(e2e_start.elapsed_time(e2e_end) / 1e3)
    if not args.no_e2e:
        assert h1.tobytes() == raw and h6.tobytes() == raw
        assert host_stream.tobytes() == stream_bytes
    e2e_seconds = sum(e2e_times) / len(e2e_times)
    if world > 1:
        t = torch.tensor([e2e_seconds], dtype=torch.float64, device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_seconds = float(t.item())
    e2e_value = world * 3 * U / e2e_seconds / 1e9

    if rank != 0:
        return
    cpu = None
    if world == 1 and not args.no_cpu:
        sample_raw, s1, s6 = cpu_sample()
        threads = os.cpu_count() or 1
        cpu_port(sample_raw, s1, s6, threads)
        cpu_time = cpu_port(sample_raw, s1, s6, threads)
        cpu = {"value": round(3 * len(sample_raw) / cpu_time / 1e9, 4), "unit": "GB/s",
               "cores": threads, "kind": "port",
               "sample": "16 MiB slice of config 1: zlib L1 + L6 decode (one thread per "
                         "stream) and chunk-parallel compress at 32 KiB, oracle port"}
    line = {
        "metric": METRIC, "value": round(value, 4), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per_step * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8",
        "data": "synthetic", "config": dict(CONFIG, uncompressed_bytes_per_step=3 * U,
                                            parallelism="replicas" if world > 1 else "1 GPU",
                                            compression_ratio=round(ratio, 5),
                                            zlib_l1_ratio=round(len(l1) / U, 5),
                                            zlib_l6_ratio=round(len(l6) / U, 5)),
        "roofline": {"bound": "hbm", "kernel": name, "achieved": round(achieved, 2),
                     "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                     "frac": round(achieved / peak, 5),
                     "traffic": traffic,
                     "algorithmic_bytes_per_launch": int(bytes_per_launch),
                     "launch_ms": round(total_ms / launches, 4)},
        "kernels_ms_per_step": {k: round(v[0] / args.steps, 3) for k, v in kernels.items()},
        "e2e": None if args.no_e2e else {
            "value": round(e2e_value, 4), "unit": "GB/s",
            "h2d_bytes_per_step": len(l1) + len(l6) + U,
            "d2h_bytes_per_step": 2 * U + length + 16},
        "cpu_baseline": cpu,
        "clocks": clocks.summary(),
        "gpu_launches": launched,
    }
    print(json.dumps(line), flush=True)


def main():
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=5)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", choices=["ours", "reference"], default="ours")
    parser.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    parser.add_argument("--no-e2e", action="store_true", help="skip the host-buffer leg")
    parser.add_argument("--size-mib", type=int, default=64,
                        help="leading MiB of the config-1 array (64 = the full workload; "
                             "smaller sizes are for profiler captures)")
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
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    try:
        run_gpu(args, rank, world)
    finally:
        if world > 1:
            import torch
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()

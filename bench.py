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
  e2e    = the same step from inputs in pinned host memory to results
           (and statuses) in pinned host memory, with the H2D copies of the
           inputs and the D2H copies of the results inside the timed region
           (host wall clock): copies in on one stream, the three codec calls
           in order on a compute stream, results out on a third stream as each
           call finishes;
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

    # The device-resident step runs its three parts in order on one stream
    # (each part fills the GPU; running them on three streams measured no
    # faster and blurs the per-kernel times).
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
    for name in ("serial_inflate_kernel", "discover_kernel", "validate_kernel", "describe_kernel",
                 "symbols_kernel", "expand_kernel", "resolve_kernel",
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
        "symbols_kernel": (len(l1), len(l6)),
        "expand_kernel": (U, U),
        "resolve_kernel": (U // 8, U // 8),
        "describe_kernel": (len(l1), len(l6)),
        "encode_chunks_kernel": (U + length,),
        "encode_pack_kernel": (2 * length,),
        "discover_kernel": (len(l1), len(l6)),
        "validate_kernel": (len(l1), len(l6)),
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
    # Step inputs sit in pinned host memory (page-locked CPU tensors) and the
    # results end there.  The step is the pipeline a user of the device API
    # writes: the inputs go in on a copy stream, the three codec calls run in
    # order on one compute stream (each waiting for its own input only), and
    # each result goes out on a third stream as soon as its call finishes, so
    # copies overlap compute.  The compressed stream goes out at its exact
    # length, read from the call's metadata.  The host wall clock spans the
    # step from the first copy to the last result and status in host memory.
    l1_host = torch.frombuffer(bytearray(l1), dtype=torch.uint8).pin_memory()
    l6_host = torch.frombuffer(bytearray(l6), dtype=torch.uint8).pin_memory()
    raw_host = torch.frombuffer(bytearray(raw), dtype=torch.uint8).pin_memory()
    out1_host = torch.empty(U, dtype=torch.uint8).pin_memory()
    out6_host = torch.empty(U, dtype=torch.uint8).pin_memory()
    comp_host = torch.empty(U + 5 * (U // CHUNK + 1) + 6, dtype=torch.uint8).pin_memory()
    meta_host = torch.empty(6, dtype=torch.int32).pin_memory()
    copy_in, compute, copy_out = (torch.cuda.Stream(device) for _ in range(3))

    def e2e_step():
        inputs, results = [], []
        with torch.cuda.stream(copy_in):
            for host in (l1_host, l6_host, raw_host):
                ready = torch.cuda.Event()
                inputs.append((host.to(device, non_blocking=True), ready))
                ready.record(copy_in)
        with torch.cuda.stream(compute):
            for k, (data, ready) in enumerate(inputs):
                compute.wait_event(ready)
                out, meta = (codec.decompress_zlib_checked(data, U, device) if k < 2 else
                             codec.compress_zlib_padded(data, device, chunk_bytes=CHUNK))
                done = torch.cuda.Event()
                done.record(compute)
                results.append((out, meta, done))
        with torch.cuda.stream(copy_out):
            for k, (out, meta, done) in enumerate(results[:2]):
                copy_out.wait_event(done)
                (out1_host, out6_host)[k].copy_(out, non_blocking=True)
                meta_host[2 * k:2 * k + 2].copy_(meta.view(torch.int32), non_blocking=True)
            c_out, c_meta, c_done = results[2]
            copy_out.wait_event(c_done)
            meta_host[4:6].copy_(c_meta.view(torch.int32), non_blocking=True)
            copy_out.synchronize()
            length = int(meta_host[4])
            comp_host[:length].copy_(c_out[:length], non_blocking=True)
            copy_out.synchronize()
        status = meta_host.tolist()
        assert status[0] == 0 and status[2] == 0 and status[5] == 0, status
        return length

    e2e_length = 0
    for k in range(0 if args.no_e2e else max(args.warmup, 1) + args.steps):
        flush.fill_(k & 255)
        torch.cuda.synchronize()
        begin = time.perf_counter()
        e2e_length = e2e_step()
        elapsed = time.perf_counter() - begin
        if k >= max(args.warmup, 1):
            e2e_times.append(elapsed)
    if not args.no_e2e:
        assert out1_host.numpy().tobytes() == raw and out6_host.numpy().tobytes() == raw
        assert comp_host[:e2e_length].numpy().tobytes() == stream_bytes
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
            "d2h_bytes_per_step": 2 * U + length + 24, "timer": "host wall clock"},
        "cpu_baseline": cpu,
        "clocks": clocks.summary(),
        "gpu_launches": launched,
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ configs 0, 2, 3
def zipf_vocabulary(seed=0):
    """Config 0 vocabulary: 4096 random lowercase words of 3-10 letters and
    their Zipf(s=1.1) rank weights."""
    rng = np.random.default_rng(seed)
    lengths = rng.integers(3, 11, 4096)
    letters = rng.integers(97, 123, (4096, 10), dtype=np.uint8)
    weights = np.arange(1, 4097, dtype=np.float64) ** -1.1
    return letters, lengths, weights / weights.sum(), rng


def zipf_text(size, seed=0):
    """Config 0 corpus: Zipf words joined by single spaces, '\n' with p = 1/12."""
    letters, lengths, p, rng = zipf_vocabulary(seed)
    n = size // 6 + 64
    while True:
        idx = rng.choice(4096, n, p=p)
        word_len = lengths[idx]
        starts = np.concatenate(([0], np.cumsum(word_len + 1)[:-1]))
        buf = np.empty(int(starts[-1] + word_len[-1] + 1), dtype=np.uint8)
        for j in range(10):
            m = word_len > j
            buf[starts[m] + j] = letters[idx[m], j]
        buf[starts + word_len] = np.where(rng.random(n) < 1 / 12, 10, 32).astype(np.uint8)
        if buf.size >= size:
            return buf[:size].tobytes()
        n *= 2


def config2_files(count=4096, seed=2):
    """Config 2: log-uniform sizes on 256 B-256 KiB (1% empty); 50% slices of
    the config-0 corpus, 25% uniform random bytes, 25% runs (geometric mean
    length 64, values 0-15)."""
    rng = np.random.default_rng(seed)
    sizes = np.exp(rng.uniform(np.log(256), np.log(262144), count)).astype(np.int64)
    sizes[rng.choice(count, count // 100, replace=False)] = 0
    kinds = rng.choice(3, count, p=[0.5, 0.25, 0.25])
    corpus = np.frombuffer(zipf_text(16 * MIB, 0), dtype=np.uint8)
    files = []
    for n, kind in zip(sizes.tolist(), kinds.tolist()):
        if kind == 0:
            start = int(rng.integers(0, corpus.size - n + 1))
            data = corpus[start:start + n]
        elif kind == 1:
            data = rng.integers(0, 256, n, dtype=np.uint8)
        else:
            runs = rng.geometric(1 / 64, n // 32 + 64)
            while runs.sum() < n:
                runs = np.concatenate((runs, rng.geometric(1 / 64, n // 32 + 64)))
            data = np.repeat(rng.integers(0, 16, runs.size, dtype=np.uint8), runs)[:n]
        files.append(data.tobytes())
    return files


def config3_records(size=1 << 30, seed=3):
    """Config 3: 64-byte records (i32 id, i32 timestamp += U{1..10}, 4 x i16
    U[-100, 100], a 20-byte config-0 word, zero padded, 28 zero bytes)."""
    n = size // 64
    rng = np.random.default_rng(seed)
    rec = np.zeros(n, dtype=[("id", "<i4"), ("ts", "<i4"), ("f", "<i2", (4,)),
                             ("word", "S20"), ("pad", "V28")])
    rec["id"] = np.arange(n, dtype=np.int32)
    rec["ts"] = np.cumsum(rng.integers(1, 11, n), dtype=np.int64).astype(np.int32)
    rec["f"] = rng.integers(-100, 101, (n, 4), dtype=np.int16)
    letters, lengths, p, _ = zipf_vocabulary(0)
    vocab = np.array([letters[i, :lengths[i]].tobytes() for i in range(4096)], dtype="S20")
    rec["word"] = vocab[rng.choice(4096, n, p=p)]
    return rec.view(np.uint8)


def _parallel_map(fn, items, threads):
    from concurrent.futures import ThreadPoolExecutor
    with ThreadPoolExecutor(max_workers=threads) as pool:
        return list(pool.map(fn, items))


# ------------------------------------------------------------------ sharded workloads
BATCH_METRIC = ("decompress & compress GB/s (uncompressed bytes; config-2 batch of 4096 "
                "files: zlib L6 batch decode + chunk-32768 batch compress)")
RECORDS_METRIC = ("compress GB/s (uncompressed bytes; config-3 1 GiB record stream, "
                  "chunk-32768 ranges)")


def batch_inputs():
    files = config2_files()
    streams = _parallel_map(lambda f: zlib_stream(f, 6), files, os.cpu_count() or 1)
    return files, streams


def cpu_batch(files, streams, threads):
    """Oracle port over a file sample: serial-route decode and compress per file."""
    from oracle import oracle

    def one(k):
        out, status = oracle.inflate_serial(streams[k], len(files[k]))
        assert status == 0 and out == files[k]
        oracle.compress(files[k], CHUNK)

    start = time.perf_counter()
    _parallel_map(one, range(len(files)), threads)
    return time.perf_counter() - start


def cpu_records(sample, threads):
    """Oracle port: chunk-parallel compress of a record sample at 32 KiB."""
    from oracle import oracle
    import ctypes
    lib = oracle.lib()
    chunks = -(-len(sample) // CHUNK)
    slot = (CHUNK * 9 + 7) // 8 + 16
    slots = np.zeros(chunks * slot, dtype=np.uint8)
    sizes = np.zeros(chunks, dtype=np.uint32)
    src = np.frombuffer(sample, dtype=np.uint8)
    per = -(-chunks // threads)

    def encode(first):
        count = min(per, chunks - first)
        lib.oracle_compress_chunks(
            src.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)), len(sample), CHUNK, first, count,
            slots[first * slot:].ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)), slot,
            sizes[first:].ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)))

    start = time.perf_counter()
    _parallel_map(encode, range(0, chunks, per), threads)
    return time.perf_counter() - start


def run_reference_sharded(args, rank, world):
    if rank != 0:
        return
    from oracle import oracle
    oracle.build()
    threads = os.cpu_count() or 1
    if args.workload == "batch":
        files, streams = batch_inputs()
        k = 512
        files, streams = files[:k], streams[:k]
        unit_bytes = 2 * sum(len(f) for f in files)
        run = lambda: cpu_batch(files, streams, threads)
        metric, sample = BATCH_METRIC, ("first 512 of the 4096 config-2 files: serial-route "
                                        "decode + compress per file, oracle port, one file "
                                        "per thread")
    else:
        data = config3_records(64 * MIB)
        unit_bytes = data.size
        run = lambda: cpu_records(data.tobytes(), threads)
        metric, sample = RECORDS_METRIC, ("64 MiB of config-3 records, chunk-parallel "
                                          "compress at 32 KiB, oracle port")
    for _ in range(args.warmup):
        run()
    seconds = sum(run() for _ in range(args.steps)) / args.steps
    value = unit_bytes / seconds / 1e9
    print(json.dumps({
        "impl": "reference", "metric": metric, "value": round(value, 4), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(seconds * 1e3, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "u8", "data": "synthetic",
        "config": {"workload": args.workload},
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": threads,
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0}}), flush=True)


def _timed_steps(torch, args, step, stream, flush, device, world):
    """K steps bracketed by barrier + synchronize; returns (seconds, clocks)."""
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler(device.index) as clocks:
        for k in range(args.steps):
            flush.fill_(k & 255)
            starts[k].record(stream)
            step()
            ends[k].record(stream)
        torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    return sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / 1e3, clocks


def _max_over_ranks(torch, value, device, world):
    if world > 1:
        t = torch.tensor([value], dtype=torch.float64, device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        value = float(t.item())
    return value


def _kernel_times(lib, names):
    import ctypes
    kernels = {}
    for name in names:
        total, launches = ctypes.c_double(), ctypes.c_uint64()
        lib.cuda_zlib_b200_profile_read(name.encode(), ctypes.byref(total), ctypes.byref(launches))
        if launches.value:
            kernels[name] = (total.value, launches.value)
    return kernels


def run_gpu_sharded(args, rank, world):
    import ctypes
    import torch
    import cuda_zlib as codec
    from cuda_zlib import _native, sharding

    torch.cuda.set_device(rank % torch.cuda.device_count())
    device = torch.device("cuda", torch.cuda.current_device())
    codec.compile_kernels(device)
    stream = torch.cuda.current_stream(device)
    flush = torch.empty(256 * MIB, dtype=torch.uint8, device=device)
    lib = _native.library()
    lib.cuda_zlib_b200_profile.argtypes = [ctypes.c_int]
    lib.cuda_zlib_b200_profile_read.argtypes = [ctypes.c_char_p, ctypes.POINTER(ctypes.c_double),
                                                ctypes.POINTER(ctypes.c_uint64)]
    lib.cuda_zlib_b200_launches.restype = ctypes.c_uint64

    if args.workload == "batch":
        files, streams = batch_inputs()
        total_units = 2 * sum(len(f) for f in files)
        mine = sharding.rank_files([len(f) + len(s) for f, s in zip(files, streams)], rank, world)
        my_files = [files[i] for i in mine] or [b""]
        my_streams = [streams[i] for i in mine] or [zlib_stream(b"", 6)]
        sizes = [len(f) for f in my_files]
        in_sizes = [len(s) for s in my_streams]
        packed_raw = b"".join(my_files)
        packed_z = b"".join(my_streams)
        raw_dev = torch.frombuffer(bytearray(packed_raw + b"\0"), dtype=torch.uint8)[:len(packed_raw)].to(device)
        z_dev = torch.frombuffer(bytearray(packed_z), dtype=torch.uint8).to(device)

        def step(raw_in=raw_dev, z_in=z_dev):
            out, meta = codec.decompress_zlib_batch_checked(z_in, in_sizes, sizes, device)
            slots, emeta = codec.compress_zlib_batch_padded(raw_in, sizes, device,
                                                            chunk_bytes=CHUNK)
            return out, meta, slots, emeta

        def verify(result):
            out, meta, slots, emeta = result
            assert not meta.cpu().numpy().any()
            assert out.cpu().numpy().tobytes() == packed_raw
            emeta = emeta.cpu().numpy()
            assert not emeta[:, 1].any()
            host = slots.cpu().numpy().tobytes()
            offset = 0
            for f, (length, _) in zip(my_files, emeta):
                assert zlib.decompress(host[offset:offset + int(length)]) == f
                offset += len(f) + 5 * max(1, -(-len(f) // CHUNK)) + 6
            return float(emeta[:, 0].sum()) / max(1, sum(sizes))

        h2d = len(packed_raw) + len(packed_z)
        d2h = sum(sizes) + sum(len(f) + 5 * max(1, -(-len(f) // CHUNK)) + 6 for f in my_files)
        raw_pin = torch.frombuffer(bytearray(packed_raw + b"\0"), dtype=torch.uint8)[:len(packed_raw)].pin_memory()
        z_pin = torch.frombuffer(bytearray(packed_z), dtype=torch.uint8).pin_memory()

        # End to end, pipelined: the compressed files go in first and decode
        # while the raw files go in; the decoded files go out while the raw
        # files compress.
        copy_in, compute, copy_out = (torch.cuda.Stream(device) for _ in range(3))
        host_out = torch.empty(sum(sizes), dtype=torch.uint8).pin_memory()
        host_slots = torch.empty(d2h - sum(sizes), dtype=torch.uint8).pin_memory()
        host_meta = torch.empty(2 * len(sizes), dtype=torch.int32).pin_memory()
        host_emeta = torch.empty(2 * len(sizes), dtype=torch.int32).pin_memory()

        def e2e_step():
            with torch.cuda.stream(copy_in):
                z_in = z_pin.to(device, non_blocking=True)
                z_ready = torch.cuda.Event()
                z_ready.record(copy_in)
                raw_in = raw_pin.to(device, non_blocking=True)
                raw_ready = torch.cuda.Event()
                raw_ready.record(copy_in)
            with torch.cuda.stream(compute):
                compute.wait_event(z_ready)
                out, meta = codec.decompress_zlib_batch_checked(z_in, in_sizes, sizes, device)
                decoded = torch.cuda.Event()
                decoded.record(compute)
                compute.wait_event(raw_ready)
                slots, emeta = codec.compress_zlib_batch_padded(raw_in, sizes, device,
                                                                chunk_bytes=CHUNK)
                encoded = torch.cuda.Event()
                encoded.record(compute)
            with torch.cuda.stream(copy_out):
                copy_out.wait_event(decoded)
                host_out.copy_(out, non_blocking=True)
                host_meta.copy_(meta.view(torch.int32).flatten(), non_blocking=True)
                copy_out.wait_event(encoded)
                host_slots.copy_(slots, non_blocking=True)
                host_emeta.copy_(emeta.view(torch.int32).flatten(), non_blocking=True)
                copy_out.synchronize()
            assert not host_meta.numpy().any() and not host_emeta.numpy()[1::2].any()

        algorithmic = {"serial_inflate_kernel": len(packed_z) + sum(sizes),
                       "encode_chunks_kernel": sum(sizes)}
        names = ("serial_inflate_kernel", "encode_chunks_kernel", "encode_pack_kernel")
        metric = BATCH_METRIC
        config = {"workload": "config2: 4096 files (seed 2), log-uniform 256 B-256 KiB, 1% empty; "
                              "50% Zipf text, 25% random, 25% runs; zlib L6 decode + compress "
                              "at chunk_bytes=32768",
                  "files": len(files), "uncompressed_bytes_per_step": total_units,
                  "parallelism": "files LPT-sharded over %d GPU(s)" % world,
                  "l2": "flushed between steps (256 MiB write)"}
    else:
        data = config3_records()
        total_units = data.size
        max_range = ((1 << 28) - 6) * CHUNK // (CHUNK + 5)
        ranges = sharding.rank_ranges(data.size, CHUNK, rank, world, max_range)
        lo, hi = ranges[0][0], ranges[-1][1]
        last_rank = max(r for r in range(world)
                        if sharding.rank_ranges(data.size, CHUNK, r, world, max_range))
        mine = torch.from_numpy(data[lo:hi])
        src_dev = mine.to(device)
        outs, metas = [], []
        for start, stop in ranges:
            n = stop - start
            cap = n + 5 * max(1, -(-n // CHUNK)) + 6
            outs.append(torch.empty(cap, dtype=torch.uint8, device=device))
            metas.append(torch.zeros(3, dtype=torch.uint32, device=device))

        def step(src=src_dev):
            for k, (start, stop) in enumerate(ranges):
                last = rank == last_rank and k == len(ranges) - 1
                piece = src[start - lo:stop - lo]
                if piece.device.type == "cpu":
                    piece = piece.to(device)
                _native.check(lib.cuda_zlib_compress_range(
                    piece.data_ptr(), stop - start, CHUNK, int(last), outs[k].data_ptr(),
                    outs[k].numel(), metas[k].data_ptr(), stream.cuda_stream), "range")
            return outs, metas

        def verify(result):
            total = 0
            for (start, stop), out, meta in zip(ranges, *result):
                length, status, adler = (int(v) for v in meta.cpu())
                assert status == 0 and adler == zlib.adler32(data[start:stop])
                body = out[:length].cpu().numpy().tobytes()
                d = zlib.decompressobj(-15)
                assert d.decompress(body) == data[start:stop].tobytes()
                total += length
            return total / max(1, hi - lo)

        src_pin = mine.pin_memory()
        # End to end, pipelined over pieces of at most 32 MiB (whole chunks):
        # a piece goes in on a copy stream, compresses on a compute stream once
        # it is in, and its body goes out at its exact length as soon as its
        # metadata says how long it is, while later pieces copy and compress.
        piece_bytes = 1024 * CHUNK
        pieces = [(a, min(a + piece_bytes, stop)) for start, stop in ranges
                  for a in range(start, stop, piece_bytes)] or [(lo, hi)]
        piece_out = [torch.empty(b - a + 5 * max(1, -(-(b - a) // CHUNK)) + 6, dtype=torch.uint8,
                                 device=device) for a, b in pieces]
        piece_meta = [torch.zeros(3, dtype=torch.uint32, device=device) for _ in pieces]
        host_meta = torch.empty(3 * len(pieces), dtype=torch.int32).pin_memory()
        host_body = torch.empty(sum(o.numel() for o in piece_out), dtype=torch.uint8).pin_memory()
        copy_in, compute, copy_out, body_out = (torch.cuda.Stream(device) for _ in range(4))
        h2d = hi - lo
        d2h_done = [0]

        def e2e_step():
            done = []
            for k, (a, b) in enumerate(pieces):
                with torch.cuda.stream(copy_in):
                    piece = src_pin[a - lo:b - lo].to(device, non_blocking=True)
                    ready = torch.cuda.Event()
                    ready.record(copy_in)
                with torch.cuda.stream(compute):
                    compute.wait_event(ready)
                    last = rank == last_rank and b == hi
                    _native.check(lib.cuda_zlib_compress_range(
                        piece.data_ptr(), b - a, CHUNK, int(last), piece_out[k].data_ptr(),
                        piece_out[k].numel(), piece_meta[k].data_ptr(), compute.cuda_stream),
                        "range")
                    finished = torch.cuda.Event()
                    finished.record(compute)
                with torch.cuda.stream(copy_out):
                    copy_out.wait_event(finished)
                    host_meta[3 * k:3 * k + 3].copy_(piece_meta[k].view(torch.int32),
                                                     non_blocking=True)
                    done.append((piece, torch.cuda.Event()))
                    done[-1][1].record(copy_out)
            # Bodies go out on their own stream, each once its piece's
            # metadata (hence the piece) is done, not behind later pieces.
            at = 0
            with torch.cuda.stream(body_out):
                for k, (piece, meta_in) in enumerate(done):
                    meta_in.synchronize()
                    length, status = int(host_meta[3 * k]), int(host_meta[3 * k + 1])
                    assert status == 0
                    host_body[at:at + length].copy_(piece_out[k][:length], non_blocking=True)
                    at += length
                body_out.synchronize()
            d2h_done[0] = at + 12 * len(pieces)

        algorithmic = {"encode_chunks_kernel": hi - lo}
        names = ("encode_chunks_kernel", "encode_pack_kernel")
        metric = RECORDS_METRIC
        config = {"workload": "config3: 1 GiB of 64-byte records (seed 3), compressed as "
                              "chunk-aligned ranges at chunk_bytes=32768 (the 262144 chunk of "
                              "the config is outside the reference's [256, 65535] bound)",
                  "uncompressed_bytes_per_step": total_units,
                  "parallelism": "chunk ranges over %d GPU(s)" % world,
                  "l2": "inputs larger than L2; also flushed between steps"}

    for _ in range(args.warmup):
        result = step()
    torch.cuda.synchronize()
    ratio = verify(result)
    lib.cuda_zlib_b200_profile(1)
    launches_before = lib.cuda_zlib_b200_launches()
    seconds, clocks = _timed_steps(torch, args, step, stream, flush, device, world)
    launched = lib.cuda_zlib_b200_launches() - launches_before
    kernels = _kernel_times(lib, names)
    lib.cuda_zlib_b200_profile(0)
    seconds = _max_over_ranks(torch, seconds, device, world)
    per_step = seconds / args.steps
    value = total_units / per_step / 1e9

    e2e_times = []
    for k in range(max(args.warmup, 1) + args.steps):
        flush.fill_(k & 255)
        torch.cuda.synchronize()
        start = time.perf_counter()
        e2e_step()
        torch.cuda.synchronize()
        if k >= max(args.warmup, 1):
            e2e_times.append(time.perf_counter() - start)
    e2e_seconds = _max_over_ranks(torch, sum(e2e_times) / len(e2e_times), device, world)
    if args.workload != "batch":
        d2h = d2h_done[0]
    roofline = None
    if kernels:
        name, (total_ms, launches) = max(kernels.items(), key=lambda kv: kv[1][0])
        per_launch = algorithmic.get(name, 0) / max(1, launches // args.steps)
        achieved = per_launch / (total_ms / launches / 1e3) / 1e9
        peak, peak_kind = measured_peak()
        roofline = {"bound": "hbm", "kernel": name, "achieved": round(achieved, 2),
                    "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                    "frac": round(achieved / peak, 5), "traffic": committed_traffic(name),
                    "algorithmic_bytes_per_launch": int(per_launch),
                    "launch_ms": round(total_ms / launches, 4)}
    if rank != 0:
        return
    cpu = None
    if world == 1 and not args.no_cpu:
        threads = os.cpu_count() or 1
        if args.workload == "batch":
            k = 512
            t = cpu_batch(files[:k], streams[:k], threads)
            cpu = {"value": round(2 * sum(len(f) for f in files[:k]) / t / 1e9, 4),
                   "sample": "first 512 config-2 files, decode + compress per file"}
        else:
            sample = data[:64 * MIB].tobytes()
            t = cpu_records(sample, threads)
            cpu = {"value": round(len(sample) / t / 1e9, 4),
                   "sample": "64 MiB of config-3 records, chunk-parallel compress"}
        cpu.update(unit="GB/s", cores=threads, kind="port")
    config["compression_ratio_rank0"] = round(ratio, 5)
    print(json.dumps({
        "metric": metric, "value": round(value, 4), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per_step * 1e3, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "u8",
        "data": "synthetic", "config": config, "roofline": roofline,
        "kernels_ms_per_step": {k: round(v[0] / args.steps, 3) for k, v in kernels.items()},
        "e2e": {"value": round(total_units / e2e_seconds / 1e9, 4), "unit": "GB/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "timer": "host wall clock"},
        "cpu_baseline": cpu, "clocks": clocks.summary(), "gpu_launches": launched}), flush=True)


def main():
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=5)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", choices=["ours", "reference"], default="ours")
    parser.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    parser.add_argument("--no-e2e", action="store_true", help="skip the host-buffer leg")
    parser.add_argument("--workload", choices=["config1", "batch", "records"], default="config1",
                        help="config1 (default; replicas at N>1), batch (config 2, files "
                             "LPT-sharded over ranks) or records (config 3, chunk ranges "
                             "sharded over ranks)")
    parser.add_argument("--size-mib", type=int, default=64,
                        help="leading MiB of the config-1 array (64 = the full workload; "
                             "smaller sizes are for profiler captures)")
    args = parser.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.impl == "reference":
        if args.workload == "config1":
            run_reference(args, rank, world)
        else:
            run_reference_sharded(args, rank, world)
        return
    if world > 1:
        import datetime
        import torch
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    try:
        if args.workload == "config1":
            run_gpu(args, rank, world)
        else:
            run_gpu_sharded(args, rank, world)
    finally:
        if world > 1:
            import torch
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()

"""Seeded synthetic inputs of the five BASELINE configurations.

Shared by bench.py and the tests, so that the parity tests decode and encode
exactly the data the benchmark times.  No public dataset is involved: every
generator restates the configuration's description (sizes, seeds, value
distributions) with numpy's default_rng.

  config 0  16 MiB of Zipf(1.1) text over a 4096-word vocabulary (seed 0)
  config 1  64 MiB float32 random walk plus a 60-per-4096 sine (seed 1)
  config 2  4096 files, log-uniform 256 B - 256 KiB, 1% empty; 50% text
            slices, 25% uniform random bytes, 25% byte runs (seed 2)
  config 3  1 GiB of 64-byte records (seed 3)
  config 4a 65,536 files of exactly 64 KiB with the config-2 content mix
  config 4b three 256 MiB streams: zeros, uniform random bytes, and
            period-32768 repeats of a random 32 KiB block (seed 4)

CPU-zlib streams of these inputs are made with several host threads
(zlib releases the GIL while it compresses).
"""
import os
import zlib
from concurrent.futures import ThreadPoolExecutor

import numpy as np

MIB = 1 << 20


# ------------------------------------------------------------------ config 0
def zipf_vocabulary(seed=0):
    """4096 random lowercase words of 3-10 letters and their Zipf(s=1.1)
    rank probabilities (k^-1.1 over k = 1..4096)."""
    rng = np.random.default_rng(seed)
    lengths = rng.integers(3, 11, 4096)
    letters = rng.integers(97, 123, (4096, 10), dtype=np.uint8)
    weights = np.arange(1, 4097, dtype=np.float64) ** -1.1
    return letters, lengths, weights / weights.sum(), rng


def zipf_text(size=16 * MIB, seed=0):
    """Config 0: Zipf words joined by single spaces, '\\n' with p = 1/12."""
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


_CORPUS = {}


def corpus():
    """The config-0 text as a uint8 array (cached; config 2 and 4a slice it)."""
    if "text" not in _CORPUS:
        _CORPUS["text"] = np.frombuffer(zipf_text(16 * MIB, 0), dtype=np.uint8)
    return _CORPUS["text"]


# ------------------------------------------------------------------ config 1
def config1_float32(samples=16777216, seed=1):
    """Config 1: float32 LE x[i] = x[i-1] + N(0, 1e-3) + 1e-2 sin(2 pi 60 i / 4096)."""
    rng = np.random.default_rng(seed)
    walk = np.cumsum(rng.normal(0.0, 1e-3, samples))
    i = np.arange(samples, dtype=np.float64)
    x = walk + 1e-2 * np.sin(2 * np.pi * 60 * i / 4096)
    return x.astype("<f4").tobytes()


# ------------------------------------------------------------------ configs 2, 4a
def _runs(rng, n):
    """n bytes of runs: geometric lengths with mean 64, values 0-15."""
    runs = rng.geometric(1 / 64, n // 32 + 64)
    while runs.sum() < n:
        runs = np.concatenate((runs, rng.geometric(1 / 64, n // 32 + 64)))
    return np.repeat(rng.integers(0, 16, runs.size, dtype=np.uint8), runs)[:n]


def config2_files(count=4096, seed=2):
    """Config 2: log-uniform sizes on 256 B-256 KiB (1% empty); 50% slices of
    the config-0 corpus, 25% uniform random bytes, 25% runs."""
    rng = np.random.default_rng(seed)
    sizes = np.exp(rng.uniform(np.log(256), np.log(262144), count)).astype(np.int64)
    sizes[rng.choice(count, count // 100, replace=False)] = 0
    kinds = rng.choice(3, count, p=[0.5, 0.25, 0.25])
    text = corpus()
    files = []
    for n, kind in zip(sizes.tolist(), kinds.tolist()):
        if kind == 0:
            start = int(rng.integers(0, text.size - n + 1))
            data = text[start:start + n]
        elif kind == 1:
            data = rng.integers(0, 256, n, dtype=np.uint8)
        else:
            data = _runs(rng, n)
        files.append(data.tobytes())
    return files


KIND_NAMES = ("text", "random", "runs")


def config4a_kinds(count=65536, seed=4):
    """Content kind (0 text, 1 random, 2 runs) and text offset of every
    config-4a file, drawn once from the seed."""
    rng = np.random.default_rng(seed)
    kinds = rng.choice(3, count, p=[0.5, 0.25, 0.25])
    offsets = rng.integers(0, corpus().size - 65536 + 1, count)
    return kinds, offsets


def config4a_files(indices=None, count=65536, size=65536, seed=4):
    """Config 4a: files of exactly `size` bytes with the config-2 mix.

    Every file is a function of (seed, index) alone, so a rank can make just
    its own files.  Returns (packed uint8 array of len(indices) * size bytes,
    kinds of those files)."""
    kinds, offsets = config4a_kinds(count, seed)
    indices = range(count) if indices is None else indices
    indices = list(indices)
    packed = np.empty(len(indices) * size, dtype=np.uint8)
    text = corpus()

    def make(first):
        for k in range(first, min(first + 256, len(indices))):
            i = indices[k]
            dst = packed[k * size:(k + 1) * size]
            if kinds[i] == 0:
                dst[:] = text[offsets[i]:offsets[i] + size]
            else:
                rng = np.random.default_rng([seed, int(i)])
                dst[:] = rng.integers(0, 256, size, dtype=np.uint8) if kinds[i] == 1 else \
                    _runs(rng, size)

    parallel_map(make, range(0, len(indices), 256))
    return packed, kinds[indices]


# ------------------------------------------------------------------ config 3
def config3_records(size=1 << 30, seed=3):
    """Config 3: 64-byte records: i32 sequential id, i32 timestamp += U{1..10},
    four i16 from U[-100, 100], a 20-byte config-0 word (Zipf, zero padded)
    and 28 zero bytes (the description's fields total 36 bytes)."""
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


# ------------------------------------------------------------------ config 4b
def config4b_streams(size=256 * MIB, seed=4):
    """Config 4b: {'zeros', 'random', 'period'} -> uint8 arrays of `size`."""
    rng = np.random.default_rng(seed)
    block = rng.integers(0, 256, 32768, dtype=np.uint8)
    return {"zeros": np.zeros(size, dtype=np.uint8),
            "random": rng.integers(0, 256, size, dtype=np.uint8),
            "period": np.tile(block, -(-size // 32768))[:size]}


# ------------------------------------------------------------------ CPU zlib
def zlib_stream(raw, level=6, strategy=zlib.Z_DEFAULT_STRATEGY):
    """One RFC 1950 stream of `raw` made by the host's zlib."""
    c = zlib.compressobj(level, zlib.DEFLATED, zlib.MAX_WBITS, 8, strategy)
    return c.compress(raw) + c.flush()


def parallel_map(fn, items, threads=None):
    with ThreadPoolExecutor(max_workers=threads or os.cpu_count() or 1) as pool:
        return list(pool.map(fn, items))


def zlib_files(packed, size, level=6, threads=None):
    """zlib streams of the equal-size files packed in `packed`."""
    count = len(packed) // size if size else 0
    return parallel_map(lambda k: zlib_stream(packed[k * size:(k + 1) * size].tobytes(), level),
                        range(count), threads)

"""Multi-GPU sharding host logic, on CPU.

* plan_files (LPT over files) and plan_ranges (chunk-aligned ranges of one
  stream) partition their work exactly and evenly;
* Adler-32 combination and the header/body/trailer splice reproduce the
  one-device stream: the per-chunk bodies come from the CPU oracle's chunk
  encoder, so splicing ranges must give oracle.compress of the whole input;
* with world_size 2 over gloo, every rank derives its share on its own and
  the shares, gathered, cover every item once.
"""
import os
import random
import socket
import zlib

import numpy as np
import pytest
import torch.multiprocessing as mp

from cuda_zlib import sharding
from oracle import oracle


# ---------------------------------------------------------------- planners
@pytest.mark.parametrize("parts", [1, 2, 3, 8])
def test_plan_files_is_a_balanced_partition(parts):
    rng = random.Random(parts)
    weights = [int(rng.lognormvariate(10, 2)) for _ in range(500)] + [0] * 5
    plan = sharding.plan_files(weights, parts)
    assert len(plan) == parts
    flat = sorted(i for b in plan for i in b)
    assert flat == list(range(len(weights)))
    assert all(b == sorted(b) for b in plan)
    loads = [sum(weights[i] for i in b) for b in plan]
    # LPT: the heaviest bin exceeds the lightest by at most one item.
    assert max(loads) - min(loads) <= max(weights)
    assert plan == sharding.plan_files(weights, parts)


def test_plan_files_edge_cases():
    assert sharding.plan_files([], 3) == [[], [], []]
    assert sharding.plan_files([7], 4) == [[0], [], [], []]
    assert sharding.plan_files([5, 5, 5, 5], 2) == [[0, 2], [1, 3]]
    for bad in (0, -1, 1.5, True):
        with pytest.raises(ValueError):
            sharding.plan_files([1], bad)
    with pytest.raises(ValueError):
        sharding.plan_files([-1], 2)


@pytest.mark.parametrize("size, chunk, parts, max_range", [
    (0, 256, 1, None), (0, 32768, 4, None), (1, 256, 3, None), (100000, 32768, 3, None),
    (10 * 32768, 32768, 2, 3 * 32768), (12345678, 65535, 8, None),
    (3 << 28, 32768, 2, (1 << 28) - 8192), (999, 256, 8, 600),
])
def test_plan_ranges_tile_the_stream(size, chunk, parts, max_range):
    plan = sharding.plan_ranges(size, chunk, parts, max_range)
    assert len(plan) == parts
    flat = [r for ranges in plan for r in ranges]
    assert flat[0][0] == 0 and flat[-1][1] == size
    for (a, b), (c, _) in zip(flat, flat[1:]):
        assert b == c and b % chunk == 0
    for a, b in flat:
        assert a % chunk == 0 and (b > a or size == 0)
        if max_range is not None:
            assert b - a <= max(chunk, max_range)
    chunks = [sum(-(-(b - a) // chunk) for a, b in ranges) for ranges in plan]
    if size:
        assert max(chunks) - min(chunks) <= 1


# ---------------------------------------------------------------- splicing
def test_adler32_combine_matches_zlib():
    rng = random.Random(1)
    for _ in range(200):
        a = rng.randbytes(rng.choice([0, 1, 100, 70000]))
        b = rng.randbytes(rng.choice([0, 1, 5, 65521, 200000]))
        assert sharding.adler32_combine(zlib.adler32(a), zlib.adler32(b), len(b)) == \
            zlib.adler32(a + b)
    parts = [rng.randbytes(rng.randint(0, 5000)) for _ in range(20)]
    assert sharding.combine_adlers([zlib.adler32(p) for p in parts],
                                   [len(p) for p in parts]) == zlib.adler32(b"".join(parts))


def _oracle_chunk_bodies(raw, chunk):
    """Per-chunk raw Deflate bodies of the one-stream encoding, from the oracle."""
    import ctypes
    lib = oracle.lib()
    chunks = max(1, -(-len(raw) // chunk))
    slot = (chunk * 9 + 7) // 8 + 16
    slots = np.zeros(chunks * slot, dtype=np.uint8)
    sizes = np.zeros(chunks, dtype=np.uint32)
    src = np.frombuffer(raw + b"\0", dtype=np.uint8)
    lib.oracle_compress_chunks(src.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)), len(raw),
                               chunk, 0, chunks,
                               slots.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)), slot,
                               sizes.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)))
    return [slots[k * slot:k * slot + int(sizes[k])].tobytes() for k in range(chunks)]


@pytest.mark.parametrize("size, chunk, parts", [(0, 4096, 2), (5000, 256, 3),
                                                (300000, 32768, 4), (131072, 32768, 8)])
def test_spliced_ranges_equal_the_one_device_stream(size, chunk, parts):
    rng = random.Random(size)
    raw = bytes(rng.choices(range(20), k=size // 2)) + rng.randbytes(size - size // 2)
    bodies = _oracle_chunk_bodies(raw, chunk)
    pieces, adlers, lengths = [], [], []
    for ranges in sharding.plan_ranges(size, chunk, parts):
        for start, stop in ranges:
            first, count = start // chunk, max(1, -(-(stop - start) // chunk))
            pieces.append(b"".join(bodies[first:first + count]))
            adlers.append(zlib.adler32(raw[start:stop]))
            lengths.append(stop - start)
    stream = (sharding.splice_header() + b"".join(pieces) +
              sharding.splice_trailer(sharding.combine_adlers(adlers, lengths)))
    assert stream == oracle.compress(raw, chunk)
    assert zlib.decompress(stream) == raw


# ---------------------------------------------------------------- gloo ranks
def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, weights, size, chunk, results):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        files = sharding.rank_files(weights, rank, world)
        ranges = sharding.rank_ranges(size, chunk, rank, world)
        load = sum(weights[i] for i in files)
        gathered = [None] * world
        dist.all_gather_object(gathered, (files, ranges, load))
        if rank == 0:
            results.put(gathered)
    finally:
        dist.destroy_process_group()


def test_ranks_derive_disjoint_covering_shares_over_gloo():
    world = 2
    rng = random.Random(4)
    weights = [rng.randint(0, 1 << 18) for _ in range(4096)]
    size, chunk = 64 << 20, 32768
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main,
                         args=(r, world, port, weights, size, chunk, results))
             for r in range(world)]
    for p in procs:
        p.start()
    gathered = results.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    files = sorted(i for f, _, _ in gathered for i in f)
    assert files == list(range(len(weights)))
    loads = [load for _, _, load in gathered]
    assert max(loads) - min(loads) <= max(weights)
    ranges = [r for _, rs, _ in gathered for r in rs]
    assert ranges[0][0] == 0 and ranges[-1][1] == size
    assert all(b == c for (_, b), (c, _) in zip(ranges, ranges[1:]))
    assert gathered[0][0] == sharding.plan_files(weights, world)[0]

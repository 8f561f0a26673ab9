"""Host-side checks of the benchmark harness (no GPU).

The clock sampler passes nvidia-smi the GPU that a CUDA device index maps to:
nvidia-smi numbers GPUs physically and ignores CUDA_VISIBLE_DEVICES, so on a
box that exposes a subset of its GPUs the CUDA index alone names another GPU.
"""
import importlib.util
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_harness", os.path.join(ROOT, "bench.py"))
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


@pytest.mark.parametrize("visible, index, expected", [
    (None, 0, "0"), (None, 3, "3"),
    ("4,6", 0, "4"), ("4,6", 1, "6"), (" 5 , 7 ", 1, "7"),
    ("GPU-1111,GPU-2222", 1, "GPU-2222"),
    ("2", 1, "1"),  # index beyond the list: left as given
])
def test_clock_sampler_queries_the_mapped_gpu(bench, monkeypatch, visible, index, expected):
    if visible is None:
        monkeypatch.delenv("CUDA_VISIBLE_DEVICES", raising=False)
    else:
        monkeypatch.setenv("CUDA_VISIBLE_DEVICES", visible)
    assert bench.ClockSampler(index).index == expected

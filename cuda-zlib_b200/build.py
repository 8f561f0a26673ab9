"""Build the codec's CUDA library for sm_100a (B200) in-tree.

    python cuda-zlib_b200/build.py            # incremental
    python cuda-zlib_b200/build.py --force    # rebuild everything

Output: cuda-zlib_b200/cuda_zlib/libcuda_zlib_b200.so, with the CUDA runtime
linked statically so it shares the driver's primary context with PyTorch (or
any other runtime) without depending on a particular libcudart version.
Objects go to cuda-zlib_b200/_build/.  Also builds
cuda-zlib_b200/cuda_zlib/libcuda_zlib_xla.so, the four XLA FFI handlers over
that C ABI (ffi/cuda_zlib_xla.cc), against jaxlib's FFI header when jax is
installed and against the stand-in header in ffi/standin otherwise.
"""
import concurrent.futures
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIBRARY = os.path.join(HERE, "cuda_zlib", "libcuda_zlib_b200.so")
FFI = os.path.join(HERE, "ffi")
XLA_LIBRARY = os.path.join(HERE, "cuda_zlib", "libcuda_zlib_xla.so")
SOURCES = ["codec.cu", "deflate.cu", "inflate_serial.cu", "inflate_general.cu", "crc32.cu",
           "inflate_parallel.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
         "--expt-relaxed-constexpr"]


def _nvcc():
    for candidate in (os.environ.get("CUDACXX"), shutil.which("nvcc"),
                      os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")):
        if candidate and os.path.exists(candidate):
            return candidate
    raise RuntimeError("nvcc not found; set CUDACXX or CUDA_HOME")


def _headers():
    paths = [os.path.join(CSRC, name) for name in os.listdir(CSRC)
             if name.endswith((".h", ".cuh"))]
    paths.append(os.path.join(os.path.dirname(HERE), "include", "cuda_zlib_b200.h"))
    return paths


def _stale(target, inputs):
    if not os.path.exists(target):
        return True
    stamp = os.path.getmtime(target)
    return any(os.path.getmtime(path) > stamp for path in inputs)


def build(force=False, verbose=False):
    """Compile every source that changed and link the library; return its path."""
    nvcc = _nvcc()
    os.makedirs(BUILD, exist_ok=True)
    headers = _headers()
    jobs = []
    objects = []
    for name in SOURCES:
        source = os.path.join(CSRC, name)
        obj = os.path.join(BUILD, name.replace(".cu", ".o"))
        objects.append(obj)
        if force or _stale(obj, [source] + headers):
            jobs.append([nvcc, *ARCH, *FLAGS, "-c", source, "-o", obj])

    def run(command):
        result = subprocess.run(command, capture_output=True, text=True)
        if result.returncode:
            raise RuntimeError("nvcc failed:\n" + " ".join(command) + "\n" + result.stderr)
        if verbose and result.stderr:
            print(result.stderr, file=sys.stderr)

    with concurrent.futures.ThreadPoolExecutor(max_workers=len(SOURCES)) as pool:
        list(pool.map(run, jobs))
    if force or jobs or _stale(LIBRARY, objects):
        run([nvcc, *ARCH, "-shared", "-cudart", "static", "-o", LIBRARY, *objects,
             "-Xlinker", "--no-undefined", "-lrt", "-ldl", "-lpthread"])
    build_xla(force)
    return LIBRARY


def xla_include():
    """(include dir of xla/ffi/api/ffi.h, "jaxlib" | "stand-in")."""
    try:
        import jax.ffi
        return jax.ffi.include_dir(), "jaxlib"
    except Exception:  # jax is not installed: the stand-in declarations
        return os.path.join(FFI, "standin"), "stand-in"


def build_xla(force=False):
    """The XLA FFI handler library (ffi/cuda_zlib_xla.cc) over the C ABI."""
    include, _ = xla_include()
    source = os.path.join(FFI, "cuda_zlib_xla.cc")
    headers = [os.path.join(include, "xla", "ffi", "api", "ffi.h"),
               os.path.join(os.path.dirname(HERE), "include", "cuda_zlib_b200.h"), LIBRARY]
    if not force and not _stale(XLA_LIBRARY, [source] + [h for h in headers if os.path.exists(h)]):
        return XLA_LIBRARY
    cuda = os.path.dirname(os.path.dirname(_nvcc()))
    command = [os.environ.get("CXX", "g++"), "-std=c++17", "-O2", "-fPIC", "-shared", "-Wall",
               "-I" + include, "-I" + os.path.join(os.path.dirname(HERE), "include"),
               "-I" + os.path.join(cuda, "include"), source, "-o", XLA_LIBRARY,
               "-L" + os.path.dirname(LIBRARY), "-l:" + os.path.basename(LIBRARY),
               "-Wl,-rpath,$ORIGIN", "-Wl,--no-undefined"]
    result = subprocess.run(command, capture_output=True, text=True)
    if result.returncode:
        raise RuntimeError("XLA FFI handler build failed:\n" + " ".join(command) + "\n" +
                           result.stderr)
    return XLA_LIBRARY


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))

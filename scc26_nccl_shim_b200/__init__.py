"""B200-native NCCL interposer: Python side.

The product is the native library ``lib/libnccl_b200.so`` (an LD_PRELOAD
NCCL interposer with sm_100a kernels). This package locates and loads it,
binds the CUDA-free core library ``lib/libnb_core.so`` for CPU tests, and
provides the NCCL-ABI client, data generators, clock sampling and the
formal-model checkers used by the tests and the benchmark.

Subpackages:
  ops/       ctypes bindings to the kernels (single-GPU virtual-rank runs)
  parallel/  the NCCL C ABI client (comm init, grouped collectives)
  utils/     seeded data, clock sampling, timing helpers
  models/    explicit-state checkers of the GroupFallback / HostLaneReuse models
"""
import os

ROOT = os.path.dirname(os.path.abspath(__file__))
LIB_DIR = os.path.join(ROOT, "lib")
LIB_PATH = os.path.join(LIB_DIR, "libnccl_b200.so")
CORE_PATH = os.path.join(LIB_DIR, "libnb_core.so")
REPO = os.path.dirname(ROOT)


class NativeLibraryMissing(RuntimeError):
    """Raised when a native library was not built (run `make` at the repo root)."""


def require(path: str) -> str:
    if not os.path.exists(path):
        raise NativeLibraryMissing(f"{path} is missing: build it with `make -C {REPO}`")
    return path


def real_nccl_path() -> str:
    """The libnccl.so.2 that torch ships (the one the interposer forwards to)."""
    try:
        import nvidia.nccl  # type: ignore
        for base in nvidia.nccl.__path__:
            cand = os.path.join(base, "lib", "libnccl.so.2")
            if os.path.exists(cand):
                return cand
    except ImportError:
        pass
    return "libnccl.so.2"

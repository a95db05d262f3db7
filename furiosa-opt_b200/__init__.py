"""furiosa-opt B200 execution backend: the CPU emulator's value-op hot path (BufStorage) as sm_100a
CUDA kernels behind furiosa-opt-std's Backend seam. See include/fopt_b200.h for the C ABI."""
from . import _lib, dist, dtypes, ops, workloads  # noqa: F401
from .backend import B200, Graph, Mapping, SafeTensors, Storage, m  # noqa: F401

__all__ = ["B200", "Mapping", "SafeTensors", "Storage", "m", "ops", "dtypes"]

"""chelis_b200 -- B200-native (sm_100a) CUDA backend for the Chelis tensor-DAG
hot path: matmul dispatch, fused elementwise / reduction groups and their
adjoints, exposed as the C ABI of include/chelis_cuda.h (libchelis_cuda.so).

`chelis_b200.lib` is the ctypes binding of that ABI; `chelis_b200.ops` calls
it on torch-owned device memory; `chelis_b200.workloads` generates the seeded
synthetic inputs of the benchmark configurations.
"""
from . import lib  # noqa: F401

__all__ = ["lib"]

"""ctypes binding of libchelis_cuda.so (the C ABI declared in
include/chelis_cuda.h).

There is no fallback: if the shared library is missing or cannot be loaded
the import raises, and every entry point that returns a non-zero status
raises ChelisCudaError with the library's message.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libchelis_cuda.so")

c_i64 = ctypes.c_int64
c_u64 = ctypes.c_uint64
c_i32 = ctypes.c_int32
c_int = ctypes.c_int
c_f32 = ctypes.c_float
c_vp = ctypes.c_void_p


class GpuTensor(ctypes.Structure):
    """chelis_gpu_tensor (crates/chelis-backend-hip/runtime/chelis_device_descriptor.h:8-18)."""
    _fields_ = [
        ("data", c_vp),
        ("shape", ctypes.POINTER(c_i64)),
        ("strides", ctypes.POINTER(c_i64)),
        ("count", c_i64),
        ("byte_capacity", c_i64),
        ("rank", c_i32),
        ("dtype", ctypes.c_uint8),
        ("ownership", ctypes.c_uint8),
        ("reserved", ctypes.c_uint8 * 2),
    ]


class BlockParams(ctypes.Structure):
    """chelis_block_params (include/chelis_cuda.h)."""
    _fields_ = [(n, c_i64) for n in ("batch", "seq", "d_model", "heads", "d_ff")] + [
        ("eps", c_f32)] + [(n, c_vp) for n in (
            "x", "dy", "w_qkv", "w_o", "w_1", "w_2", "ln1_gamma", "ln1_beta", "ln2_gamma",
            "ln2_beta", "y", "dx", "dw_qkv", "dw_o", "dw_1", "dw_2", "dln1_gamma", "dln1_beta",
            "dln2_gamma", "dln2_beta")]


DTYPE_F32, DTYPE_F64, DTYPE_I32, DTYPE_BOOL, DTYPE_I64 = 0, 1, 2, 3, 4
DTYPE_BF16, DTYPE_F16 = 5, 6
GEMM_3XTF32, GEMM_EXACT_TREE = 0, 1
DGEMM_AUTO, DGEMM_DMMA, DGEMM_FFMA = 0, 1, 2
ROWS_EXACT, ROWS_FAST = 0, 1
STATUS_NAMES = {0: "OK", 1: "DOMAIN", 2: "OVERFLOW", 3: "CUDA", 4: "UNSUPPORTED", 5: "TIMEOUT",
                6: "NO_DEVICE", 7: "FAIL"}


class ChelisCudaError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


class Scalar(ctypes.Structure):
    """chelis_scalar (crates/chelis-runtime/include/chelis_runtime.h:26)."""
    _fields_ = [("dtype", ctypes.c_uint8), ("reserved", ctypes.c_uint8 * 7), ("bits", c_u64)]


class HostView(ctypes.Structure):
    """chelis_read_view / chelis_write_view (chelis_runtime_views.h:7-18)."""
    _fields_ = [("data", c_vp), ("count", c_i64), ("dtype", ctypes.c_uint8),
                ("reserved", ctypes.c_uint8 * 7)]


def tagged_i64(v: int) -> Scalar:
    """A canonical tagged i64 scalar (the metadata plan's argument form)."""
    s = Scalar()
    s.dtype = DTYPE_I64
    s.bits = v & 0xFFFFFFFFFFFFFFFF
    return s


def exemplar(dtype: int) -> Scalar:
    s = Scalar()
    s.dtype = dtype
    return s


_P = ctypes.POINTER(GpuTensor)
_PP = ctypes.POINTER(c_vp)
_SP = ctypes.POINTER(Scalar)

# name -> (restype, argtypes); every int-returning entry is a status code.
SIGNATURES = {
    "chelis_cuda_version": (c_int, []),
    "chelis_cuda_last_error": (ctypes.c_char_p, []),
    "chelis_cuda_init": (c_int, [c_i32]),
    "chelis_cuda_set_stream": (c_int, [c_vp]),
    "chelis_cuda_get_stream": (c_vp, []),
    "chelis_cuda_synchronize": (c_int, []),
    "chelis_cuda_device_status": (c_int, []),
    "chelis_cuda_launch_count": (c_u64, []),
    "chelis_cuda_set_wait_limit": (c_int, [ctypes.c_uint32]),
    "chelis_cuda_get_wait_limit": (ctypes.c_uint32, []),
    "chelis_cuda_selftest_bounded_wait": (c_int, [c_int]),
    "chelis_cuda_set_gemm_mode": (c_int, [c_int]),
    "chelis_cuda_get_gemm_mode": (c_int, []),
    "chelis_cuda_set_rows_mode": (c_int, [c_int]),
    "chelis_cuda_get_rows_mode": (c_int, []),
    "chelis_device_tensor_alloc_shape": (c_vp, [ctypes.c_uint8, c_i32, ctypes.POINTER(c_i64)]),
    "chelis_device_tensor_borrow_shape": (c_vp, [ctypes.c_uint8, c_i32, ctypes.POINTER(c_i64), c_vp, c_i64]),
    "chelis_device_tensor_import": (c_vp, [_P]),
    "chelis_device_tensor_view": (_P, [c_vp]),
    "chelis_device_tensor_device": (c_i32, [c_vp]),
    "chelis_device_tensor_clone": (c_vp, [c_vp]),
    "chelis_device_tensor_release": (None, [c_vp]),
    "chelis_device_tensor_copy_from_host_bytes": (c_int, [c_vp, c_vp, c_i64]),
    "chelis_device_tensor_copy_to_host_bytes": (c_int, [c_vp, c_i64, c_vp]),
    "chelis_cuda_sgemm_row_major": (c_int, [_P, _P, _P, c_i64, c_i64, c_i64]),
    "chelis_cuda_dgemm_row_major": (c_int, [_P, _P, _P, c_i64, c_i64, c_i64]),
    "chelis_cuda_sgemm_batched_row_major": (c_int, [_P, _P, _P, c_i64, c_i64, c_i64, c_i64]),
    "chelis_cuda_sgemm_strided_batched_row_major": (c_int, [_P, _P, _P, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64]),
    "chelis_cuda_dgemm_batched_row_major": (c_int, [_P, _P, _P, c_i64, c_i64, c_i64, c_i64]),
    "chelis_cuda_dgemm_strided_batched_row_major": (c_int, [_P, _P, _P, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64]),
    "chelis_cuda_sgemm": (c_int, [c_int, c_int, c_i64, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_i64, c_i64, c_i64]),
    "chelis_cuda_dgemm": (c_int, [c_int, c_int, c_i64, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_i64, c_i64, c_i64]),
    "chelis_cuda_set_gemm_pairs": (c_int, [c_int]),
    "chelis_cuda_get_gemm_pairs": (c_int, []),
    "chelis_cuda_attention_causal_fwd": (c_int, [c_i64, c_i64, c_i64, c_f32, c_vp, c_vp, c_vp, c_vp, c_vp]),
    "chelis_cuda_attention_causal_bwd": (c_int, [c_i64, c_i64, c_i64, c_f32] + [c_vp] * 9),
    "chelis_cuda_sgemm_host": (c_int, [c_int, c_int, c_i64, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_i64, c_i64, c_i64]),
    "chelis_cuda_dgemm_host": (c_int, [c_int, c_int, c_i64, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_i64, c_i64, c_i64]),
    "chelis_cuda_tf32x3_split": (c_int, [c_int, c_int, c_i64, c_i64, c_vp, c_i64, c_i64, c_i64, c_vp, c_vp]),
    "chelis_cuda_sgemm_tf32x3_presplit": (c_int, [c_i64, c_i64, c_i64, c_i64, c_int, c_vp, c_vp, c_int, c_vp, c_vp, c_vp, c_i64, c_i64]),
    "chelis_cuda_row_sum_f32": (c_int, [c_vp, c_i64, c_i64, c_vp]),
    "chelis_cuda_col_sum_f32": (c_int, [c_vp, c_i64, c_i64, c_vp]),
    "chelis_cuda_row_max_f32": (c_int, [c_vp, c_i64, c_i64, c_vp]),
    "chelis_cuda_count_bool": (c_int, [c_vp, c_i64, c_vp]),
    "chelis_cuda_dropout_f32": (c_int, [c_vp, c_vp, c_i64, c_u64, c_f32, c_i64]),
    "chelis_cuda_dropout_mask": (c_int, [c_vp, c_i64, c_u64, c_f32, c_i64]),
    "chelis_cuda_layer_norm_f32": (c_int, [c_vp, c_vp, c_vp, c_f32, c_vp, c_i64, c_i64]),
    "chelis_cuda_softmax_rows_f32": (c_int, [c_vp, c_vp, c_i64, c_i64]),
    "chelis_cuda_softmax_rows_bwd_f32": (c_int, [c_vp, c_vp, c_vp, c_i64, c_i64]),
    "chelis_cuda_chain_fwd": (c_int, [c_vp, c_vp, c_vp, c_f32, c_u64, c_f32, c_i64, c_i64, c_i64, c_vp, c_vp]),
    "chelis_cuda_chain_bwd": (c_int, [c_vp, c_vp, c_vp, c_f32, c_u64, c_f32, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp, c_vp]),
    "chelis_cuda_chain_saved_bytes": (c_i64, [c_i64, c_i64]),
    "chelis_cuda_chain_fwd_save": (c_int, [c_vp, c_vp, c_vp, c_f32, c_u64, c_f32, c_i64, c_i64, c_i64, c_vp, c_vp]),
    "chelis_cuda_chain_bwd_saved": (c_int, [c_vp, c_vp, c_vp, c_f32, c_f32, c_i64, c_i64, c_vp, c_vp, c_vp, c_vp]),
    "chelis_cuda_chain_bwd_noalloc":(c_int, [c_vp, c_vp, c_vp, c_f32, c_u64, c_f32, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp, c_vp]),
    "chelis_cuda_cumsum_f64": (c_int, [c_vp, c_vp, c_i64, c_i64, c_int]),
    "chelis_cuda_cumsum_f32": (c_int, [c_vp, c_vp, c_i64, c_i64, c_int]),
    "chelis_cuda_portfolio_f64": (c_int, [c_vp, c_vp, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp]),
    "chelis_cuda_mlp_step": (c_int, [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp, c_vp, c_vp, c_vp]),
    "chelis_cuda_block_workspace_bytes": (c_i64, [ctypes.POINTER(BlockParams)]),
    "chelis_cuda_block_step": (c_int, [ctypes.POINTER(BlockParams), c_vp]),
    "chelis_cuda_block_step_dp": (c_int, [ctypes.POINTER(BlockParams), c_vp]),
    "chelis_cuda_block_timing": (c_int, [c_int]),
    "chelis_cuda_block_phase_ms": (c_int, [ctypes.POINTER(c_f32), c_i32]),
    "chelis_cuda_block_phase_name": (ctypes.c_char_p, [c_i32]),
    "chelis_cuda_fused_elementwise": (c_int, [c_i32, c_vp, c_i32, _PP, ctypes.POINTER(c_i64), c_i32, ctypes.POINTER(c_i64), c_i32, c_vp]),
    "chelis_cuda_set_fused_jit": (c_int, [c_int]),
    "chelis_cuda_get_fused_jit": (c_int, []),
    "chelis_cuda_fused_jit_launches": (c_i64, []),
    "chelis_cuda_fused_reduce": (c_int, [c_i32, c_vp, c_i32, _PP, ctypes.POINTER(c_i64), c_i32, ctypes.POINTER(c_i64), c_i32, c_i32, c_i32, c_vp]),
    "chelis_cuda_relu": (c_int, [c_i32, c_vp, c_vp, c_i64]),
    "chelis_cuda_relu_adjoint": (c_int, [c_i32, c_vp, c_vp, c_vp, c_i64]),
    "chelis_cuda_gelu_f32": (c_int, [c_vp, c_vp, c_i64]),
    "chelis_cuda_gelu_adjoint_f32": (c_int, [c_vp, c_vp, c_vp, c_i64]),
    "chelis_cuda_layer_norm_bwd_f32": (c_int, [c_vp, c_vp, c_f32, c_vp, c_i64, c_i64, c_vp, c_vp, c_vp]),
    "chelis_cuda_cross_entropy_f32": (c_int, [c_vp, c_vp, c_i64, c_i64, c_vp, c_vp]),
    "chelis_cuda_dp_shard": (c_int, [c_i64, c_i32, c_i32, ctypes.POINTER(c_i64), ctypes.POINTER(c_i64)]),
    "chelis_cuda_dp_unique_id": (c_int, [c_vp]),
    "chelis_cuda_dp_init": (c_int, [c_i32, c_i32, c_vp]),
    "chelis_cuda_dp_allreduce_sum": (c_int, [c_i32, c_vp, c_i64]),
    "chelis_cuda_dp_world": (c_int, [ctypes.POINTER(c_i32), ctypes.POINTER(c_i32)]),
    "chelis_cuda_dp_finalize": (c_int, [c_i32]),
    "chelis_chain_fwd_device": (c_int, [_PP, c_i32, _PP, c_i32]),
    "chelis_chain_grad_device": (c_int, [_PP, c_i32, _PP, c_i32]),
    "chelis_portfolio_device": (c_int, [_PP, c_i32, _PP, c_i32]),
    "chelis_matmul_device": (c_int, [_PP, c_i32, _PP, c_i32]),
    # modes, per-call GEMM, shutdown
    "chelis_cuda_set_dgemm_kernel": (c_int, [c_int]),
    "chelis_cuda_get_dgemm_kernel": (c_int, []),
    "chelis_cuda_set_thread_modes": (c_int, [c_int, c_int, c_int]),
    "chelis_cuda_get_thread_modes": (c_int, [ctypes.POINTER(c_int)] * 3),
    "chelis_cuda_dgemm_kernel_for": (c_int, [c_int, c_int, c_i64, c_i64, c_i64, c_i64]),
    "chelis_cuda_shutdown": (c_int, []),
    "chelis_cuda_sgemm_ex": (c_int, [c_int, c_int, c_int, c_i64, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_i64, c_i64, c_i64]),
    "chelis_cuda_dgemm_ex": (c_int, [c_int, c_int, c_int, c_int, c_i64, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_i64, c_i64, c_i64]),
    # host runtime subset (include/chelis_host_runtime.h)
    "chelis_scalar_from_bits": (Scalar, [ctypes.c_uint8, c_u64]),
    "chelis_dtype_size": (c_i64, [ctypes.c_uint8]),
    "chelis_metadata_plan_new": (c_vp, [Scalar, _SP, Scalar]),
    "chelis_metadata_plan_view": (c_vp, [Scalar, _SP, _SP, Scalar, Scalar]),
    "chelis_metadata_plan_rank": (c_i32, [c_vp]),
    "chelis_metadata_plan_shape": (ctypes.POINTER(c_i64), [c_vp]),
    "chelis_metadata_plan_strides": (ctypes.POINTER(c_i64), [c_vp]),
    "chelis_metadata_plan_count": (c_i64, [c_vp]),
    "chelis_metadata_plan_byte_count": (c_i64, [c_vp]),
    "chelis_metadata_plan_byte_offset": (c_i64, [c_vp, Scalar]),
    "chelis_metadata_plan_dtype": (ctypes.c_uint8, [c_vp]),
    "chelis_metadata_plan_check_capacity": (None, [c_vp, Scalar]),
    "chelis_metadata_plan_release": (None, [c_vp]),
    "chelis_alloc": (c_vp, [c_i32, ctypes.POINTER(c_i64), ctypes.c_uint8]),
    "chelis_tensor_entry_borrow": (c_vp, [c_i32, ctypes.POINTER(c_i64), ctypes.c_uint8, c_vp, c_i64]),
    "chelis_tensor_retain": (None, [c_vp]),
    "chelis_tensor_release": (None, [c_vp]),
    "chelis_tensor_read_view": (HostView, [c_vp]),
    "chelis_tensor_begin_write": (c_vp, [c_vp]),
    "chelis_tensor_write_view": (HostView, [c_vp]),
    "chelis_tensor_end_write": (None, [c_vp]),
    "chelis_tensor_rank": (c_i32, [c_vp]),
    "chelis_tensor_shape": (c_i64, [c_vp, c_i32]),
    "chelis_tensor_numel": (c_i64, [c_vp]),
    "chelis_tensor_byte_count": (c_i64, [c_vp]),
    # device owner under the reference's names, and the host-array entries
    "chelis_device_tensor_alloc": (c_vp, [c_vp]),
    "chelis_device_tensor_borrow": (c_vp, [c_vp, c_vp, Scalar]),
    "chelis_device_tensor_copy_from_host": (None, [c_vp, c_vp]),
    "chelis_device_tensor_copy_to_host": (None, [c_vp, c_vp]),
    "chelis_device_tensor_alloc_status": (c_int, [c_vp, _PP]),
    "chelis_device_tensor_borrow_status": (c_int, [c_vp, c_vp, Scalar, _PP]),
    "chelis_device_tensor_copy_from_host_status": (c_int, [c_vp, c_vp]),
    "chelis_device_tensor_copy_to_host_status": (c_int, [c_vp, c_vp]),
    "chelis_chain_fwd": (None, [_PP, c_int, _PP, c_int]),
    "chelis_chain_grad": (None, [_PP, c_int, _PP, c_int]),
    "chelis_portfolio": (None, [_PP, c_int, _PP, c_int]),
    "chelis_matmul": (None, [_PP, c_int, _PP, c_int]),
    "chelis_chain_fwd_status": (c_int, [_PP, c_int, _PP, c_int]),
    "chelis_chain_grad_status": (c_int, [_PP, c_int, _PP, c_int]),
    "chelis_portfolio_status": (c_int, [_PP, c_int, _PP, c_int]),
    "chelis_matmul_status": (c_int, [_PP, c_int, _PP, c_int]),
    "chelis_cuda_bf16_gemm_f32_acc_row_major": (c_int, [_P, _P, _P, c_i64, c_i64, c_i64]),
    "chelis_cuda_f16_gemm_f32_acc_row_major": (c_int, [_P, _P, _P, c_i64, c_i64, c_i64]),
    "chelis_cuda_gemm16": (c_int, [c_i32, c_int, c_int, c_i64, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_i64, c_i64, c_i64]),
    "chelis_cuda_crmath_f32": (c_int, [c_i32, c_vp, c_vp, c_i64]),
    "chelis_cuda_crmath_sweep_f32": (c_int, [c_i32, ctypes.c_uint32, c_i64, c_vp]),
    # DAG executor (include/chelis_dag.h)
    "chelis_dag_from_json": (c_int, [ctypes.c_char_p, c_i64, ctypes.POINTER(c_vp)]),
    "chelis_dag_release": (None, [c_vp]),
    "chelis_dag_input_count": (c_i32, [c_vp]),
    "chelis_dag_input_label": (ctypes.c_char_p, [c_vp, c_i32]),
    "chelis_dag_output_count": (c_i32, [c_vp]),
    "chelis_dag_output_label": (ctypes.c_char_p, [c_vp, c_i32]),
    "chelis_dag_arena_bytes": (c_i64, [c_vp]),
    "chelis_dag_live_peak_bytes": (c_i64, [c_vp]),
    "chelis_dag_slot_count": (c_i32, [c_vp]),
    "chelis_dag_output_bytes": (c_i64, [c_vp]),
    "chelis_dag_symbol_count": (c_i32, [c_vp]),
    "chelis_dag_symbol_name": (ctypes.c_char_p, [c_vp, c_i32]),
    "chelis_dag_bind": (c_int, [c_vp, ctypes.POINTER(c_i64), c_i32, ctypes.POINTER(c_vp)]),
    "chelis_dag_run_device": (c_int, [c_vp, _PP, c_i32, _PP, c_i32]),
    "chelis_dag_run_device_arena": (c_int, [c_vp, _PP, c_i32, _PP, c_i32, c_vp, c_i64]),
    "chelis_dag_run": (c_int, [c_vp, _PP, c_int, _PP, c_int]),
}

_lib = None


def load() -> ctypes.CDLL:
    """Load (and on first use declare) libchelis_cuda.so.  Raises if absent."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: run `python -m chelis_b200.build` (nvcc, sm_100a); "
                "there is no CPU fallback")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    msg = load().chelis_cuda_last_error()
    return msg.decode() if msg else ""


def check(status: int) -> None:
    if status != 0:
        raise ChelisCudaError(status, last_error())


def call(name: str, *args) -> None:
    """Call a status-returning entry point and raise on failure."""
    check(getattr(load(), name)(*args))

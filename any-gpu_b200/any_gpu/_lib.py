"""ctypes binding of libagpu.so (declared in include/agpu.h).

The library is loaded from this package directory only; there is no other
implementation to fall back to.  If it is missing, importing raises.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libagpu.so"

c_dev = C.c_void_p
c_buf = C.c_void_p
c_status = C.c_int
P_buf = C.POINTER(C.c_void_p)
P_f32 = C.POINTER(C.c_float)
u32, u64, f32, i32 = C.c_uint32, C.c_uint64, C.c_float, C.c_int

# name -> (restype, argtypes).  Kept in the order of include/agpu.h.
SIGNATURES: dict[str, tuple] = {
    "agpu_last_error_message": (C.c_char_p, []),
    "agpu_status_string": (C.c_char_p, [c_status]),
    "agpu_device_create": (c_status, [i32, C.POINTER(c_dev)]),
    "agpu_device_destroy": (c_status, [c_dev]),
    "agpu_device_name": (c_status, [c_dev, C.c_char_p, C.c_size_t]),
    "agpu_device_sm_count": (c_status, [c_dev, C.POINTER(i32)]),
    "agpu_device_ordinal": (c_status, [c_dev, C.POINTER(i32)]),
    "agpu_device_stream": (C.c_void_p, [c_dev]),
    "agpu_synchronize": (c_status, [c_dev]),
    "agpu_set_precision": (c_status, [c_dev, i32]),
    "agpu_get_precision": (c_status, [c_dev, C.POINTER(i32)]),
    "agpu_set_thread_precision": (c_status, [i32]),
    "agpu_get_thread_precision": (i32, []),
    "agpu_device_launch_count": (u64, [c_dev]),
    "agpu_upload": (c_status, [c_dev, C.c_void_p, u64, P_buf]),
    "agpu_alloc": (c_status, [c_dev, u64, P_buf]),
    "agpu_read": (c_status, [c_dev, c_buf, C.c_void_p, u64]),
    "agpu_write": (c_status, [c_dev, c_buf, C.c_void_p, u64]),
    "agpu_write_async": (c_status, [c_dev, c_buf, u64, C.c_void_p, u64, C.c_void_p]),
    "agpu_read_async": (c_status, [c_dev, c_buf, u64, C.c_void_p, u64, C.c_void_p]),
    "agpu_buffer_free": (c_status, [c_buf]),
    "agpu_buffer_len": (u64, [c_buf]),
    "agpu_buffer_device_ptr": (C.c_void_p, [c_buf]),
    "agpu_matmul": (c_status, [c_dev, c_buf, c_buf, u32, u32, u32, P_buf]),
    "agpu_batch_matmul": (c_status, [c_dev, c_buf, c_buf, u32, u32, u32, u32, P_buf]),
    "agpu_batch_matmul_softmax": (c_status, [c_dev, c_buf, c_buf, u32, u32, u32, u32, P_buf]),
    "agpu_gemm": (c_status, [c_dev, c_buf, c_buf, u32, u32, u32, u32, i32, i32, P_buf]),
    "agpu_gemm_ex": (c_status, [c_dev, c_buf, c_buf, c_buf, c_buf, u32, u32, u32, u32, i32, i32,
                                i32, P_buf]),
    "agpu_softmax": (c_status, [c_dev, c_buf, u32, u32, P_buf]),
    "agpu_conv2d": (c_status, [c_dev, c_buf, c_buf, c_buf] + [u32] * 14 + [P_buf]),
    "agpu_conv2d_group_norm_swish": (c_status, [c_dev, c_buf, c_buf, c_buf] + [u32] * 14
                                     + [c_buf, c_buf, u32, f32, P_buf]),
    "agpu_conv_transpose2d": (c_status, [c_dev, c_buf, c_buf, c_buf] + [u32] * 16 + [P_buf]),
    "agpu_conv2d_grad_weight": (c_status, [c_dev, c_buf, c_buf] + [u32] * 16 + [P_buf]),
    "agpu_conv2d_grad_bias": (c_status, [c_dev, c_buf, u32, u32, u32, u32, P_buf]),
    "agpu_group_norm": (c_status, [c_dev, c_buf, c_buf, c_buf, u32, u32, u32, u32, f32,
                                   P_buf]),
    "agpu_group_norm_swish": (c_status, [c_dev, c_buf, c_buf, c_buf, u32, u32, u32, u32, f32,
                                         P_buf]),
    "agpu_group_norm_backward": (c_status, [c_dev, c_buf, c_buf, c_buf, u32, u32, u32, u32, f32,
                                            P_buf, P_buf, P_buf]),
    "agpu_scaled_dot_product_attention": (c_status, [c_dev, c_buf, c_buf, c_buf, u32, u32, u32,
                                                     P_buf]),
    "agpu_sdpa_causal": (c_status, [c_dev, c_buf, c_buf, c_buf, u32, u32, u32, P_buf]),
    "agpu_sdpa_backward": (c_status, [c_dev, c_buf, c_buf, c_buf, c_buf, u32, u32, u32, i32,
                                      P_buf, P_buf, P_buf]),
    "agpu_rmsnorm": (c_status, [c_dev, c_buf, c_buf, u32, u32, f32, P_buf]),
    "agpu_rope": (c_status, [c_dev, c_buf, u32, u32, u32, u32, f32, P_buf]),
    "agpu_swish_mul": (c_status, [c_dev, c_buf, c_buf, P_buf]),
    "agpu_add": (c_status, [c_dev, c_buf, c_buf, P_buf]),
    "agpu_sub": (c_status, [c_dev, c_buf, c_buf, P_buf]),
    "agpu_mul": (c_status, [c_dev, c_buf, c_buf, P_buf]),
    "agpu_relu": (c_status, [c_dev, c_buf, P_buf]),
    "agpu_sigmoid": (c_status, [c_dev, c_buf, P_buf]),
    "agpu_swish": (c_status, [c_dev, c_buf, P_buf]),
    "agpu_tanh_act": (c_status, [c_dev, c_buf, P_buf]),
    "agpu_scale": (c_status, [c_dev, c_buf, f32, P_buf]),
    "agpu_relu_backward": (c_status, [c_dev, c_buf, c_buf, P_buf]),
    "agpu_sigmoid_backward": (c_status, [c_dev, c_buf, c_buf, P_buf]),
    "agpu_swish_backward": (c_status, [c_dev, c_buf, c_buf, P_buf]),
    "agpu_tanh_backward": (c_status, [c_dev, c_buf, c_buf, P_buf]),
    "agpu_transpose": (c_status, [c_dev, c_buf, u32, u32, u32, u32, P_buf]),
    "agpu_add_per_col": (c_status, [c_dev, c_buf, c_buf, u32, u32, P_buf]),
    "agpu_add_broadcast": (c_status, [c_dev, c_buf, c_buf, u32, u32, P_buf]),
    "agpu_sum_inner": (c_status, [c_dev, c_buf, u32, u32, P_buf]),
    "agpu_sum_rows": (c_status, [c_dev, c_buf, u32, u32, P_buf]),
    "agpu_concat": (c_status, [c_dev, c_buf, c_buf, u32, u32, u32, P_buf]),
    "agpu_slice_per_block": (c_status, [c_dev, c_buf, u32, u32, u32, u32, P_buf]),
    "agpu_upsample_nearest2d": (c_status, [c_dev, c_buf, u32, u32, u32, u32, u32, u32, P_buf]),
    "agpu_upsample_nearest2d_backward": (c_status, [c_dev, c_buf, u32, u32, u32, u32, u32, u32,
                                                    P_buf]),
    "agpu_mse_loss": (c_status, [c_dev, c_buf, c_buf, P_buf]),
    "agpu_launch_batch_matmul": (c_status, [c_dev, C.c_void_p, C.c_void_p, C.c_void_p,
                                            u32, u32, u32, u32, C.c_void_p]),
    "agpu_launch_gemm": (c_status, [c_dev, C.c_void_p, C.c_void_p, C.c_void_p, u32, u32, u32,
                                    u32, i32, i32, C.c_void_p]),
    "agpu_launch_conv2d": (c_status, [c_dev] + [C.c_void_p] * 4 + [u32] * 14 + [C.c_void_p]),
    "agpu_launch_batch_matmul_softmax": (c_status, [c_dev] + [C.c_void_p] * 3 + [u32] * 4
                                         + [C.c_void_p]),
    "agpu_launch_conv2d_group_norm_swish": (c_status, [c_dev] + [C.c_void_p] * 4 + [u32] * 14
                                            + [C.c_void_p, C.c_void_p, u32, f32, C.c_void_p]),
    "agpu_launch_group_norm": (c_status, [c_dev, C.c_void_p, C.c_void_p, C.c_void_p,
                                          C.c_void_p, u32, u32, u32, u32, f32, i32,
                                          C.c_void_p]),
    "agpu_launch_group_norm_backward": (c_status, [c_dev] + [C.c_void_p] * 6 +
                                        [u32, u32, u32, u32, f32, C.c_void_p]),
    "agpu_adamw_step": (c_status, [c_dev] + [C.POINTER(C.c_void_p)] * 4 +
                        [u32, f32, f32, f32, f32, f32, u32]),
    "agpu_launch_adamw": (c_status, [c_dev, C.c_void_p, u32, f32, f32, f32, f32, f32, u32,
                                     C.c_void_p]),
    "agpu_launch_sdpa": (c_status, [c_dev] + [C.c_void_p] * 4 + [u32, u32, u32, i32,
                                                                 C.c_void_p]),
    "agpu_launch_sdpa_backward": (c_status, [c_dev] + [C.c_void_p] * 7 + [u32, u32, u32, i32,
                                                                      C.c_void_p]),
    "agpu_launch_gemm_ex": (c_status, [c_dev] + [C.c_void_p] * 3 + [u32] * 4 + [i32, i32]
                            + [C.c_void_p] * 2 + [i32, C.c_void_p]),
    "agpu_launch_sdpa_strided": (c_status, [c_dev] + [C.c_void_p] * 4 + [u32] * 4
                                 + [C.c_void_p] * 4 + [i32, C.c_void_p]),
    "agpu_launch_rmsnorm": (c_status, [c_dev] + [C.c_void_p] * 3 + [u64, u32, f32, C.c_void_p]),
    "agpu_launch_rope": (c_status, [c_dev, C.c_void_p, C.c_void_p, u32, u32, u32, u32, u64, f32,
                                    C.c_void_p]),
    "agpu_launch_swish_mul": (c_status, [c_dev] + [C.c_void_p] * 3 + [u64, u32, u64, u64, u64,
                                                                      C.c_void_p]),
    "agpu_launch_softmax": (c_status, [c_dev, C.c_void_p, C.c_void_p, u64, u32, C.c_void_p]),
    "agpu_group_norm_noalloc": (c_status, [C.c_void_p] * 4 + [u32, u32, u32, u32, f32, i32,
                                                              C.c_void_p]),
    "agpu_ipc_export": (c_status, [c_dev, C.c_void_p, C.c_void_p, C.POINTER(u64)]),
    "agpu_ipc_import": (c_status, [c_dev, C.c_void_p, C.POINTER(C.c_void_p)]),
    "agpu_ipc_close": (c_status, [c_dev, C.c_void_p]),
    "agpu_ipc_event_create": (c_status, [c_dev, C.POINTER(C.c_void_p), C.c_void_p]),
    "agpu_ipc_event_import": (c_status, [c_dev, C.c_void_p, C.POINTER(C.c_void_p)]),
    "agpu_event_destroy": (c_status, [c_dev, C.c_void_p]),
    "agpu_event_record": (c_status, [c_dev, C.c_void_p, C.c_void_p]),
    "agpu_stream_wait_event": (c_status, [c_dev, C.c_void_p, C.c_void_p]),
    "agpu_copy_async": (c_status, [c_dev, C.c_void_p, C.c_void_p, u64, C.c_void_p]),
    "agpu_signal_peers": (c_status, [c_dev, C.POINTER(C.c_void_p), u32, u32, C.c_void_p]),
    "agpu_wait_flags": (c_status, [c_dev, C.c_void_p, u32, u32, u32, C.c_void_p]),
    "agpu_selftest_wait_timeout": (c_status, [c_dev, u32, C.c_void_p]),
}

class AttnLayout(C.Structure):
    """agpu_attn_layout: element strides of one attention operand."""
    _fields_ = [("seq_stride", u64), ("head_stride", u64), ("batch_stride", u64)]


_LIB = None


def load() -> C.CDLL:
    """Load libagpu.so and attach signatures (raises if it was not built)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python any-gpu_b200/build.py` "
            "(there is no non-CUDA implementation of these ops)")
    lib = C.CDLL(os.fspath(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _LIB = lib
    return lib

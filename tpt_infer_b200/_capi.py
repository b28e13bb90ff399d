"""ctypes binding of ``libtpt_cuda.so`` (declarations: include/tpt_cuda.h).

The library is loaded from this package directory only. If it is missing the
import fails loudly: there is no CPU fallback anywhere in this package.
"""
from __future__ import annotations

import ctypes as C
import os

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libtpt_cuda.so")

if not os.path.exists(LIB_PATH):
    raise ImportError(
        f"{LIB_PATH} is not built; run `python tpt_infer_b200/build.py` (the CUDA backend has no CPU fallback)")

lib = C.CDLL(LIB_PATH)

vp = C.c_void_p
sz = C.c_size_t
f32p = C.POINTER(C.c_float)
i32p = C.POINTER(C.c_int32)
szp = C.POINTER(C.c_size_t)
ctxp = vp
wp = vp

# name -> (restype, argtypes); every symbol the header declares
SIGNATURES = {
    "tpt_cuda_ctx_create": (C.c_int, [C.c_int, vp, C.POINTER(vp)]),
    "tpt_cuda_ctx_destroy": (C.c_int, [ctxp]),
    "tpt_cuda_ctx_sync": (C.c_int, [ctxp]),
    "tpt_cuda_ctx_stream": (vp, [ctxp]),
    "tpt_cuda_ctx_device": (C.c_int, [ctxp]),
    "tpt_cuda_backend_name": (C.c_char_p, []),
    "tpt_cuda_status_str": (C.c_char_p, [C.c_int]),
    "tpt_cuda_last_error": (C.c_char_p, [ctxp]),
    "tpt_cuda_last_size_mismatch": (None, [ctxp, szp, szp]),
    "tpt_cuda_ctx_launch_count": (C.c_uint64, [ctxp]),
    "tpt_cuda_capture_begin": (C.c_int, [ctxp]),
    "tpt_cuda_capture_end": (C.c_int, [ctxp, C.POINTER(C.c_void_p)]),
    "tpt_cuda_graph_launch": (C.c_int, [ctxp, vp]),
    "tpt_cuda_graph_kernels": (C.c_uint64, [vp]),
    "tpt_cuda_graph_destroy": (C.c_int, [vp]),
    "tpt_cuda_matmul": (C.c_int, [ctxp, vp, sz, sz, sz, vp, sz, sz, sz, vp, sz]),
    "tpt_cuda_conv2d": (C.c_int, [ctxp, vp, sz, szp, vp, sz, szp, vp, sz, sz, sz, sz, sz]),
    "tpt_cuda_elementwise_add": (C.c_int, [ctxp, vp, sz, vp, sz, vp, sz]),
    "tpt_cuda_relu": (C.c_int, [ctxp, vp, sz, vp, sz]),
    "tpt_cuda_softmax": (C.c_int, [ctxp, vp, sz, vp, sz, sz]),
    "tpt_cuda_sigmoid": (C.c_int, [ctxp, vp, sz, vp, sz]),
    "tpt_cuda_gelu": (C.c_int, [ctxp, vp, sz, vp, sz]),
    "tpt_cuda_matmul_dev": (C.c_int, [ctxp, vp, sz, sz, vp, sz, vp]),
    "tpt_cuda_conv2d_dev": (C.c_int, [ctxp, vp, szp, vp, szp, vp, sz, sz, sz, sz]),
    "tpt_cuda_elementwise_add_dev": (C.c_int, [ctxp, vp, vp, vp, sz]),
    "tpt_cuda_relu_dev": (C.c_int, [ctxp, vp, vp, sz]),
    "tpt_cuda_softmax_dev": (C.c_int, [ctxp, vp, vp, sz, sz]),
    "tpt_cuda_sigmoid_dev": (C.c_int, [ctxp, vp, vp, sz]),
    "tpt_cuda_gelu_dev": (C.c_int, [ctxp, vp, vp, sz]),
    "tpt_cuda_quantize_i8_symmetric": (C.c_int, [ctxp, vp, sz, vp, f32p]),
    "tpt_cuda_quantize_i8_symmetric_per_channel": (C.c_int, [ctxp, vp, sz, sz, vp, vp]),
    "tpt_cuda_quantize_i8_asymmetric": (C.c_int, [ctxp, vp, sz, vp, f32p, i32p]),
    "tpt_cuda_pack_i4": (C.c_int, [ctxp, vp, sz, vp]),
    "tpt_cuda_unpack_i4": (C.c_int, [ctxp, vp, sz, sz, vp, szp]),
    "tpt_cuda_quantize_i4_symmetric": (C.c_int, [ctxp, vp, sz, vp, f32p]),
    "tpt_cuda_quantize_i4_symmetric_per_channel": (C.c_int, [ctxp, vp, sz, sz, vp, vp]),
    "tpt_cuda_dequantize_i8_symmetric": (C.c_int, [ctxp, vp, sz, C.c_float, vp]),
    "tpt_cuda_dequantize_i8_symmetric_per_channel": (C.c_int, [ctxp, vp, sz, vp, sz, vp]),
    "tpt_cuda_dequantize_i4_symmetric_per_channel": (C.c_int, [ctxp, vp, sz, sz, vp, sz, vp]),
    "tpt_cuda_dequantize_i8_asymmetric": (C.c_int, [ctxp, vp, sz, C.c_float, C.c_int32, vp]),
    "tpt_cuda_dequantize_i4_symmetric": (C.c_int, [ctxp, vp, sz, sz, C.c_float, vp, szp]),
    "tpt_cuda_quantized_matmul_i8": (C.c_int, [ctxp, vp, sz, sz, sz, C.c_float, vp, sz, sz, sz, vp, sz, vp, sz]),
    "tpt_cuda_quantize_i8_symmetric_dev": (C.c_int, [ctxp, vp, sz, vp, vp]),
    "tpt_cuda_quantize_i8_static_dev": (C.c_int, [ctxp, vp, sz, C.c_float, vp]),
    "tpt_cuda_weights_upload_i8": (C.c_int, [ctxp, vp, vp, sz, sz, C.POINTER(vp)]),
    "tpt_cuda_weights_upload_i4": (C.c_int, [ctxp, vp, sz, vp, sz, sz, C.POINTER(vp)]),
    "tpt_cuda_weights_free": (C.c_int, [wp]),
    "tpt_cuda_weights_shape": (C.c_int, [wp, szp, szp]),
    "tpt_cuda_w8a8_gemm": (C.c_int, [ctxp, vp, sz, sz, C.c_float, wp, vp, C.c_int, vp]),
    "tpt_cuda_w8a8_gemm_dev": (C.c_int, [ctxp, vp, sz, C.c_float, wp, vp, C.c_int, vp]),
    "tpt_cuda_w8a8_gemm_acc_dev": (C.c_int, [ctxp, vp, sz, wp, vp]),
    "tpt_cuda_w4_gemm": (C.c_int, [ctxp, vp, sz, sz, wp, vp, C.c_int, vp]),
    "tpt_cuda_w4_gemm_dev": (C.c_int, [ctxp, vp, sz, wp, vp, C.c_int, vp]),
    "tpt_cuda_quantize_i8_symmetric_noalloc": (C.c_int, [vp, sz, vp, vp, vp]),
    "tpt_cuda_plan_create": (C.c_int, [ctxp, C.POINTER(vp)]),
    "tpt_cuda_plan_destroy": (C.c_int, [vp]),
    "tpt_cuda_gemm": (C.c_int, [vp, vp, sz, sz, sz, C.c_int, vp, sz, sz, C.c_int, vp, sz, C.c_float, C.c_float,
                                vp, sz]),
    "tpt_cuda_gemm_dev": (C.c_int, [vp, vp, sz, sz, C.c_int, vp, sz, C.c_int, vp, sz, C.c_float, C.c_float, vp]),
    "tpt_cuda_plan_add_tensor": (C.c_int, [vp, C.c_int, sz, C.POINTER(C.c_int)]),
    "tpt_cuda_plan_add_const": (C.c_int, [vp, vp, sz, C.POINTER(C.c_int)]),
    "tpt_cuda_plan_add_op": (C.c_int, [vp, vp]),
    "tpt_cuda_plan_finalize": (C.c_int, [vp]),
    "tpt_cuda_plan_reuse_arena": (C.c_int, [vp, C.POINTER(C.c_int), sz]),
    "tpt_cuda_ctx_set_wait_limit": (C.c_int, [ctxp, C.c_uint32]),
    "tpt_cuda_selftest_bounded_wait": (C.c_int, [ctxp, C.POINTER(C.c_uint)]),
    "tpt_cuda_comm_set_timeout": (C.c_int, [C.c_double]),
    "tpt_cuda_plan_run_batches": (C.c_int, [vp, C.POINTER(C.c_int), C.POINTER(vp), sz, C.POINTER(C.c_int), C.POINTER(vp), sz, sz]),
    "tpt_cuda_plan_arena_bytes": (C.c_int, [vp, szp]),
    "tpt_cuda_plan_tensor_ptr": (C.c_int, [vp, C.c_int, C.POINTER(vp)]),
    "tpt_cuda_plan_set_calibration": (C.c_int, [vp, C.c_int]),
    "tpt_cuda_plan_freeze_scales": (C.c_int, [vp]),
    "tpt_cuda_plan_get_scales": (C.c_int, [vp, vp, sz, szp]),
    "tpt_cuda_plan_set_scales": (C.c_int, [vp, vp, sz]),
    "tpt_cuda_plan_run_device": (C.c_int, [vp]),
    "tpt_cuda_plan_set_graph": (C.c_int, [vp, C.c_int]),
    "tpt_cuda_plan_run": (C.c_int, [vp, vp, vp, sz, vp, vp, sz]),
    # multi-GPU
    "tpt_cuda_comm_unique_id": (C.c_int, [vp, sz]),
    "tpt_cuda_comm_create": (C.c_int, [vp, vp, sz, C.c_int, C.c_int, C.POINTER(vp)]),
    "tpt_cuda_comm_destroy": (C.c_int, [vp]),
    "tpt_cuda_comm_size": (C.c_int, [vp, C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    "tpt_cuda_all_gather_dev": (C.c_int, [vp, vp, vp, sz]),
    "tpt_cuda_plan_set_comm": (C.c_int, [vp, vp]),
}

COMM_ID_BYTES = 128


class PlanOp(C.Structure):
    """tpt_plan_op (include/tpt_cuda.h)."""

    _fields_ = [("kind", C.c_int), ("in0", C.c_int), ("in1", C.c_int), ("in2", C.c_int), ("out", C.c_int),
                ("w", C.c_void_p), ("act", C.c_int), ("f0", C.c_float), ("dims", C.c_size_t * 16)]

for _name, (_res, _args) in SIGNATURES.items():
    _fn = getattr(lib, _name)
    _fn.restype = _res
    _fn.argtypes = _args

"""ctypes front end of the CPU oracle (``oracle/tpt_oracle.c``).

TEST INFRASTRUCTURE ONLY. This module is the parity checker for the CUDA
backend and the timed CPU baseline. Only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline / reference legs import it; the CUDA product
path (``tpt_infer_b200``) never does and has no CPU fallback.

Each wrapper names the tpt-infer function it restates (paths relative to the
tpt-infer repository root); the C source carries the file:line citations.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))

SIZE_MISMATCH, SHAPE_MISMATCH, UNSUPPORTED, INVALID = 1, 2, 3, 4
ACT_NONE, ACT_RELU, ACT_GELU = 0, 1, 2


class OracleError(Exception):
    """Mirror of OpError (crates/tpt-infer-ops/src/backend.rs:6-20)."""

    def __init__(self, code, expected=None, actual=None):
        self.code = code
        self.expected = expected
        self.actual = actual
        super().__init__(f"oracle status {code} (expected={expected}, actual={actual})")


def _host_has_avx512() -> bool:
    try:
        with open("/proc/cpuinfo") as f:
            flags = f.read()
        return " avx512f" in flags and " avx512bw" in flags
    except OSError:
        return False


def build() -> None:
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def _load():
    name = "libtpt_oracle_v4.so" if _host_has_avx512() else "libtpt_oracle_v3.so"
    path = os.path.join(_HERE, name)
    if not os.path.exists(path):
        build()
    return C.CDLL(path)


_lib = _load()
ISA = "avx512" if _host_has_avx512() else "avx2"

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_sz = C.c_size_t
_szp = np.ctypeslib.ndpointer(np.uintp, flags="C_CONTIGUOUS")


def _sig(name, res, *args):
    fn = getattr(_lib, name)
    fn.restype = res
    fn.argtypes = list(args)
    return fn


_sig("tpto_last_size_mismatch", None, C.POINTER(_sz), C.POINTER(_sz))
_sig("tpto_lcg_sym", None, _f32p, _sz, C.c_uint32)
_sig("tpto_lcg_uniform", None, _f32p, _sz, C.c_uint32)
_sig("tpto_normal", None, _f32p, _sz, C.c_uint32, C.c_float, C.c_float)
_sig("tpto_matmul_naive", C.c_int, _f32p, _sz, _sz, _sz, _f32p, _sz, _sz, _sz, _f32p, _sz)
_sig("tpto_gemm", C.c_int, _f32p, _sz, _sz, _sz, C.c_int, _f32p, _sz, _sz, C.c_int, C.c_void_p, _sz, C.c_float,
     C.c_float, _f32p, _sz)
_sig("tpto_matmul_avx", C.c_int, _f32p, _sz, _sz, _sz, _f32p, _sz, _sz, _sz, _f32p, _sz, C.c_int)
_sig("tpto_conv2d", C.c_int, _f32p, _sz, _szp, _f32p, _sz, _szp, _f32p, _sz, _sz, _sz, _sz, _sz, C.c_int)
_sig("tpto_elementwise_add", C.c_int, _f32p, _sz, _f32p, _sz, _f32p, _sz)
for _n in ("tpto_relu", "tpto_sigmoid", "tpto_gelu"):
    _sig(_n, C.c_int, _f32p, _sz, _f32p, _sz)
_sig("tpto_softmax", C.c_int, _f32p, _sz, _f32p, _sz, _sz)
_sig("tpto_quantize_i8_symmetric", C.c_float, _f32p, _sz, _i8p)
_sig("tpto_quantize_i8_asymmetric", None, _f32p, _sz, _i8p, C.POINTER(C.c_float), C.POINTER(C.c_int32))
_sig("tpto_quantize_i8_symmetric_per_channel", C.c_int, _f32p, _sz, _sz, _i8p, _f32p)
_sig("tpto_pack_i4", C.c_int, _i8p, _sz, _u8p)
_sig("tpto_unpack_i4", _sz, _u8p, _sz, _sz, _i8p)
_sig("tpto_quantize_i4_symmetric", C.c_float, _f32p, _sz, _u8p)
_sig("tpto_quantize_i4_symmetric_per_channel", C.c_int, _f32p, _sz, _sz, _u8p, _f32p)
_sig("tpto_dequantize_i8_symmetric", None, _i8p, _sz, C.c_float, _f32p)
_sig("tpto_dequantize_i8_asymmetric", None, _i8p, _sz, C.c_float, C.c_int32, _f32p)
_sig("tpto_dequantize_i8_symmetric_per_channel", C.c_int, _i8p, _sz, _f32p, _sz, _f32p)
_sig("tpto_dequantize_i4_symmetric", None, _u8p, _sz, _sz, C.c_float, _f32p)
_sig("tpto_dequantize_i4_symmetric_per_channel", None, _u8p, _sz, _sz, _f32p, _sz, _f32p)
_sig("tpto_quantized_matmul_i8", C.c_int, _i8p, _sz, _sz, _sz, C.c_float, _i8p, _sz, _sz, _sz,
     _f32p, _sz, _f32p, _sz)
_sig("tpto_i8_gemm_acc", None, _i8p, _i8p, _sz, _sz, _sz, _i32p, C.c_int)
_sig("tpto_w8a8_gemm", None, _i8p, _i8p, _sz, _sz, _sz, C.c_float, _f32p, C.c_void_p, C.c_int, _f32p, C.c_int)
_sig("tpto_w8a8_gemm_refloop", None, _i8p, _i8p, _sz, _sz, _sz, C.c_float, _f32p, C.c_void_p, _f32p,
     _sz, _sz, C.c_int)
_sig("tpto_requant_i8", C.c_float, C.c_float, C.c_float, C.POINTER(C.c_int8))
_sig("tpto_quantize_i8_static", None, _f32p, _sz, C.c_float, _i8p)
_sig("tpto_absmax", C.c_float, _f32p, _sz)
_sig("tpto_w4_gemm", None, _f32p, _u8p, _f32p, _sz, _sz, _sz, C.c_void_p, C.c_int, _f32p, C.c_int)
_sig("tpto_max_pool2d", None, _f32p, _sz, _sz, _sz, _sz, _sz, _sz, _sz, _sz, _sz, _sz, _f32p, _sz, _sz)
_sig("tpto_average_pool2d", None, _f32p, _sz, _sz, _sz, _sz, _sz, _sz, _sz, _sz, _sz, _sz, _f32p, _sz, _sz)
_sig("tpto_add_bias_nchw", None, _f32p, _sz, _sz, _sz, _f32p)
_sig("tpto_add_bias_rows", None, _f32p, _sz, _sz, _f32p)
_sig("tpto_layernorm", None, _f32p, _sz, _sz, _f32p, _f32p, C.c_float, _f32p)
_sig("tpto_gelu_det_array", None, _f32p, _sz, _f32p)
_sig("tpto_exp_det_array", None, _f32p, _sz, _f32p)
_sig("tpto_attention_i8", None, _f32p, _sz, _sz, _sz, C.c_float, _f32p, _sz, _sz)
_sig("tpto_layernorm_res", None, _f32p, C.c_void_p, _sz, _sz, _f32p, _f32p, C.c_float, _f32p)
_sig("tpto_binary", None, C.c_int, _f32p, _szp, _sz, _f32p, _szp, _sz, _f32p, _szp, _sz)
_sig("tpto_batch_norm", None, _f32p, _sz, _f32p, _f32p, _f32p, _f32p, _sz, _sz, C.c_float, _f32p)
_sig("tpto_transpose", None, _f32p, _szp, _sz, _szp, _f32p)
_sig("tpto_concat_copy_one", None, _f32p, _sz, _sz, _sz, _sz, _f32p, _sz)


def _check(st):
    if st:
        e, a = _sz(), _sz()
        _lib.tpto_last_size_mismatch(C.byref(e), C.byref(a))
        if st == SIZE_MISMATCH:
            raise OracleError(st, e.value, a.value)
        raise OracleError(st)


def _f32(x):
    return np.ascontiguousarray(x, dtype=np.float32)


def _ptr_or_none(arr):
    return None if arr is None else arr.ctypes.data_as(C.c_void_p)


# ---------------------------------------------------------------- generators
def lcg_sym(n, seed):
    """dispatch.rs:274-282 test LCG mapped to [-1, 1)."""
    out = np.empty(n, np.float32)
    _lib.tpto_lcg_sym(out, n, seed)
    return out


def lcg_uniform(n, seed):
    out = np.empty(n, np.float32)
    _lib.tpto_lcg_uniform(out, n, seed)
    return out


def normal(n, seed, mean=0.0, std=1.0):
    out = np.empty(n, np.float32)
    _lib.tpto_normal(out, n, seed, mean, std)
    return out


# ---------------------------------------------------------------- Backend ops
def matmul_naive(a, a_shape, b, b_shape, out_len=None):
    a, b = _f32(a).ravel(), _f32(b).ravel()
    m, k = a_shape
    kb, n = b_shape
    out = np.empty(m * n if out_len is None else out_len, np.float32)
    _check(_lib.tpto_matmul_naive(a, a.size, m, k, b, b.size, kb, n, out, out.size))
    return out


def gemm(a, m, k, b, n, c=None, alpha=1.0, beta=1.0, trans_a=False, trans_b=False, out_len=None):
    """ONNX Gemm (tpto_gemm): Y = alpha * op(A) op(B) + beta * C."""
    a, b = _f32(a).ravel(), _f32(b).ravel()
    cc = None if c is None else _f32(c).ravel()
    out = np.empty(m * n if out_len is None else out_len, np.float32)
    _check(_lib.tpto_gemm(a, a.size, m, k, int(trans_a), b, b.size, n, int(trans_b), _ptr_or_none(cc),
                          0 if cc is None else cc.size, alpha, beta, out, out.size))
    return out


def matmul(a, a_shape, b, b_shape, threads=1, out_len=None):
    """avx512.rs:55-78 / avx2.rs:47-66 (bit-identical to naive.rs:13-33)."""
    a, b = _f32(a).ravel(), _f32(b).ravel()
    m, k = a_shape
    kb, n = b_shape
    out = np.empty(m * n if out_len is None else out_len, np.float32)
    _check(_lib.tpto_matmul_avx(a, a.size, m, k, b, b.size, kb, n, out, out.size, threads))
    return out


def conv_out_hw(in_shape, w_shape, stride=(1, 1), pad=(0, 0)):
    oh = (in_shape[2] + 2 * pad[0] - w_shape[2]) // stride[0] + 1
    ow = (in_shape[3] + 2 * pad[1] - w_shape[3]) // stride[1] + 1
    return oh, ow


def conv2d(x, in_shape, w, w_shape, stride=(1, 1), pad=(0, 0), threads=1, out_len=None):
    """naive.rs:36-83 (every CPU backend delegates conv here)."""
    x, w = _f32(x).ravel(), _f32(w).ravel()
    if out_len is None:
        oh, ow = conv_out_hw(in_shape, w_shape, stride, pad)
        out_len = in_shape[0] * w_shape[0] * oh * ow
    out = np.empty(max(out_len, 0), np.float32)
    _check(_lib.tpto_conv2d(x, x.size, np.array(in_shape, np.uintp), w, w.size, np.array(w_shape, np.uintp),
                            out, out.size, stride[0], stride[1], pad[0], pad[1], threads))
    return out


def elementwise_add(a, b, out_len=None):
    a, b = _f32(a).ravel(), _f32(b).ravel()
    out = np.empty(a.size if out_len is None else out_len, np.float32)
    _check(_lib.tpto_elementwise_add(a, a.size, b, b.size, out, out.size))
    return out


def _unary(fn, a, out_len=None):
    a = _f32(a).ravel()
    out = np.empty(a.size if out_len is None else out_len, np.float32)
    _check(fn(a, a.size, out, out.size))
    return out


def relu(a, out_len=None):
    return _unary(_lib.tpto_relu, a, out_len)


def sigmoid(a, out_len=None):
    return _unary(_lib.tpto_sigmoid, a, out_len)


def gelu(a, out_len=None):
    return _unary(_lib.tpto_gelu, a, out_len)


def softmax(a, row_len, out_len=None):
    a = _f32(a).ravel()
    out = np.empty(a.size if out_len is None else out_len, np.float32)
    _check(_lib.tpto_softmax(a, a.size, out, out.size, row_len))
    return out


# ---------------------------------------------------------------- quantize
def quantize_i8_symmetric(x):
    x = _f32(x).ravel()
    q = np.empty(x.size, np.int8)
    s = _lib.tpto_quantize_i8_symmetric(x, x.size, q)
    return q, np.float32(s)


def quantize_i8_asymmetric(x):
    x = _f32(x).ravel()
    q = np.empty(x.size, np.int8)
    s, zp = C.c_float(), C.c_int32()
    _lib.tpto_quantize_i8_asymmetric(x, x.size, q, C.byref(s), C.byref(zp))
    return q, np.float32(s.value), int(zp.value)


def quantize_i8_symmetric_per_channel(x, rows):
    x = _f32(x).ravel()
    q = np.empty(x.size, np.int8)
    s = np.empty(max(rows, 1), np.float32)
    _check(_lib.tpto_quantize_i8_symmetric_per_channel(x, x.size, rows, q, s))
    return q, s[:rows]


def pack_i4(v):
    v = np.ascontiguousarray(v, np.int8).ravel()
    out = np.zeros((v.size + 1) // 2, np.uint8)
    _check(_lib.tpto_pack_i4(v, v.size, out))
    return out


def unpack_i4(packed, n):
    packed = np.ascontiguousarray(packed, np.uint8).ravel()
    out = np.zeros(n, np.int8)
    c = _lib.tpto_unpack_i4(packed, packed.size, n, out)
    return out[:c]


def quantize_i4_symmetric(x):
    x = _f32(x).ravel()
    p = np.zeros((x.size + 1) // 2, np.uint8)
    s = _lib.tpto_quantize_i4_symmetric(x, x.size, p)
    return p, np.float32(s)


def quantize_i4_symmetric_per_channel(x, rows):
    x = _f32(x).ravel()
    cols = x.size // rows if rows else 0
    p = np.zeros(max(rows * ((cols + 1) // 2), 1), np.uint8)
    s = np.empty(max(rows, 1), np.float32)
    _check(_lib.tpto_quantize_i4_symmetric_per_channel(x, x.size, rows, p, s))
    return p[: rows * ((cols + 1) // 2)], s[:rows]


def dequantize_i8_symmetric(q, scale):
    q = np.ascontiguousarray(q, np.int8).ravel()
    out = np.empty(q.size, np.float32)
    _lib.tpto_dequantize_i8_symmetric(q, q.size, scale, out)
    return out


def dequantize_i8_asymmetric(q, scale, zp):
    q = np.ascontiguousarray(q, np.int8).ravel()
    out = np.empty(q.size, np.float32)
    _lib.tpto_dequantize_i8_asymmetric(q, q.size, scale, zp, out)
    return out


def dequantize_i8_symmetric_per_channel(q, scales):
    q = np.ascontiguousarray(q, np.int8).ravel()
    scales = _f32(scales).ravel()
    out = np.empty(q.size, np.float32)
    _check(_lib.tpto_dequantize_i8_symmetric_per_channel(q, q.size, scales, scales.size, out))
    return out


def dequantize_i4_symmetric(packed, n, scale):
    packed = np.ascontiguousarray(packed, np.uint8).ravel()
    out = np.zeros(n, np.float32)
    _lib.tpto_dequantize_i4_symmetric(packed, packed.size, n, scale, out)
    return out[: min(n, 2 * packed.size)]


def dequantize_i4_symmetric_per_channel(packed, row_elems, scales):
    packed = np.ascontiguousarray(packed, np.uint8).ravel()
    scales = _f32(scales).ravel()
    out = np.zeros(row_elems * scales.size, np.float32)
    _lib.tpto_dequantize_i4_symmetric_per_channel(packed, packed.size, row_elems, scales, scales.size, out)
    return out


def quantized_matmul_i8(a, a_shape, a_scale, b, b_shape, b_scales):
    """ptq.rs:293-324 (per-tensor; B is [k, n])."""
    a = np.ascontiguousarray(a, np.int8).ravel()
    b = np.ascontiguousarray(b, np.int8).ravel()
    b_scales = _f32(b_scales).ravel()
    out = np.empty(a_shape[0] * b_shape[1], np.float32)
    _check(_lib.tpto_quantized_matmul_i8(a, a.size, a_shape[0], a_shape[1], a_scale, b, b.size,
                                         b_shape[0], b_shape[1], b_scales, b_scales.size, out, out.size))
    return out


# ------------------------------------------------- per-channel W8A8 and W4
def i8_gemm_acc(a, wt, m, n, k, threads=1):
    a = np.ascontiguousarray(a, np.int8).ravel()
    wt = np.ascontiguousarray(wt, np.int8).ravel()
    acc = np.empty(m * n, np.int32)
    _lib.tpto_i8_gemm_acc(a, wt, m, n, k, acc, threads)
    return acc


def w8a8_gemm(a, wt, m, n, k, a_scale, w_scales, bias=None, act=ACT_NONE, threads=1):
    a = np.ascontiguousarray(a, np.int8).ravel()
    wt = np.ascontiguousarray(wt, np.int8).ravel()
    w_scales = _f32(w_scales).ravel()
    bias = None if bias is None else _f32(bias).ravel()
    y = np.empty(m * n, np.float32)
    _lib.tpto_w8a8_gemm(a, wt, m, n, k, a_scale, w_scales, _ptr_or_none(bias), act, y, threads)
    return y


def w8a8_gemm_refloop(a, b_kn, m, n, k, a_scale, w_scales, bias, rows, threads):
    """The reference's own loop (ptq.rs:312-319, B [k, n] strided) over rows [0, rows)."""
    a = np.ascontiguousarray(a, np.int8).ravel()
    b_kn = np.ascontiguousarray(b_kn, np.int8).ravel()
    w_scales = _f32(w_scales).ravel()
    bias = None if bias is None else _f32(bias).ravel()
    y = np.zeros(m * n, np.float32)
    _lib.tpto_w8a8_gemm_refloop(a, b_kn, m, n, k, a_scale, w_scales, _ptr_or_none(bias), y, 0, rows, threads)
    return y


def quantize_i8_static(x, scale):
    x = _f32(x).ravel()
    q = np.empty(x.size, np.int8)
    _lib.tpto_quantize_i8_static(x, x.size, np.float32(scale), q)
    return q


def absmax(x):
    x = _f32(x).ravel()
    return np.float32(_lib.tpto_absmax(x, x.size))


def sym_scale(m):
    """quantize_i8_symmetric's scale rule (quant.rs:27-31) for a max |x|."""
    m = np.float32(m)
    return np.float32(1.0) if m == 0 else np.float32(m / np.float32(127.0))


def requant_i8(y, out_scale):
    q = C.c_int8()
    _lib.tpto_requant_i8(y, out_scale, C.byref(q))
    return int(q.value)


def w4_gemm(x, wt_packed, w_scales, m, n, k, bias=None, act=ACT_NONE, threads=1):
    x = _f32(x).ravel()
    wt_packed = np.ascontiguousarray(wt_packed, np.uint8).ravel()
    w_scales = _f32(w_scales).ravel()
    bias = None if bias is None else _f32(bias).ravel()
    y = np.empty(m * n, np.float32)
    _lib.tpto_w4_gemm(x, wt_packed, w_scales, m, n, k, _ptr_or_none(bias), act, y, threads)
    return y


# ---------------------------------------------------------------- runtime kernels
def max_pool2d(x, n, c, h, w, kernel, stride, pad):
    x = _f32(x).ravel()
    oh = (h + 2 * pad[0] - kernel[0]) // stride[0] + 1
    ow = (w + 2 * pad[1] - kernel[1]) // stride[1] + 1
    out = np.empty(n * c * oh * ow, np.float32)
    _lib.tpto_max_pool2d(x, n, c, h, w, kernel[0], kernel[1], stride[0], stride[1], pad[0], pad[1], out, oh, ow)
    return out


def average_pool2d(x, n, c, h, w, kernel, stride, pad):
    x = _f32(x).ravel()
    oh = (h + 2 * pad[0] - kernel[0]) // stride[0] + 1
    ow = (w + 2 * pad[1] - kernel[1]) // stride[1] + 1
    out = np.empty(n * c * oh * ow, np.float32)
    _lib.tpto_average_pool2d(x, n, c, h, w, kernel[0], kernel[1], stride[0], stride[1], pad[0], pad[1],
                             out, oh, ow)
    return out


def add_bias_nchw(out, n, c, hw, bias):
    out = _f32(out).ravel().copy()
    _lib.tpto_add_bias_nchw(out, n, c, hw, _f32(bias).ravel())
    return out


def add_bias_rows(out, rows, cols, bias):
    out = _f32(out).ravel().copy()
    _lib.tpto_add_bias_rows(out, rows, cols, _f32(bias).ravel())
    return out


def layernorm(x, rows, cols, gamma, beta, eps=1e-5):
    x = _f32(x).ravel()
    y = np.empty(rows * cols, np.float32)
    _lib.tpto_layernorm(x, rows, cols, _f32(gamma).ravel(), _f32(beta).ravel(), eps, y)
    return y


# ------------------------------------------------------------------ runtime dispatch table
BIN_ADD, BIN_SUB, BIN_MUL, BIN_DIV = 0, 1, 2, 3


def _dims(d):
    return np.ascontiguousarray(np.asarray(d, np.uintp).ravel())


def broadcast_shape(ad, bd):
    """numpy broadcasting of two shapes, or None (kernels.rs:43-58 check_broadcast)."""
    r = max(len(ad), len(bd))
    a = [1] * (r - len(ad)) + list(ad)
    b = [1] * (r - len(bd)) + list(bd)
    out = []
    for x, y in zip(a, b):
        if x != y and x != 1 and y != 1:
            return None
        out.append(max(x, y))
    return out


def binary(op, a, ad, b, bd, od=None):
    """kernels::binary (crates/tpt-infer-runtime/src/kernels.rs:92-137)."""
    od = list(od if od is not None else broadcast_shape(ad, bd))
    a, b = _f32(a).ravel(), _f32(b).ravel()
    out = np.empty(int(np.prod(od, dtype=np.int64)), np.float32)
    _lib.tpto_binary(op, a, _dims(ad), len(ad), b, _dims(bd), len(bd), out, _dims(od), len(od))
    return out


def batch_norm(x, x_dims, scale, bias, mean, var, eps):
    """kernels::batch_norm (kernels.rs:425-476): channel mode for rank-4 x with one
    parameter per channel, else element mode."""
    x = _f32(x).ravel()
    scale, bias, mean, var = (_f32(v).ravel() for v in (scale, bias, mean, var))
    hw = int(x_dims[2] * x_dims[3]) if len(x_dims) == 4 and scale.size == x_dims[1] else 0
    out = np.empty(x.size, np.float32)
    _lib.tpto_batch_norm(x, x.size, scale, bias, mean, var, scale.size, hw, eps, out)
    return out


def transpose(x, x_dims, perm):
    """kernels::transpose (kernels.rs:484-532)."""
    x = _f32(x).ravel()
    out = np.empty(x.size, np.float32)
    _lib.tpto_transpose(x, _dims(x_dims), len(x_dims), _dims(perm), out)
    return out


def concat(inputs, dims_list, axis):
    """Concat of the runtime (exec.rs:471-513) through concat_copy_one (kernels.rs:548-588)."""
    rank = len(dims_list[0])
    ax = axis + rank if axis < 0 else axis
    od = list(dims_list[0])
    od[ax] = sum(d[ax] for d in dims_list)
    inner = int(np.prod(od[ax + 1:], dtype=np.int64))
    out = np.empty(int(np.prod(od, dtype=np.int64)), np.float32)
    off = 0
    for x, d in zip(inputs, dims_list):
        x = _f32(x).ravel()
        _lib.tpto_concat_copy_one(out, od[ax], off, d[ax], inner, x, x.size)
        off += d[ax]
    return out, od


def gelu_det(a):
    """The device's deterministic GELU (det_math.cuh), bit-exact restatement."""
    a = _f32(a).ravel()
    out = np.empty(a.size, np.float32)
    _lib.tpto_gelu_det_array(a, a.size, out)
    return out


def exp_det(a):
    """The device's deterministic exp (det_math.cuh), bit-exact restatement."""
    a = _f32(a).ravel()
    out = np.empty(a.size, np.float32)
    _lib.tpto_exp_det_array(a, a.size, out)
    return out


def layernorm_res(x, res, rows, cols, gamma, beta, eps=1e-5):
    """LayerNorm(x + res) in the device order (the fused residual layernorm)."""
    x = _f32(x).ravel()
    r = _f32(res).ravel()
    y = np.empty(rows * cols, np.float32)
    _lib.tpto_layernorm_res(x, r.ctypes.data_as(C.c_void_p), rows, cols, _f32(gamma).ravel(), _f32(beta).ravel(),
                            eps, y)
    return y


def attention_i8(qkv, batch, seq, heads, scale, b0=0, b1=None):
    """The device's integer tensor-core attention (attention_i8.cu), bit-exact;
    rows of batches [b0, b1) are filled."""
    qkv = _f32(qkv).ravel()
    b1 = batch if b1 is None else b1
    out = np.zeros(batch * seq * heads * 64, np.float32)
    _lib.tpto_attention_i8(qkv, batch, seq, heads, scale, out, b0, b1)
    return out

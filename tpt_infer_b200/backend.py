"""``CudaBackend``: the host-side mirror of tpt-infer's ``Backend`` trait
(crates/tpt-infer-ops/src/backend.rs:98-147) over the C ABI of
``libtpt_cuda.so``.

Method names, argument meaning and error behaviour follow the trait: every
method writes into a caller-provided output buffer and raises ``OpError`` with
the reference's variant (``SizeMismatch{expected, actual}``, ``ShapeMismatch``,
``Unsupported``, ``Invalid``) where the reference returns ``Err``. Host
buffers are numpy arrays (the trait's ``&[f32]`` slices). ``*_dev`` methods
take torch CUDA tensors and enqueue on the backend's stream.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from ._capi import lib

OK, SIZE_MISMATCH, SHAPE_MISMATCH, UNSUPPORTED, INVALID = 0, 1, 2, 3, 4
CUDA_ERROR, OUT_OF_MEMORY, TIMEOUT, NCCL_ERROR, DEVICE_CHECK = 5, 6, 7, 8, 9
ACT_NONE, ACT_RELU, ACT_GELU = 0, 1, 2

_KIND = {SIZE_MISMATCH: "SizeMismatch", SHAPE_MISMATCH: "ShapeMismatch", UNSUPPORTED: "Unsupported",
         INVALID: "Invalid"}


class OpError(Exception):
    """OpError (backend.rs:6-20). ``kind`` names the variant; SizeMismatch carries
    ``expected`` and ``actual``."""

    def __init__(self, code, expected=None, actual=None, detail=""):
        self.code = code
        self.kind = _KIND.get(code, "Cuda")
        self.expected = expected
        self.actual = actual
        msg = {
            SIZE_MISMATCH: f"size mismatch: expected {expected} elements, got {actual}",
            SHAPE_MISMATCH: "shape mismatch",
            UNSUPPORTED: "operation not supported by this backend",
            INVALID: "invalid argument",
        }.get(code, lib.tpt_cuda_status_str(code).decode())
        super().__init__(msg + (f" ({detail})" if detail else ""))

    def __eq__(self, other):
        return isinstance(other, OpError) and (self.code, self.expected, self.actual) == (
            other.code, other.expected, other.actual)

    __hash__ = Exception.__hash__


@dataclass(frozen=True)
class Conv2dOptions:
    """Conv2dOptions (backend.rs:49-58)."""

    stride_h: int = 1
    stride_w: int = 1
    pad_h: int = 0
    pad_w: int = 0

    @staticmethod
    def with_stride_padding(stride_h, stride_w, pad_h, pad_w):
        return Conv2dOptions(stride_h, stride_w, pad_h, pad_w)


def _ptr(arr):
    return arr.ctypes.data_as(C.c_void_p) if arr is not None else None


def _host(arr, dtype):
    a = np.asarray(arr)
    if a.dtype != dtype or not a.flags.c_contiguous:
        a = np.ascontiguousarray(a, dtype=dtype)
    return a


def _out(out, dtype):
    if not isinstance(out, np.ndarray) or out.dtype != dtype or not out.flags.c_contiguous:
        raise TypeError(f"out must be a C-contiguous numpy {np.dtype(dtype).name} array")
    return out


def _tptr(t):
    """Device pointer of a torch tensor (or None)."""
    return None if t is None else C.c_void_p(t.data_ptr())


class Weights:
    """A packed quantized weight resident in device memory (uploaded once)."""

    def __init__(self, backend, handle, kind, n, k):
        self._be = backend
        self.handle = handle
        self.kind = kind
        self.n = n
        self.k = k

    def free(self):
        if self.handle:
            lib.tpt_cuda_weights_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Graph:
    """A recorded launch sequence (tpt_cuda_capture_begin/_end)."""

    def __init__(self, be, handle):
        self.be, self.h = be, handle

    @property
    def kernels(self) -> int:
        return int(lib.tpt_cuda_graph_kernels(self.h))

    def launch(self):
        self.be._check(lib.tpt_cuda_graph_launch(self.be.ctx, self.h))

    def close(self):
        if self.h:
            lib.tpt_cuda_graph_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class CudaBackend:
    """The CUDA implementation of the Backend trait on one B200."""

    def __init__(self, ctx, device):
        self._ctx = ctx
        self.device = device

    # -- construction, like WebGpuBackend::new() -> Option<Self> (webgpu.rs:272)
    @classmethod
    def new(cls, device: int = 0, stream=None):
        """Returns a backend on ``device`` or None when no usable sm_100 device exists.
        ``stream`` may be a torch.cuda.Stream (its handle is used) or None (own stream)."""
        h = C.c_void_p()
        s = None
        if stream is not None:
            s = C.c_void_p(stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream))
        st = lib.tpt_cuda_ctx_create(device, s, C.byref(h))
        if st != OK:
            return None
        return cls(h, device)

    def close(self):
        if self._ctx:
            lib.tpt_cuda_ctx_destroy(self._ctx)
            self._ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def ctx(self):
        return self._ctx

    @property
    def stream_handle(self) -> int:
        return int(lib.tpt_cuda_ctx_stream(self._ctx) or 0)

    def launch_count(self) -> int:
        return int(lib.tpt_cuda_ctx_launch_count(self._ctx))

    def sync(self):
        self._check(lib.tpt_cuda_ctx_sync(self._ctx))

    def capture(self, fn):
        """Records the device-pointer calls ``fn()`` issues on this context into a
        CUDA graph (run ``fn`` once before, so every workspace is sized)."""
        self._check(lib.tpt_cuda_capture_begin(self._ctx))
        err = None
        try:
            fn()
        except Exception as e:  # the recording must still be closed
            err = e
        h = C.c_void_p()
        st = lib.tpt_cuda_capture_end(self._ctx, C.byref(h))
        if err is not None:
            if h.value:
                lib.tpt_cuda_graph_destroy(h)
            raise err
        self._check(st)
        return Graph(self, h)

    def name(self) -> str:
        """Backend::name (backend.rs:100)."""
        return lib.tpt_cuda_backend_name().decode()

    def _check(self, st):
        if st == OK:
            return
        if st == SIZE_MISMATCH:
            e, a = C.c_size_t(), C.c_size_t()
            lib.tpt_cuda_last_size_mismatch(self._ctx, C.byref(e), C.byref(a))
            raise OpError(st, e.value, a.value)
        detail = lib.tpt_cuda_last_error(self._ctx).decode() if st >= CUDA_ERROR else ""
        raise OpError(st, detail=detail)

    # ------------------------------------------------------------ trait methods
    def gemm(self, a, m, k, b, n, c=None, alpha=1.0, beta=1.0, trans_a=False, trans_b=False, out=None):
        """ONNX Gemm, Y = alpha * op(A) op(B) + beta * C (the attributes tpt-infer's
        loader drops, crates/tpt-infer-onnx/src/registry.rs:21); C is [n] or [m, n]."""
        a, b = _host(a, np.float32).ravel(), _host(b, np.float32).ravel()
        cc = None if c is None else _host(c, np.float32).ravel()
        y = np.empty(m * n, np.float32) if out is None else _out(out, np.float32)
        self._check(lib.tpt_cuda_gemm(self._ctx, _ptr(a), a.size, m, k, int(trans_a), _ptr(b), b.size, n,
                                      int(trans_b), _ptr(cc), 0 if cc is None else cc.size, float(alpha),
                                      float(beta), _ptr(y), y.size))
        return y

    def matmul(self, a, a_shape, b, b_shape, out):
        """Backend::matmul (backend.rs:106-113): out[m,n] = a[m,k] @ b[k,n]."""
        a, b, out = _host(a, np.float32).ravel(), _host(b, np.float32).ravel(), _out(out, np.float32)
        m, k = a_shape
        kb, n = b_shape
        self._check(lib.tpt_cuda_matmul(self._ctx, _ptr(a), a.size, m, k, _ptr(b), b.size, kb, n, _ptr(out),
                                        out.size))

    def conv2d(self, inp, in_shape, weight, w_shape, out, options: Conv2dOptions = Conv2dOptions()):
        """Backend::conv2d (backend.rs:119-127): NCHW input, OIHW weight."""
        inp, weight, out = _host(inp, np.float32).ravel(), _host(weight, np.float32).ravel(), _out(out, np.float32)
        ish = (C.c_size_t * 4)(*in_shape)
        wsh = (C.c_size_t * 4)(*w_shape)
        self._check(lib.tpt_cuda_conv2d(self._ctx, _ptr(inp), inp.size, ish, _ptr(weight), weight.size, wsh,
                                        _ptr(out), out.size, options.stride_h, options.stride_w, options.pad_h,
                                        options.pad_w))

    def elementwise_add(self, a, b, out):
        """Backend::elementwise_add (backend.rs:130)."""
        a, b, out = _host(a, np.float32).ravel(), _host(b, np.float32).ravel(), _out(out, np.float32)
        self._check(lib.tpt_cuda_elementwise_add(self._ctx, _ptr(a), a.size, _ptr(b), b.size, _ptr(out), out.size))

    def _unary(self, fn, a, out):
        a, out = _host(a, np.float32).ravel(), _out(out, np.float32)
        self._check(fn(self._ctx, _ptr(a), a.size, _ptr(out), out.size))

    def relu(self, a, out):
        """Backend::relu (backend.rs:133)."""
        self._unary(lib.tpt_cuda_relu, a, out)

    def sigmoid(self, a, out):
        """Backend::sigmoid (backend.rs:142)."""
        self._unary(lib.tpt_cuda_sigmoid, a, out)

    def gelu(self, a, out):
        """Backend::gelu (backend.rs:146)."""
        self._unary(lib.tpt_cuda_gelu, a, out)

    def softmax(self, a, out, row_len):
        """Backend::softmax (backend.rs:139)."""
        a, out = _host(a, np.float32).ravel(), _out(out, np.float32)
        self._check(lib.tpt_cuda_softmax(self._ctx, _ptr(a), a.size, _ptr(out), out.size, row_len))

    # ------------------------------------------------------------ quantize crate
    def quantize_i8_symmetric(self, data):
        """quantize_i8_symmetric (quant.rs:25-40) -> (q int8, scale)."""
        x = _host(data, np.float32).ravel()
        q = np.empty(x.size, np.int8)
        s = C.c_float()
        self._check(lib.tpt_cuda_quantize_i8_symmetric(self._ctx, _ptr(x), x.size, _ptr(q), C.byref(s)))
        return q, np.float32(s.value)

    def quantize_i8_symmetric_per_channel(self, data, rows):
        """quantize_i8_symmetric_per_channel (quant.rs:95-107) -> (q, scales[rows])."""
        x = _host(data, np.float32).ravel()
        q = np.empty(x.size, np.int8)
        s = np.empty(max(rows, 1), np.float32)
        self._check(lib.tpt_cuda_quantize_i8_symmetric_per_channel(self._ctx, _ptr(x), x.size, rows, _ptr(q),
                                                                   _ptr(s)))
        return q, s[:rows]

    def quantize_i8_asymmetric(self, data):
        """quantize_i8_asymmetric (quant.rs:45-90) -> (q, scale, zero_point)."""
        x = _host(data, np.float32).ravel()
        q = np.empty(x.size, np.int8)
        s, z = C.c_float(), C.c_int32()
        self._check(lib.tpt_cuda_quantize_i8_asymmetric(self._ctx, _ptr(x), x.size, _ptr(q), C.byref(s),
                                                        C.byref(z)))
        return q, np.float32(s.value), int(z.value)

    def pack_i4(self, values):
        """pack_i4 (quant.rs:123-140); out-of-range values raise OpError(Invalid)."""
        v = _host(values, np.int8).ravel()
        out = np.zeros((v.size + 1) // 2, np.uint8)
        self._check(lib.tpt_cuda_pack_i4(self._ctx, _ptr(v), v.size, _ptr(out)))
        return out

    def unpack_i4(self, packed, n):
        """unpack_i4 (quant.rs:143-157)."""
        p = _host(packed, np.uint8).ravel()
        out = np.zeros(n, np.int8)
        w = C.c_size_t()
        self._check(lib.tpt_cuda_unpack_i4(self._ctx, _ptr(p), p.size, n, _ptr(out), C.byref(w)))
        return out[: w.value]

    def quantize_i4_symmetric(self, data):
        """quantize_i4_symmetric (quant.rs:171-186) -> (packed, scale)."""
        x = _host(data, np.float32).ravel()
        p = np.zeros((x.size + 1) // 2, np.uint8)
        s = C.c_float()
        self._check(lib.tpt_cuda_quantize_i4_symmetric(self._ctx, _ptr(x), x.size, _ptr(p), C.byref(s)))
        return p, np.float32(s.value)

    def quantize_i4_symmetric_per_channel(self, data, rows):
        """quantize_i4_symmetric_per_channel (quant.rs:192-204) -> (packed, scales)."""
        x = _host(data, np.float32).ravel()
        cols = x.size // rows if rows else 0
        p = np.zeros(max(rows * ((cols + 1) // 2), 1), np.uint8)
        s = np.empty(max(rows, 1), np.float32)
        self._check(lib.tpt_cuda_quantize_i4_symmetric_per_channel(self._ctx, _ptr(x), x.size, rows, _ptr(p),
                                                                   _ptr(s)))
        return p[: rows * ((cols + 1) // 2)], s[:rows]

    def dequantize_i8_symmetric(self, q, scale):
        """dequantize_i8_symmetric (dequant.rs:13-15)."""
        q = _host(q, np.int8).ravel()
        out = np.empty(q.size, np.float32)
        self._check(lib.tpt_cuda_dequantize_i8_symmetric(self._ctx, _ptr(q), q.size, float(scale), _ptr(out)))
        return out

    def dequantize_i8_symmetric_per_channel(self, q, scales):
        """dequantize_i8_symmetric_per_channel (dequant.rs:26-37)."""
        q, s = _host(q, np.int8).ravel(), _host(scales, np.float32).ravel()
        out = np.empty(q.size, np.float32)
        self._check(lib.tpt_cuda_dequantize_i8_symmetric_per_channel(self._ctx, _ptr(q), q.size, _ptr(s), s.size,
                                                                     _ptr(out)))
        return out

    def dequantize_i8_asymmetric(self, q, scale, zero_point):
        """dequantize_i8_asymmetric (dequant.rs:18-22): (q - zero_point) * scale."""
        q = _host(q, np.int8).ravel()
        out = np.empty(q.size, np.float32)
        self._check(lib.tpt_cuda_dequantize_i8_asymmetric(self._ctx, _ptr(q), q.size, float(scale), int(zero_point),
                                                          _ptr(out)))
        return out

    def dequantize_i4_symmetric(self, packed, n, scale):
        """dequantize_i4_symmetric (dequant.rs:45-50): min(n, 2 * len(packed)) values."""
        p = _host(packed, np.uint8).ravel()
        out = np.empty(max(min(n, 2 * p.size), 1), np.float32)
        w = C.c_size_t()
        self._check(lib.tpt_cuda_dequantize_i4_symmetric(self._ctx, _ptr(p), p.size, n, float(scale), _ptr(out),
                                                         C.byref(w)))
        return out[:w.value]

    def dequantize_i4_symmetric_per_channel(self, packed, row_elems, scales):
        """dequantize_i4_symmetric_per_channel (dequant.rs:56-71)."""
        p, s = _host(packed, np.uint8).ravel(), _host(scales, np.float32).ravel()
        out = np.zeros(row_elems * s.size, np.float32)
        self._check(lib.tpt_cuda_dequantize_i4_symmetric_per_channel(self._ctx, _ptr(p), p.size, row_elems,
                                                                     _ptr(s), s.size, _ptr(out)))
        return out

    def quantized_matmul_i8(self, a, a_shape, a_scale, b, b_shape, b_scales, out):
        """quantized_matmul_i8 (ptq.rs:293-324): B [k, n], per-tensor b_scales[0]."""
        a, b = _host(a, np.int8).ravel(), _host(b, np.int8).ravel()
        bs = _host(b_scales, np.float32).ravel()
        out = _out(out, np.float32)
        self._check(lib.tpt_cuda_quantized_matmul_i8(self._ctx, _ptr(a), a.size, a_shape[0], a_shape[1],
                                                     float(a_scale), _ptr(b), b.size, b_shape[0], b_shape[1],
                                                     _ptr(bs) if bs.size else None, bs.size, _ptr(out), out.size))

    # ------------------------------------------------------------ packed weights + GEMMs
    def upload_i8(self, wt_nk, scales, n, k) -> Weights:
        """Uploads W^T [n, k] int8 + n scales (the QuantizedTensor bytes)."""
        wt, s = _host(wt_nk, np.int8).ravel(), _host(scales, np.float32).ravel()
        if wt.size != n * k or s.size != n:
            raise OpError(SIZE_MISMATCH, n * k, wt.size)
        h = C.c_void_p()
        self._check(lib.tpt_cuda_weights_upload_i8(self._ctx, _ptr(wt), _ptr(s), n, k, C.byref(h)))
        return Weights(self, h, 8, n, k)

    def upload_i4(self, packed, scales, n, k) -> Weights:
        """Uploads n nibble rows of k/2 bytes (low nibble first) + n scales."""
        p, s = _host(packed, np.uint8).ravel(), _host(scales, np.float32).ravel()
        if s.size != n:
            raise OpError(SIZE_MISMATCH, n, s.size)
        h = C.c_void_p()
        self._check(lib.tpt_cuda_weights_upload_i4(self._ctx, _ptr(p), p.size, _ptr(s), n, k, C.byref(h)))
        return Weights(self, h, 4, n, k)

    def w8a8_gemm(self, a, m, k, a_scale, w: Weights, bias=None, act=ACT_NONE, out=None):
        """Per-channel W8A8 GEMM on host buffers -> y [m, n] f32."""
        a = _host(a, np.int8).ravel()
        if a.size != m * k:
            raise OpError(SIZE_MISMATCH, m * k, a.size)
        b = None if bias is None else _host(bias, np.float32).ravel()
        y = np.empty(m * w.n, np.float32) if out is None else _out(out, np.float32)
        self._check(lib.tpt_cuda_w8a8_gemm(self._ctx, _ptr(a), m, k, float(a_scale), w.handle, _ptr(b), act,
                                           _ptr(y)))
        return y

    def w4_gemm(self, x, m, k, w: Weights, bias=None, act=ACT_NONE, out=None):
        """W4 GEMM on host buffers: x [m, k] f32 -> y [m, n] f32."""
        x = _host(x, np.float32).ravel()
        if x.size != m * k:
            raise OpError(SIZE_MISMATCH, m * k, x.size)
        b = None if bias is None else _host(bias, np.float32).ravel()
        y = np.empty(m * w.n, np.float32) if out is None else _out(out, np.float32)
        self._check(lib.tpt_cuda_w4_gemm(self._ctx, _ptr(x), m, k, w.handle, _ptr(b), act, _ptr(y)))
        return y

    # device-pointer forms (torch CUDA tensors; enqueued on the backend stream)
    def w8a8_gemm_dev(self, a, m, a_scale, w: Weights, bias, act, out):
        self._check(lib.tpt_cuda_w8a8_gemm_dev(self._ctx, _tptr(a), m, float(a_scale), w.handle, _tptr(bias), act,
                                               _tptr(out)))

    def w8a8_gemm_acc_dev(self, a, m, w: Weights, acc):
        self._check(lib.tpt_cuda_w8a8_gemm_acc_dev(self._ctx, _tptr(a), m, w.handle, _tptr(acc)))

    def w4_gemm_dev(self, x, m, w: Weights, bias, act, out):
        self._check(lib.tpt_cuda_w4_gemm_dev(self._ctx, _tptr(x), m, w.handle, _tptr(bias), act, _tptr(out)))

    def quantize_i8_symmetric_dev(self, x, q, scale_dev):
        self._check(lib.tpt_cuda_quantize_i8_symmetric_dev(self._ctx, _tptr(x), x.numel(), _tptr(q),
                                                           _tptr(scale_dev)))

    def matmul_dev(self, a, m, k, b, n, out):
        self._check(lib.tpt_cuda_matmul_dev(self._ctx, _tptr(a), m, k, _tptr(b), n, _tptr(out)))

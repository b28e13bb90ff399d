"""Oracle compositions of the model workloads (TEST INFRASTRUCTURE ONLY).

Each function replays, on the CPU oracle's primitives, the node sequence that
the corresponding device plan in ``tpt_infer_b200/graphs.py`` runs -- the way
tpt-infer's runtime would execute those nodes one by one
(crates/tpt-infer-runtime/src/exec.rs:347-533): f32 MatMul (naive.rs:13-33),
broadcast bias adds (kernels.rs:150-178), Relu/Softmax (naive.rs:95-125),
max/average pooling (kernels.rs:271-390), and the quantized-weight path
(quant.rs / ptq.rs, with this backend's per-channel W8A8 epilogue).

Calibration is replayed exactly: on each calibration run a quantization point
uses that run's scale (max|x| / 127) and records max|x|; the frozen scale is the
running maximum / 127.
"""
from __future__ import annotations

import numpy as np

from . import oracle as O

TH = 8  # OpenMP threads for the heavy oracle kernels


def _relu(x):
    return np.where(x > 0, x, np.float32(0.0)).astype(np.float32)


# ------------------------------------------------------------------ MLP
def mlp_f32(x, W, batch):
    h = O.matmul(x, (batch, 784), W.w1, (784, 512), threads=TH)
    h = _relu(O.add_bias_rows(h, batch, 512, W.b1))
    z = O.matmul(h, (batch, 512), W.w2, (512, 10), threads=TH)
    z = O.add_bias_rows(z, batch, 10, W.b2)
    return O.softmax(z, 10)


def mlp_int8(x, W, batch, q, scales):
    """q = (q1, s1, q2, s2) per-channel weights; scales = (a1, a2) activation scales."""
    q1, s1, q2, s2 = q
    a1, a2 = scales
    xq = O.quantize_i8_static(x, a1)
    h = O.w8a8_gemm(xq, q1, batch, 512, 784, a1, s1, W.b1, O.ACT_RELU, threads=TH)
    hq = O.quantize_i8_static(h, a2)
    z = O.w8a8_gemm(hq, q2, batch, 10, 512, a2, s2, W.b2, O.ACT_NONE, threads=TH)
    return O.softmax(z, 10)


def mlp_int8_calibrate(cal_batches, W, batch, q):
    q1, s1, q2, s2 = q
    m1 = m2 = np.float32(0.0)
    for xb in cal_batches:
        a = O.absmax(xb)
        m1 = max(m1, a)
        sc = O.sym_scale(a)
        h = O.w8a8_gemm(O.quantize_i8_static(xb, sc), q1, batch, 512, 784, sc, s1, W.b1, O.ACT_RELU, threads=TH)
        m2 = max(m2, O.absmax(h))
    return O.sym_scale(m1), O.sym_scale(m2)


# ------------------------------------------------------------------ ResNet-18 (NHWC)
def _im2col(x_nhwc, k, s, pad, kp):
    n, h, w, c = x_nhwc.shape
    oh, ow = (h + 2 * pad - k) // s + 1, (w + 2 * pad - k) // s + 1
    xp = np.zeros((n, h + 2 * pad, w + 2 * pad, c), x_nhwc.dtype)
    xp[:, pad:pad + h, pad:pad + w, :] = x_nhwc
    taps = [xp[:, ky:ky + s * oh:s, kx:kx + s * ow:s, :] for ky in range(k) for kx in range(k)]
    col = np.stack(taps, axis=3).reshape(n * oh * ow, k * k * c)
    if kp != col.shape[1]:
        col = np.concatenate([col, np.zeros((col.shape[0], kp - col.shape[1]), col.dtype)], axis=1)
    return np.ascontiguousarray(col), oh, ow


def _conv(xq_nhwc, cv, a_scale, act):
    col, oh, ow = _im2col(xq_nhwc, cv.k, cv.stride, cv.pad, cv.qw.k)
    n = xq_nhwc.shape[0]
    y = O.w8a8_gemm(col, cv.qw.q, col.shape[0], cv.cout, cv.qw.k, a_scale, cv.qw.scales, cv.qw.bias, act, threads=TH)
    return y.reshape(n, oh, ow, cv.cout)


class _Scales:
    """Quantization points in plan order: either replayed calibration or given."""

    def __init__(self, given=None):
        self.given = None if given is None else list(given)
        self.maxes = []
        self.i = 0

    def point(self, x):
        if self.given is not None:
            s = np.float32(self.given[self.i])
        else:
            a = O.absmax(x)
            if self.i >= len(self.maxes):
                self.maxes.append(np.float32(0.0))
            self.maxes[self.i] = max(self.maxes[self.i], a)
            s = O.sym_scale(a)
        self.i += 1
        return s

    def frozen(self):
        return np.array([O.sym_scale(m) for m in self.maxes], np.float32)


def resnet18(x_nchw, spec, batch, scales=None, calib=None):
    """Logits [batch, 1000]. ``scales``: frozen activation scales in plan order, or
    ``calib`` (a _Scales) to replay a calibration run."""
    sc = calib if calib is not None else _Scales(scales)
    x = np.asarray(x_nchw, np.float32).reshape(batch, 3, 224, 224)
    x_nhwc = np.ascontiguousarray(x.transpose(0, 2, 3, 1))
    s0 = sc.point(x_nhwc)
    xq = O.quantize_i8_static(x_nhwc, s0).reshape(x_nhwc.shape)
    y = _conv(xq, spec.convs[0], s0, O.ACT_RELU)
    nchw = np.ascontiguousarray(y.transpose(0, 3, 1, 2))
    mp = O.max_pool2d(nchw, batch, 64, y.shape[1], y.shape[2], (3, 3), (2, 2), (1, 1))
    oh = (y.shape[1] + 2 - 3) // 2 + 1
    cur = np.ascontiguousarray(mp.reshape(batch, 64, oh, oh).transpose(0, 2, 3, 1))
    ci = 1
    for cin, cout, s in [(64, 64, 1), (64, 64, 1), (64, 128, 2), (128, 128, 1), (128, 256, 2), (256, 256, 1),
                         (256, 512, 2), (512, 512, 1)]:
        sx = sc.point(cur)
        cq = O.quantize_i8_static(cur, sx).reshape(cur.shape)
        h1 = _conv(cq, spec.convs[ci], sx, O.ACT_RELU)
        s1 = sc.point(h1)
        h1q = O.quantize_i8_static(h1, s1).reshape(h1.shape)
        h2 = _conv(h1q, spec.convs[ci + 1], s1, O.ACT_NONE)
        ci += 2
        if s != 1 or cin != cout:
            short = _conv(cq, spec.convs[ci], sx, O.ACT_NONE)
            ci += 1
        else:
            short = cur
        cur = _relu((h2 + short).astype(np.float32))
    n, hh, ww, c = cur.shape
    g = O.average_pool2d(np.ascontiguousarray(cur.transpose(0, 3, 1, 2)), n, c, hh, ww, (hh, ww), (1, 1), (0, 0))
    logits = O.matmul(g, (n, 512), spec.fc_w, (512, 1000), threads=TH)
    return O.add_bias_rows(logits, n, 1000, spec.fc_b)


# ------------------------------------------------------------------ BERT-shaped encoder
def _attention(qkv, batch, seq, heads, d, scale):
    """The plan's fused attention, the device's integer tensor-core arithmetic
    (tpto_attention_i8; D = 64)."""
    assert d == 64
    return O.attention_i8(qkv, batch, seq, heads, scale).reshape(batch * seq, heads * d)


def bert(x, layers_w, batch, seq, scales=None, calib=None, heads=12, hidden=768, ffn=3072, eps=1e-5):
    sc = calib if calib is not None else _Scales(scales)
    T = batch * seq
    cur = np.asarray(x, np.float32).reshape(T, hidden)
    for lw in layers_w:
        s = sc.point(cur)
        qkv = O.w8a8_gemm(O.quantize_i8_static(cur, s), lw.qkv.q, T, 3 * hidden, hidden, s, lw.qkv.scales,
                          lw.qkv.bias, O.ACT_NONE, threads=TH)
        ctx = _attention(qkv, batch, seq, heads, hidden // heads, 0.125)
        s = sc.point(ctx)
        o = O.w8a8_gemm(O.quantize_i8_static(ctx, s), lw.o.q, T, hidden, hidden, s, lw.o.scales, lw.o.bias,
                        O.ACT_NONE, threads=TH)
        h1 = O.layernorm((o + cur.ravel()).astype(np.float32), T, hidden, lw.g1, lw.b1, eps)
        s = sc.point(h1)
        f = O.w8a8_gemm(O.quantize_i8_static(h1, s), lw.f1.q, T, ffn, hidden, s, lw.f1.scales, lw.f1.bias,
                        O.ACT_GELU, threads=TH)
        s = sc.point(f)
        f2 = O.w8a8_gemm(O.quantize_i8_static(f, s), lw.f2.q, T, hidden, ffn, s, lw.f2.scales, lw.f2.bias,
                         O.ACT_NONE, threads=TH)
        cur = O.layernorm((f2 + h1).astype(np.float32), T, hidden, lw.g2, lw.b2, eps).reshape(T, hidden)
    return cur.ravel()

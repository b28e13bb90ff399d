"""Device-resident plans for the model workloads, over the C ABI's plan API.

``Plan`` wraps ``tpt_cuda_plan_*`` (the device counterpart of tpt-infer's
``execute_graph``, crates/tpt-infer-runtime/src/exec.rs:570-635). The builders
lay out the three model workloads the way tpt-infer's runtime would execute
them node by node, with the quantized-weight path of tpt-infer-quantize:

- ``mlp``: Gemm 784->512, ReLU, Gemm 512->10, Softmax, in f32 (the reference's
  MatMul/Add/Relu/Softmax nodes) or with INT8 per-output-channel weights and
  calibrated per-tensor activation scales.
- ``resnet18``: a ResNet-18-shaped CNN in NHWC: INT8 convolutions as im2col +
  W8A8 GEMM with fused bias (folded BatchNorm) and ReLU, max pool, residual
  adds, global average pool, f32 Gemm 512->1000.
- ``bert``: a BERT-base-shaped encoder: INT8 Q/K/V/O and FFN projections,
  fused f32 attention, GELU, residual adds, post-LayerNorm.

Weight tensors are synthesised with the seeded generators of ``synth`` and
quantized on the device with the reference's quantizer rules
(quantize_i8_symmetric_per_channel, per output channel = per row of W^T).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np

from . import _capi, synth
from ._capi import lib
from .backend import ACT_GELU, ACT_NONE, ACT_RELU, CudaBackend, OpError

F32, I8 = 0, 1
OP_QUANTIZE, OP_LINEAR, OP_MATMUL, OP_BIAS_ACT, OP_ADD_ACT, OP_SOFTMAX, OP_LAYERNORM, OP_ATTENTION = range(1, 9)
OP_NCHW_Q8, OP_IM2COL, OP_MAXPOOL, OP_GAP = 9, 10, 11, 12
OP_ALLGATHER, OP_PANELS_TO_ROWS, OP_GEMM = 13, 14, 15
OP_BINARY, OP_UNARY, OP_POOL_NCHW, OP_BATCHNORM, OP_TRANSPOSE, OP_CONCAT, OP_CONV2D, OP_BATCHED_MATMUL = range(16, 24)


class Plan:
    """A device-resident execution plan on one CudaBackend context."""

    def __init__(self, be: CudaBackend):
        self.be = be
        h = C.c_void_p()
        be._check(lib.tpt_cuda_plan_create(be.ctx, C.byref(h)))
        self.h = h
        self.weights = []  # keep uploaded weight handles alive
        self.numel = {}
        self.dtype = {}

    def tensor(self, dtype, numel):
        i = C.c_int()
        self.be._check(lib.tpt_cuda_plan_add_tensor(self.h, dtype, int(numel), C.byref(i)))
        self.numel[i.value] = int(numel)
        self.dtype[i.value] = dtype
        return i.value

    def const(self, arr):
        a = np.ascontiguousarray(arr, np.float32).ravel()
        i = C.c_int()
        self.be._check(lib.tpt_cuda_plan_add_const(self.h, a.ctypes.data_as(C.c_void_p), a.size, C.byref(i)))
        self.numel[i.value] = a.size
        self.dtype[i.value] = F32
        return i.value

    def op(self, kind, in0, out, in1=-1, in2=-1, w=None, act=ACT_NONE, f0=0.0, dims=()):
        o = _capi.PlanOp()
        o.kind, o.in0, o.in1, o.in2, o.out = kind, in0, in1, in2, out
        o.w = w.handle if w is not None else None
        o.act, o.f0 = act, f0
        for j, d in enumerate(dims):
            o.dims[j] = int(d)
        self.be._check(lib.tpt_cuda_plan_add_op(self.h, C.byref(o)))

    def set_comm(self, comm):
        """The communicator of the plan's ALLGATHER ops and rank-global scales."""
        self.comm = comm
        self.be._check(lib.tpt_cuda_plan_set_comm(self.h, comm.h))

    def reuse(self, keep):
        """Before finalize: arena offsets by liveness; only ``keep`` can be fetched."""
        ids = list(keep)
        arr = (C.c_int * max(len(ids), 1))(*ids)
        self.be._check(lib.tpt_cuda_plan_reuse_arena(self.h, arr, len(ids)))

    def finalize(self):
        self.be._check(lib.tpt_cuda_plan_finalize(self.h))

    def arena_bytes(self):
        b = C.c_size_t()
        lib.tpt_cuda_plan_arena_bytes(self.h, C.byref(b))
        return b.value

    def ptr(self, tid):
        p = C.c_void_p()
        self.be._check(lib.tpt_cuda_plan_tensor_ptr(self.h, tid, C.byref(p)))
        return p.value

    def calibrate(self, on=True):
        self.be._check(lib.tpt_cuda_plan_set_calibration(self.h, 1 if on else 0))

    def freeze(self):
        self.be._check(lib.tpt_cuda_plan_freeze_scales(self.h))

    def scales(self):
        """Static scales of the quantization points, in op order."""
        n = C.c_size_t()
        lib.tpt_cuda_plan_get_scales(self.h, None, 0, C.byref(n))
        out = np.zeros(n.value, np.float32)
        lib.tpt_cuda_plan_get_scales(self.h, out.ctypes.data_as(C.c_void_p), n.value, C.byref(n))
        return out

    def set_scales(self, scales):
        """Imports static scales (one per quantization point, op order)."""
        a = np.ascontiguousarray(scales, np.float32)
        self.be._check(lib.tpt_cuda_plan_set_scales(self.h, a.ctypes.data_as(C.c_void_p), a.size))

    def set_graph(self, on=True):
        """Replays a recorded launch sequence once scales are frozen (CUDA graph)."""
        self.be._check(lib.tpt_cuda_plan_set_graph(self.h, int(bool(on))))

    def run_device(self):
        self.be._check(lib.tpt_cuda_plan_run_device(self.h))

    def run(self, inputs: dict, outputs: list):
        """H2D of ``inputs`` {tensor id: host array}, the ops, D2H of ``outputs``."""
        ids = list(inputs)
        arrs = [np.ascontiguousarray(inputs[i], np.float32).ravel() for i in ids]
        for i, a in zip(ids, arrs):
            if a.size != self.numel[i]:
                raise OpError(1, self.numel[i], a.size)
        outs = [np.empty(self.numel[o], np.float32) for o in outputs]
        in_ids = (C.c_int * len(ids))(*ids)
        in_p = (C.c_void_p * len(ids))(*[a.ctypes.data for a in arrs])
        out_ids = (C.c_int * len(outputs))(*outputs)
        out_p = (C.c_void_p * len(outputs))(*[a.ctypes.data for a in outs])
        self.be._check(lib.tpt_cuda_plan_run(self.h, in_ids, in_p, len(ids), out_ids, out_p, len(outputs)))
        return outs

    def run_batches(self, in_ids, batches, out_ids, outputs=None):
        """tpt_cuda_plan_run_batches: len(batches) runs, batches[s] = the host inputs
        of step s (one array per id of ``in_ids``); the next step's inputs are
        copied while the current one computes. ``outputs[s][j]`` (preallocated
        f32 arrays, page-locked for overlap) receive the results."""
        n, ni, no = len(batches), len(in_ids), len(out_ids)
        if outputs is None:
            outputs = [[np.empty(self.numel[o], np.float32) for o in out_ids] for _ in range(n)]
        ins = []
        for b in batches:
            for i, a in zip(in_ids, b):
                if a.dtype != np.float32 or not a.flags.c_contiguous or a.size != self.numel[i]:
                    raise OpError(1, self.numel[i], a.size)
                ins.append(a.ctypes.data)
        outs = [o.ctypes.data for row in outputs for o in row]
        self.be._check(lib.tpt_cuda_plan_run_batches(
            self.h, (C.c_int * max(ni, 1))(*in_ids), (C.c_void_p * max(len(ins), 1))(*ins), ni,
            (C.c_int * max(no, 1))(*out_ids), (C.c_void_p * max(len(outs), 1))(*outs), no, n))
        return outputs

    def close(self):
        if self.h:
            lib.tpt_cuda_plan_destroy(self.h)
            self.h = None
        for w in self.weights:
            w.free()
        self.weights = []

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ------------------------------------------------------------------ weights
@dataclass
class QLinear:
    """An INT8 per-output-channel weight: W^T [n, k] quantized row by row."""

    n: int
    k: int
    q: np.ndarray        # int8 [n, k]
    scales: np.ndarray   # f32 [n]
    bias: np.ndarray     # f32 [n]


def make_qlinear(be, n, k, seed, std, bias_std=0.0, kp=None):
    """W ~ N(0, std) with W^T [n, k]; quantize_i8_symmetric_per_channel(W^T, rows=n)
    (crates/tpt-infer-quantize/src/quant.rs:95-107) on the device. kp pads k with
    zero columns."""
    wt = synth.normal(n * k, seed, 0.0, std)
    q, s = be.quantize_i8_symmetric_per_channel(wt, n)
    q = q.reshape(n, k)
    if kp is not None and kp != k:
        qp = np.zeros((n, kp), np.int8)
        qp[:, :k] = q
        q = qp
    b = synth.normal(n, seed + 7919, 0.0, bias_std) if bias_std > 0 else np.zeros(n, np.float32)
    return QLinear(n, q.shape[1], np.ascontiguousarray(q), s, b)


# ------------------------------------------------------------------ MLP
@dataclass
class MlpWeights:
    w1: np.ndarray  # [784, 512]
    b1: np.ndarray
    w2: np.ndarray  # [512, 10]
    b2: np.ndarray


def mlp_weights(seed=10):
    """The MLP workload: W1 ~ N(0, 0.036) [784,512], b1 = 0; W2 ~ N(0, 0.06) [512,10], b2 = 0."""
    return MlpWeights(synth.normal(784 * 512, seed, 0.0, 0.036).reshape(784, 512), np.zeros(512, np.float32),
                      synth.normal(512 * 10, seed + 1, 0.0, 0.06).reshape(512, 10), np.zeros(10, np.float32))


def build_mlp_f32(be, batch, W: MlpWeights, reuse=True):
    p = Plan(be)
    x = p.tensor(F32, batch * 784)
    h = p.tensor(F32, batch * 512)
    z = p.tensor(F32, batch * 10)
    y = p.tensor(F32, batch * 10)
    w1, b1, w2, b2 = p.const(W.w1), p.const(W.b1), p.const(W.w2), p.const(W.b2)
    p.op(OP_MATMUL, x, h, in1=w1, in2=b1, act=ACT_RELU, dims=(batch, 784, 512))
    p.op(OP_MATMUL, h, z, in1=w2, in2=b2, dims=(batch, 512, 10))
    p.op(OP_SOFTMAX, z, y, dims=(batch, 10))
    if reuse:
        p.reuse([x, y, z])
    p.finalize()
    return p, x, y, z


def build_mlp_int8(be, batch, W: MlpWeights, reuse=True):
    """INT8 PTQ variant: W1, W2 per output channel (quantize W^T rows); activations
    per tensor with calibrated static scales."""
    p = Plan(be)
    q1, s1 = be.quantize_i8_symmetric_per_channel(np.ascontiguousarray(W.w1.T), 512)
    q2, s2 = be.quantize_i8_symmetric_per_channel(np.ascontiguousarray(W.w2.T), 10)
    wh1 = be.upload_i8(q1, s1, 512, 784)  # K = 784 and 512 are multiples of 16
    wh2 = be.upload_i8(q2, s2, 10, 512)
    p.weights += [wh1, wh2]
    x = p.tensor(F32, batch * 784)
    xq = p.tensor(I8, batch * 784)
    h = p.tensor(F32, batch * 512)
    hq = p.tensor(I8, batch * 512)
    z = p.tensor(F32, batch * 10)
    y = p.tensor(F32, batch * 10)
    b1, b2 = p.const(W.b1), p.const(W.b2)
    p.op(OP_QUANTIZE, x, xq, dims=(batch * 784,))
    p.op(OP_LINEAR, xq, h, in1=b1, w=wh1, act=ACT_RELU, dims=(batch,))
    p.op(OP_QUANTIZE, h, hq, dims=(batch * 512,))
    p.op(OP_LINEAR, hq, z, in1=b2, w=wh2, dims=(batch,))
    p.op(OP_SOFTMAX, z, y, dims=(batch, 10))
    if reuse:
        p.reuse([x, y, z])
    p.finalize()
    return p, x, y, z, (q1, s1, q2, s2)


# ------------------------------------------------------------------ ResNet-18
def _conv_out(h, k, s, pad):
    return (h + 2 * pad - k) // s + 1


@dataclass
class ConvSpec:
    cin: int
    cout: int
    k: int
    stride: int
    pad: int
    qw: QLinear = None   # W [cout, cin*k*k] per-channel int8, columns in (ky, kx, c) order


@dataclass
class ResNetSpec:
    convs: list = field(default_factory=list)
    fc_w: np.ndarray = None   # [512, 1000]
    fc_b: np.ndarray = None


def resnet18_weights(be, seed=100):
    """He-normal conv weights N(0, sqrt(2/fan_in)) in OIHW, quantized per output
    channel (axis 0 of OIHW, quant.rs:95-107) on the device, then reordered to
    (ky, kx, c) columns for NHWC im2col; BatchNorm folded into a bias ~ N(0, 0.01)."""
    spec = ResNetSpec()
    layers = [(3, 64, 7, 2, 3)]
    cfg = [(64, 64, 1), (64, 64, 1), (64, 128, 2), (128, 128, 1), (128, 256, 2), (256, 256, 1), (256, 512, 2),
           (512, 512, 1)]
    for cin, cout, s in cfg:
        layers.append((cin, cout, 3, s, 1))
        layers.append((cout, cout, 3, 1, 1))
        if s != 1 or cin != cout:
            layers.append((cin, cout, 1, s, 0))
    for i, (cin, cout, k, s, pad) in enumerate(layers):
        fan_in = cin * k * k
        w = synth.normal(cout * fan_in, seed + 17 * i, 0.0, float(np.sqrt(2.0 / fan_in)))  # OIHW
        q, sc = be.quantize_i8_symmetric_per_channel(w, cout)
        q = q.reshape(cout, cin, k, k).transpose(0, 2, 3, 1).reshape(cout, fan_in)  # (ky, kx, c)
        kp = (fan_in + 15) // 16 * 16
        qp = np.zeros((cout, kp), np.int8)
        qp[:, :fan_in] = q
        b = synth.normal(cout, seed + 17 * i + 5, 0.0, 0.01)
        spec.convs.append(ConvSpec(cin, cout, k, s, pad, QLinear(cout, kp, qp, sc, b)))
    spec.fc_w = synth.normal(512 * 1000, seed + 999, 0.0, float(np.sqrt(2.0 / 512))).reshape(512, 1000)
    spec.fc_b = np.zeros(1000, np.float32)
    return spec


def _stem_s2d(cv, cp):
    """The stem's 7x7 stride-2 pad-3 weights as a 4x4 stride-1 pad-2 conv over the
    2x2 space-to-depth input (channels (dy*2 + dx)*cp + c, c padded from cin to cp):
    tap (ty, tx) with sub-pixel (dy, dx) is the original tap (2ty + dy - 1,
    2tx + dx - 1), zero outside the 7x7 window. Output pixel (oy, ox) then reads
    s2d pixels (oy - 2 + ty, ox - 2 + tx): exactly the original window, so every
    int32 sum is unchanged."""
    k = cv.k
    q = cv.qw.q[:, :k * k * cv.cin].reshape(cv.cout, k, k, cv.cin)
    out = np.zeros((cv.cout, 4, 4, 2, 2, cp), np.int8)
    for ty in range(4):
        for dy in range(2):
            ky = 2 * ty + dy - 1
            if not 0 <= ky < k:
                continue
            for tx in range(4):
                for dx in range(2):
                    kx = 2 * tx + dx - 1
                    if 0 <= kx < k:
                        out[:, ty, tx, dy, dx, :cv.cin] = q[:, ky, kx, :]
    return out.reshape(cv.cout, 4 * 4 * 4 * cp)


def build_resnet18(be, batch, spec: ResNetSpec, reuse=True):
    """The stem input is held as 2x2 space-to-depth NHWC of the image padded to 4
    channels ([112, 112, 16]); the 7x7/2 stem runs as the equivalent 4x4/1 conv
    on it, so its gathers move 16-byte pixels. Outputs are unchanged (the same
    integer sums)."""
    assert spec.convs[0].k == 7 and spec.convs[0].stride == 2 and spec.convs[0].pad == 3
    p = Plan(be)
    handles = []
    STEM_C = 4
    cins = []
    for i, cv in enumerate(spec.convs):
        q, cin = cv.qw.q, cv.cin
        if i == 0:
            q, cin = _stem_s2d(cv, STEM_C), 4 * STEM_C
        wh = be.upload_i8(np.ascontiguousarray(q), cv.qw.scales, cv.qw.n, q.shape[1])
        handles.append(wh)
        cins.append(cin)
    p.weights += handles
    x = p.tensor(F32, batch * 3 * 224 * 224)
    xq = p.tensor(I8, batch * 224 * 224 * STEM_C)
    p.op(OP_NCHW_Q8, x, xq, dims=(batch, 3, 224 * 224, STEM_C, 224, 2))

    def conv(inp_q, H, W, ci, act):
        cv = spec.convs[ci]
        OH, OW = _conv_out(H, cv.k, cv.stride, cv.pad), _conv_out(W, cv.k, cv.stride, cv.pad)
        k, s, pad, ih, iw = cv.k, cv.stride, cv.pad, H, W
        if ci == 0:  # the space-to-depth form of the stem
            k, s, pad, ih, iw = 4, 1, 2, H // 2, W // 2
        M = batch * OH * OW
        kp = handles[ci].k
        col = p.tensor(I8, M * kp)
        p.op(OP_IM2COL, inp_q, col, dims=(batch, ih, iw, cins[ci], k, k, s, s, pad, pad, OH, OW, kp))
        out = p.tensor(F32, M * cv.cout)
        p.op(OP_LINEAR, col, out, in1=p.const(cv.qw.bias), w=handles[ci], act=act, dims=(M,))
        return out, OH, OW

    y, H, W = conv(xq, 224, 224, 0, ACT_RELU)                      # stem 7x7/2 -> 112
    OH, OW = _conv_out(H, 3, 2, 1), _conv_out(W, 3, 2, 1)
    mp = p.tensor(F32, batch * OH * OW * 64)
    p.op(OP_MAXPOOL, y, mp, dims=(batch, H, W, 64, 3, 3, 2, 2, 1, 1, OH, OW))
    cur, H, W, C = mp, OH, OW, 64
    ci = 1
    for cin, cout, s in [(64, 64, 1), (64, 64, 1), (64, 128, 2), (128, 128, 1), (128, 256, 2), (256, 256, 1),
                         (256, 512, 2), (512, 512, 1)]:
        cq = p.tensor(I8, batch * H * W * C)
        p.op(OP_QUANTIZE, cur, cq, dims=(batch * H * W * C,))
        h1, OH, OW = conv(cq, H, W, ci, ACT_RELU)
        h1q = p.tensor(I8, batch * OH * OW * cout)
        p.op(OP_QUANTIZE, h1, h1q, dims=(batch * OH * OW * cout,))
        h2, _, _ = conv(h1q, OH, OW, ci + 1, ACT_NONE)
        ci += 2
        if s != 1 or cin != cout:
            sc, _, _ = conv(cq, H, W, ci, ACT_NONE)
            ci += 1
        else:
            sc = cur
        out = p.tensor(F32, batch * OH * OW * cout)
        p.op(OP_ADD_ACT, h2, out, in1=sc, act=ACT_RELU, dims=(batch * OH * OW * cout,))
        cur, H, W, C = out, OH, OW, cout
    g = p.tensor(F32, batch * 512)
    p.op(OP_GAP, cur, g, dims=(batch, H * W, 512))
    logits = p.tensor(F32, batch * 1000)
    p.op(OP_MATMUL, g, logits, in1=p.const(spec.fc_w), in2=p.const(spec.fc_b), dims=(batch, 512, 1000))
    if reuse:
        p.reuse([x, logits])
    p.finalize()
    return p, x, logits


# ------------------------------------------------------------------ BERT-base
@dataclass
class BertLayerW:
    qkv: QLinear   # [2304, 768]
    o: QLinear     # [768, 768]
    f1: QLinear    # [3072, 768]
    f2: QLinear    # [768, 3072]
    g1: np.ndarray
    b1: np.ndarray
    g2: np.ndarray
    b2: np.ndarray


def bert_weights(be, layers=12, seed=5000, hidden=768, ffn=3072):
    """All weights and biases ~ N(0, 0.02); LayerNorm gamma = 1, beta = 0."""
    out = []
    for L in range(layers):
        s = seed + 101 * L
        out.append(BertLayerW(make_qlinear(be, 3 * hidden, hidden, s, 0.02, 0.02),
                              make_qlinear(be, hidden, hidden, s + 1, 0.02, 0.02),
                              make_qlinear(be, ffn, hidden, s + 2, 0.02, 0.02),
                              make_qlinear(be, hidden, ffn, s + 3, 0.02, 0.02),
                              np.ones(hidden, np.float32), np.zeros(hidden, np.float32),
                              np.ones(hidden, np.float32), np.zeros(hidden, np.float32)))
    return out


def build_bert(be, batch, seq, layers_w, heads=12, hidden=768, ffn=3072, eps=1e-5, ffn_shard=None, reuse=True):
    """``ffn_shard`` = a sharding.Comm: FFN1 column-sharded over its ranks and
    reassembled by an all-gather inside the plan (see sharding.py)."""
    from . import sharding

    p = Plan(be)
    if ffn_shard is not None:
        p.set_comm(ffn_shard)
    T = batch * seq
    x = p.tensor(F32, T * hidden)
    cur = x
    for lw in layers_w:
        hs = []
        f1 = lw.f1
        if ffn_shard is not None:
            c0, cn = sharding.column_shard(ffn, ffn_shard.world, ffn_shard.rank)
            f1 = sharding.slice_qlinear(lw.f1, c0, cn)
        for ql in (lw.qkv, lw.o, f1, lw.f2):
            wh = be.upload_i8(ql.q, ql.scales, ql.n, ql.k)
            p.weights.append(wh)
            hs.append(wh)
        xq = p.tensor(I8, T * hidden)
        p.op(OP_QUANTIZE, cur, xq, dims=(T * hidden,))
        qkv = p.tensor(F32, T * 3 * hidden)
        p.op(OP_LINEAR, xq, qkv, in1=p.const(lw.qkv.bias), w=hs[0], dims=(T,))
        ctx = p.tensor(F32, T * hidden)
        p.op(OP_ATTENTION, qkv, ctx, f0=0.125, dims=(batch, seq, heads, hidden // heads))
        cq = p.tensor(I8, T * hidden)
        p.op(OP_QUANTIZE, ctx, cq, dims=(T * hidden,))
        o = p.tensor(F32, T * hidden)
        p.op(OP_LINEAR, cq, o, in1=p.const(lw.o.bias), w=hs[1], dims=(T,))
        r1 = p.tensor(F32, T * hidden)
        p.op(OP_ADD_ACT, o, r1, in1=cur, dims=(T * hidden,))
        h1 = p.tensor(F32, T * hidden)
        p.op(OP_LAYERNORM, r1, h1, in1=p.const(lw.g1), in2=p.const(lw.b1), f0=eps, dims=(T, hidden))
        hq = p.tensor(I8, T * hidden)
        p.op(OP_QUANTIZE, h1, hq, dims=(T * hidden,))
        if ffn_shard is None:
            f = p.tensor(F32, T * ffn)
            p.op(OP_LINEAR, hq, f, in1=p.const(f1.bias), w=hs[2], act=ACT_GELU, dims=(T,))
            fq = p.tensor(I8, T * ffn)
            p.op(OP_QUANTIZE, f, fq, dims=(T * ffn,))
        else:
            P, cn = ffn_shard.world, f1.n
            fs = p.tensor(F32, T * cn)  # this rank's output channels
            p.op(OP_LINEAR, hq, fs, in1=p.const(f1.bias), w=hs[2], act=ACT_GELU, dims=(T,))
            fsq = p.tensor(I8, T * cn)
            p.op(OP_QUANTIZE, fs, fsq, dims=(T * cn, 1))  # scale of the whole [T, ffn] tensor
            g = p.tensor(I8, P * T * cn)
            p.op(OP_ALLGATHER, fsq, g, dims=(T * cn,))
            fq = p.tensor(I8, T * ffn)
            p.op(OP_PANELS_TO_ROWS, g, fq, dims=(P, T, cn))
        f2 = p.tensor(F32, T * hidden)
        p.op(OP_LINEAR, fq, f2, in1=p.const(lw.f2.bias), w=hs[3], dims=(T,))
        r2 = p.tensor(F32, T * hidden)
        p.op(OP_ADD_ACT, f2, r2, in1=h1, dims=(T * hidden,))
        h2 = p.tensor(F32, T * hidden)
        p.op(OP_LAYERNORM, r2, h2, in1=p.const(lw.g2), in2=p.const(lw.b2), f0=eps, dims=(T, hidden))
        cur = h2
    if reuse:
        p.reuse([x, cur])
    p.finalize()
    return p, x, cur

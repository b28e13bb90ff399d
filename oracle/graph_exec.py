"""Oracle execution of a ComputationGraph (TEST INFRASTRUCTURE ONLY).

Restates the reference runtime's walk (crates/tpt-infer-runtime/src/exec.rs:
347-533 dispatch, 570-635 execute_graph) on the oracle's primitives: nodes in
order, initializers bound by name, each operator through the CPU kernel the
reference dispatches it to (naive MatMul/Conv2d, kernels::binary, the
Backend's element ops, pooling, BatchNorm, Concat, Transpose), Reshape and
Flatten as copies. Extension operators of the CUDA lowering (LayerNorm, Gemm,
rank-3/4 MatMul per batch, INT8 weights with per-tensor activation scales) use
the oracle's definitions of the same arithmetic.

It reads the graph by duck typing (``nodes`` with ``op.kind``, ``op.attrs``,
``inputs``, ``dims``, ``name``; ``initializers``; ``outputs``), so it imports
nothing from the CUDA package.
"""
from __future__ import annotations

import numpy as np

from . import oracle as O

_BIN = {"Add": O.BIN_ADD, "Sub": O.BIN_SUB, "Mul": O.BIN_MUL, "Div": O.BIN_DIV}


def _numel(d):
    n = 1
    for x in d:
        n *= int(x)
    return n


def execute_graph(graph, inputs, quantized=None, scales=None, calib=None):
    """Marked outputs of ``graph`` for ``inputs`` (in graph.inputs() order).

    quantized: {initializer name: (q [N, K] int8, scales [N])} for the MatMuls
    that run W8A8; their activation quantization points take ``scales`` (in node
    order) or, with ``calib`` (a list), replay calibration: the point's scale is
    this run's max|x| / 127 and the max is appended to ``calib``."""
    vals = {}
    it = iter(inputs)
    sc = iter(scales) if scales is not None else None
    for node in graph.nodes:
        k, a = node.op.kind, node.op.attrs

        def inp(i):
            return vals[node.inputs[i]], graph.nodes[node.inputs[i]].dims

        if k == "Input":
            if node.name in graph.initializers:
                vals[node.id] = graph.initializers[node.name].data
            else:
                vals[node.id] = np.ascontiguousarray(next(it), np.float32).ravel()
            continue
        if k == "MatMul":
            (x, xd), (w, wd) = inp(0), inp(1)
            if len(xd) == 2 and len(wd) == 2:
                wname = graph.nodes[node.inputs[1]].name
                if quantized is not None and wname in quantized:
                    q, s = quantized[wname]
                    if calib is not None:
                        m = O.absmax(x)
                        calib.append(m)
                        xs = O.sym_scale(m)
                    else:
                        xs = np.float32(next(sc))
                    xq = O.quantize_i8_static(x, xs)
                    y = O.w8a8_gemm(xq, np.ascontiguousarray(q, np.int8), xd[0], wd[1], xd[1], xs, s, None,
                                    O.ACT_NONE, threads=8)
                else:
                    y = O.matmul(x, tuple(xd), w, tuple(wd), threads=8)
            else:
                y = _batched_matmul(x, xd, w, wd, node.dims)
        elif k == "Conv2d":
            (x, xd), (w, wd) = inp(0), inp(1)
            y = O.conv2d(x, tuple(xd), w, tuple(wd), a["strides"], a["padding"], threads=8)
            if len(node.inputs) == 3:
                b, bd = inp(2)
                y = O.binary(O.BIN_ADD, y, node.dims, b, bd, node.dims)
        elif k in _BIN:
            (x, xd), (y2, yd) = inp(0), inp(1)
            y = O.binary(_BIN[k], x, xd, y2, yd, node.dims)
        elif k == "Relu":
            y = O.relu(inp(0)[0])
        elif k == "Sigmoid":
            y = O.sigmoid(inp(0)[0])
        elif k == "Gelu":
            y = O.gelu(inp(0)[0])
        elif k == "Softmax":
            x, xd = inp(0)
            ax = a.get("axis", -1)
            if (ax + len(xd) if ax < 0 else ax) != len(xd) - 1:
                # exec.rs:432-441: the HAL softmax normalizes rows of the last dim only
                raise NotImplementedError("Softmax")
            y = O.softmax(x, xd[-1])
        elif k in ("Reshape", "Flatten"):
            y = np.array(inp(0)[0], np.float32, copy=True)
        elif k == "MaxPool2d":
            x, xd = inp(0)
            y = O.max_pool2d(x, *xd, a["kernel"], a["strides"], a["padding"])
        elif k == "AveragePool2d":
            x, xd = inp(0)
            y = O.average_pool2d(x, *xd, a["kernel"], a["strides"], a["padding"])
        elif k == "BatchNorm":
            x, xd = inp(0)
            y = O.batch_norm(x, xd, *(inp(i)[0] for i in range(1, 5)), a["epsilon"])
        elif k == "Concat":
            y, _ = O.concat([inp(i)[0] for i in range(len(node.inputs))],
                            [graph.nodes[i].dims for i in node.inputs], a["axis"])
        elif k == "Transpose":
            x, xd = inp(0)
            y = O.transpose(x, xd, a["perm"])
        elif k == "LayerNorm":
            x, xd = inp(0)
            y = O.layernorm(x, _numel(xd) // xd[-1], xd[-1], inp(1)[0], inp(2)[0], a["epsilon"])
        elif k == "Gemm":
            (x, xd), (w, wd) = inp(0), inp(1)
            m, kk = (xd[1], xd[0]) if a["trans_a"] else (xd[0], xd[1])
            n = wd[0] if a["trans_b"] else wd[1]
            c = inp(2)[0] if len(node.inputs) == 3 else None
            y = O.gemm(x, m, kk, w, n, c=c, alpha=a["alpha"], beta=a["beta"], trans_a=a["trans_a"],
                       trans_b=a["trans_b"])
        else:
            raise NotImplementedError(k)
        vals[node.id] = np.asarray(y, np.float32).ravel()
    return [vals[o].reshape(graph.nodes[o].dims) for o in graph.outputs]


def _batched_matmul(x, xd, w, wd, od):
    """Per batch index of the broadcast batch dims, the naive MatMul of the slices."""
    bshape = list(od[:-2])
    m, kk, n = xd[-2], xd[-1], wd[-1]
    xa = np.asarray(x, np.float32).reshape(list(xd[:-2]) + [m, kk])
    wb = np.asarray(w, np.float32).reshape(list(wd[:-2]) + [kk, n])
    xa = np.broadcast_to(xa, bshape + [m, kk]).reshape(-1, m, kk)
    wb = np.broadcast_to(wb, bshape + [kk, n]).reshape(-1, kk, n)
    out = np.empty((xa.shape[0], m, n), np.float32)
    for i in range(xa.shape[0]):
        out[i] = O.matmul(np.ascontiguousarray(xa[i]), (m, kk), np.ascontiguousarray(wb[i]), (kk, n)).reshape(m, n)
    return out

"""Graph lowering: a tpt-infer ``ComputationGraph`` onto one device plan.

The reference runtime walks a ``ComputationGraph`` in topological order and
dispatches every node to the ``Backend`` HAL or a runtime kernel
(crates/tpt-infer-runtime/src/exec.rs:347-533, 570-635), with activations in
one arena and initializers bound in place. ``lower`` performs that walk once,
ahead of time: every node becomes plan ops on the CUDA backend
(``tpt_cuda_plan_*``), every initializer a device constant uploaded once, every
non-initializer ``Input`` a graph input, and ``LoweredGraph.run`` is
``execute_graph``: H2D of the inputs, the ops, D2H of the marked outputs.

The IR mirrors the reference's (crates/tpt-infer-graph/src/operator.rs:22-104,
graph.rs): ``Node(id, op, inputs, dims, name)`` with the ``Operator`` variants
and their attributes, named ``Initializer``s, marked outputs. Two extension
operators the BERT workload needs are accepted as well: ``LayerNorm`` (the
reference maps ONNX LayerNormalization to ``Custom``, registry.rs:62) and
``Gemm`` with its ONNX attributes (the reference drops them, registry.rs:21).

Numerics: the f32 path is bit-identical to the reference's CPU backends and
runtime kernels (sequential-k MatMul/Conv, IEEE element ops, the runtime's own
BatchNorm square root). Rank-3/4 MatMul (which the reference runtime rejects,
exec.rs:360-362) runs per batch with the same MatMul arithmetic. With
``quantized`` weights, a rank-2 MatMul whose weight has an INT8 entry runs as
QUANTIZE (a calibrated per-tensor activation scale) + W8A8 GEMM with
per-output-channel weights, the quantized-weight path of this backend.

Errors mirror ``RuntimeError``/``OpError``: an unknown or ``Custom`` operator
raises ``UnsupportedOp`` at lowering time (there is no CPU fallback), a shape
the runtime would reject raises ``OpError`` with its variant's code.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from . import graphs as G
from .backend import OpError

SIZE_MISMATCH, SHAPE_MISMATCH, UNSUPPORTED, INVALID = 1, 2, 3, 4
MAX_RANK = 8  # crates/tpt-infer-core/src/shape.rs:4
# Operator kinds with a CUDA lowering (everything else raises UnsupportedOp)
SUPPORTED = frozenset({"Input", "MatMul", "Conv2d", "Add", "Sub", "Mul", "Div", "Relu", "Sigmoid", "Gelu", "Softmax",
                       "Reshape", "Flatten", "MaxPool2d", "AveragePool2d", "BatchNorm", "Concat", "Transpose",
                       "LayerNorm", "Gemm"})


class UnsupportedOp(OpError):
    """RuntimeError::UnsupportedOp / UnsupportedCustom: no CUDA lowering for the node."""

    def __init__(self, name):
        super().__init__(UNSUPPORTED)
        self.name = name
        self.args = (f"unsupported operator {name!r} on the CUDA backend",)


class NoOutputs(OpError):
    """RuntimeError::NoOutputs (exec.rs:833-846): the graph marks no output."""

    def __init__(self):
        super().__init__(INVALID)
        self.args = ("the graph has no marked output",)


# ------------------------------------------------------------------ IR
@dataclass
class Operator:
    """One variant of the reference's ``Operator`` enum (operator.rs:22-104):
    ``kind`` is the variant name, ``attrs`` its payload."""

    kind: str
    attrs: dict = field(default_factory=dict)

    # constructors named like the reference's (operator.rs:106-...)
    @staticmethod
    def input():
        return Operator("Input")

    @staticmethod
    def matmul():
        return Operator("MatMul")

    @staticmethod
    def conv2d(strides=(1, 1), padding=(0, 0)):
        return Operator("Conv2d", {"strides": tuple(strides), "padding": tuple(padding)})

    @staticmethod
    def softmax(axis=-1):
        return Operator("Softmax", {"axis": int(axis)})

    @staticmethod
    def reshape(shape):
        return Operator("Reshape", {"shape": tuple(shape)})

    @staticmethod
    def flatten(axis=1):
        return Operator("Flatten", {"axis": int(axis)})

    @staticmethod
    def max_pool2d(kernel, strides, padding):
        return Operator("MaxPool2d", {"kernel": tuple(kernel), "strides": tuple(strides), "padding": tuple(padding)})

    @staticmethod
    def average_pool2d(kernel, strides, padding):
        return Operator("AveragePool2d",
                        {"kernel": tuple(kernel), "strides": tuple(strides), "padding": tuple(padding)})

    @staticmethod
    def batch_norm(epsilon=1e-5):
        return Operator("BatchNorm", {"epsilon": float(epsilon)})

    @staticmethod
    def concat(axis):
        return Operator("Concat", {"axis": int(axis)})

    @staticmethod
    def transpose(perm):
        return Operator("Transpose", {"perm": tuple(perm)})

    @staticmethod
    def layer_norm(epsilon=1e-5):
        return Operator("LayerNorm", {"epsilon": float(epsilon)})

    @staticmethod
    def gemm(alpha=1.0, beta=1.0, trans_a=False, trans_b=False):
        return Operator("Gemm", {"alpha": float(alpha), "beta": float(beta), "trans_a": bool(trans_a),
                                 "trans_b": bool(trans_b)})

    @staticmethod
    def custom(name):
        return Operator("Custom", {"name": str(name)})

    @property
    def name(self):
        return self.attrs.get("name", self.kind) if self.kind == "Custom" else self.kind


for _k in ("Add", "Sub", "Mul", "Div", "Relu", "Sigmoid", "Gelu"):
    setattr(Operator, _k.lower(), staticmethod(lambda _k=_k: Operator(_k)))


@dataclass
class Node:
    """graph.rs Node: id, operator, input node ids (ports), output dims, name."""

    id: int
    op: Operator
    inputs: list
    dims: tuple
    name: str = ""


@dataclass
class Initializer:
    name: str
    dims: tuple
    data: np.ndarray


class ComputationGraph:
    """The reference's ComputationGraph (crates/tpt-infer-graph/src/graph.rs):
    nodes in topological order (a node's inputs are earlier nodes), named
    initializers bound to same-named Input nodes, marked outputs."""

    def __init__(self):
        self.nodes: list[Node] = []
        self.initializers: dict[str, Initializer] = {}
        self.outputs: list[int] = []

    def add_node(self, op, inputs, dims, name=""):
        nid = len(self.nodes)
        if len(dims) > MAX_RANK:
            raise OpError(INVALID)  # GraphError::RankTooLarge (graph.rs:538-542)
        for i in inputs:
            if not 0 <= i < nid:
                raise OpError(INVALID)  # GraphError: inputs must precede the node
        self.nodes.append(Node(nid, op, list(inputs), tuple(int(d) for d in dims), name))
        return nid

    def add_input(self, dims, name):
        return self.add_node(Operator.input(), [], dims, name)

    def add_initializer(self, name, dims, data):
        data = np.ascontiguousarray(data, np.float32).ravel()
        if data.size != int(np.prod(dims, dtype=np.int64)):
            raise OpError(SIZE_MISMATCH, int(np.prod(dims, dtype=np.int64)), data.size)
        self.initializers[name] = Initializer(name, tuple(int(d) for d in dims), data)

    def add_weight(self, name, dims, data):
        """An Input node bound to a same-named initializer."""
        nid = self.add_input(dims, name)
        self.add_initializer(name, dims, data)
        return nid

    def mark_output(self, nid):
        """Marks a graph output; marking a node twice keeps one entry
        (graph.rs:392-400)."""
        if not 0 <= nid < len(self.nodes):
            raise OpError(INVALID)
        if nid not in self.outputs:
            self.outputs.append(nid)

    def inputs(self):
        """Input nodes not bound to an initializer, in node order (execute_graph's binding order)."""
        return [n.id for n in self.nodes if n.op.kind == "Input" and n.name not in self.initializers]


# ------------------------------------------------------------------ lowering
def _numel(dims):
    n = 1
    for d in dims:
        n *= int(d)
    return n


def _pad(dims, rank=MAX_RANK):
    if len(dims) > rank:
        raise OpError(SHAPE_MISMATCH)
    return [1] * (rank - len(dims)) + [int(d) for d in dims]


def _bcast_mask(op_dims, out_dims, rank=MAX_RANK):
    """check_broadcast (kernels.rs:43-58) and the mask of the padded dims where the
    operand is 1 (map_coord, kernels.rs:60-66)."""
    if len(op_dims) > len(out_dims):
        raise OpError(SHAPE_MISMATCH)
    off = len(out_dims) - len(op_dims)
    for i, d in enumerate(op_dims):
        if d != 1 and d != out_dims[off + i]:
            raise OpError(SHAPE_MISMATCH)
    p = _pad(op_dims, rank)
    return sum(1 << i for i in range(rank) if p[i] == 1)


_UNARY = {"Relu": 1, "Sigmoid": 2, "Gelu": 3}
_BINARY = {"Add": 0, "Sub": 1, "Mul": 2, "Div": 3}


class LoweredGraph:
    """A ComputationGraph lowered onto one device plan; ``run`` is execute_graph."""

    def __init__(self, plan, in_ids, in_dims, out_ids, out_dims):
        self.plan = plan
        self.in_ids, self.in_dims = in_ids, in_dims
        self.out_ids, self.out_dims = out_ids, out_dims

    def run(self, inputs):
        """inputs in ComputationGraph.inputs() order -> one array per marked output
        (execute_graph, exec.rs:570-635)."""
        if len(inputs) != len(self.in_ids):
            raise OpError(INVALID)
        feed = {}
        for tid, dims, x in zip(self.in_ids, self.in_dims, inputs):
            x = np.ascontiguousarray(x, np.float32).ravel()
            if x.size != _numel(dims):
                raise OpError(SIZE_MISMATCH, _numel(dims), x.size)
            feed[tid] = x
        outs = self.plan.run(feed, list(dict.fromkeys(self.out_ids)))
        by_id = dict(zip(dict.fromkeys(self.out_ids), outs))
        return [by_id[t].reshape(d) for t, d in zip(self.out_ids, self.out_dims)]

    def calibrate(self, batches):
        """Calibration runs for the quantization points (INT8 weights): each batch is
        a list of inputs; the scales freeze at the running max|x| / 127."""
        self.plan.calibrate(True)
        for b in batches:
            self.run(b)
        self.plan.freeze()

    def close(self):
        self.plan.close()


def lower(graph: ComputationGraph, be, quantized=None) -> LoweredGraph:
    """Lowers ``graph`` onto a plan of the CUDA backend ``be``.

    ``quantized``: None (f32 everywhere), "all" (every rank-2 MatMul whose weight
    is an initializer [K, N] with K % 16 == 0 gets INT8 per-output-channel
    weights, quantized on the device with quantize_i8_symmetric_per_channel of
    W^T, quant.rs:95-107), or a dict {initializer name: (q int8 [N, K], scales
    [N])} of already quantized weights in that layout.
    """
    # graph-level errors before any device work: no marked output, and a node
    # kind with no CUDA lowering (UnsupportedCustom for custom ops, as the
    # reference's dispatch reports them, exec.rs:527-531)
    if not graph.outputs:
        raise NoOutputs()
    for node in graph.nodes:
        if node.op.kind not in SUPPORTED:
            raise UnsupportedOp(node.op.name)
    p = G.Plan(be)
    tid = {}     # node id -> plan tensor id
    in_ids, in_dims = [], []
    consts = {}  # initializer name -> plan tensor id

    def const(name):
        if name not in consts:
            consts[name] = p.const(graph.initializers[name].data)
        return consts[name]

    def port(node, i):
        src = graph.nodes[node.inputs[i]]
        return tid[src.id], src.dims

    def is_init(node, i):
        src = graph.nodes[node.inputs[i]]
        return src.op.kind == "Input" and src.name in graph.initializers

    def out_tensor(node):
        t = p.tensor(G.F32, _numel(node.dims))
        tid[node.id] = t
        return t

    try:
        for node in graph.nodes:
            _lower_node(graph, node, p, tid, in_ids, in_dims, const, port, is_init, out_tensor, be, quantized)
        p.reuse(list(dict.fromkeys(in_ids + [tid[o] for o in graph.outputs])))
        p.finalize()
    except Exception:
        p.close()
        raise
    out_ids = [tid[o] for o in graph.outputs]
    out_dims = [graph.nodes[o].dims for o in graph.outputs]
    return LoweredGraph(p, in_ids, in_dims, out_ids, out_dims)


def _lower_node(graph, node, p, tid, in_ids, in_dims, const, port, is_init, out_tensor, be, quantized):
    """One step of the dispatch table (exec.rs:347-533), emitted as plan ops."""
    k = node.op.kind
    a = node.op.attrs
    if k == "Input":
        if node.name in graph.initializers:
            init = graph.initializers[node.name]
            if _numel(init.dims) != _numel(node.dims):
                raise OpError(SIZE_MISMATCH, _numel(node.dims), _numel(init.dims))
            tid[node.id] = const(node.name)
        else:
            t = out_tensor(node)
            in_ids.append(t)
            in_dims.append(node.dims)
        return
    if k == "MatMul":
        if len(node.inputs) != 2:
            raise OpError(INVALID)
        (ta, ad), (tb, bd) = port(node, 0), port(node, 1)
        if len(ad) == 2 and len(bd) == 2:
            m, kk, kb, n = ad[0], ad[1], bd[0], bd[1]
            if kk != kb:
                raise OpError(SHAPE_MISMATCH)  # validate_matmul (backend.rs:149-183)
            if tuple(node.dims) != (m, n):
                raise OpError(SIZE_MISMATCH, m * n, _numel(node.dims))
            wname = graph.nodes[node.inputs[1]].name if is_init(node, 1) else None
            q = None
            if wname is not None and isinstance(quantized, dict):
                q = quantized.get(wname)
            elif wname is not None and quantized == "all" and kk % 16 == 0:
                w = graph.initializers[wname].data.reshape(kk, n)
                q = be.quantize_i8_symmetric_per_channel(np.ascontiguousarray(w.T), n)
            if q is not None:
                qw, qs = q
                wh = be.upload_i8(np.ascontiguousarray(qw, np.int8).reshape(n, kk), qs, n, kk)
                p.weights.append(wh)
                xq = p.tensor(G.I8, m * kk)
                p.op(G.OP_QUANTIZE, ta, xq, dims=(m * kk,))
                p.op(G.OP_LINEAR, xq, out_tensor(node), w=wh, dims=(m,))
            else:
                p.op(G.OP_MATMUL, ta, out_tensor(node), in1=tb, dims=(m, kk, n))
            return
        if len(ad) < 2 or len(bd) < 2 or len(ad) > 8 or len(bd) > 8:
            raise UnsupportedOp("MatMul")
        m, kk, kb, n = ad[-2], ad[-1], bd[-2], bd[-1]
        if kk != kb:
            raise OpError(SHAPE_MISMATCH)
        bshape = list(node.dims[:-2])
        if len(bshape) > 6 or tuple(node.dims[-2:]) != (m, n):
            raise OpError(SHAPE_MISMATCH)
        am, bm = _bcast_mask(ad[:-2], bshape, 6), _bcast_mask(bd[:-2], bshape, 6)
        p.op(G.OP_BATCHED_MATMUL, ta, out_tensor(node), in1=tb, dims=(*_pad(bshape, 6), am, bm, m, kk, n))
        return
    if k == "Conv2d":
        if len(node.inputs) not in (2, 3):
            raise OpError(INVALID)
        (tx, xd), (tw, wd) = port(node, 0), port(node, 1)
        if len(xd) != 4 or len(wd) != 4:
            raise OpError(SHAPE_MISMATCH)
        (sh, sw), (ph, pw) = a["strides"], a["padding"]
        if xd[1] != wd[1] or sh == 0 or sw == 0:
            raise OpError(SHAPE_MISMATCH if xd[1] != wd[1] else INVALID)  # validate_conv2d (backend.rs:219-284)
        oh, ow = (xd[2] + 2 * ph - wd[2]) // sh + 1, (xd[3] + 2 * pw - wd[3]) // sw + 1
        if tuple(node.dims) != (xd[0], wd[0], oh, ow):
            raise OpError(SIZE_MISMATCH, xd[0] * wd[0] * oh * ow, _numel(node.dims))
        y = p.tensor(G.F32, _numel(node.dims))
        p.op(G.OP_CONV2D, tx, y, in1=tw, dims=(*xd, wd[0], wd[2], wd[3], sh, sw, ph, pw))
        if len(node.inputs) == 3:  # exec.rs:388-391: out += bias, broadcast
            tbias, bdims = port(node, 2)
            mask = _bcast_mask(bdims, node.dims)
            out = out_tensor(node)
            p.op(G.OP_BINARY, y, out, in1=tbias, act=0, dims=(*_pad(node.dims), 0, mask))
        else:
            tid[node.id] = y
        return
    if k in _BINARY:
        if len(node.inputs) != 2:
            raise OpError(INVALID)
        (t0, d0), (t1, d1) = port(node, 0), port(node, 1)
        m0, m1 = _bcast_mask(d0, node.dims), _bcast_mask(d1, node.dims)
        p.op(G.OP_BINARY, t0, out_tensor(node), in1=t1, act=_BINARY[k], dims=(*_pad(node.dims), m0, m1))
        return
    if k in _UNARY:
        t0, d0 = port(node, 0)
        if _numel(d0) != _numel(node.dims):
            raise OpError(SIZE_MISMATCH, _numel(d0), _numel(node.dims))
        p.op(G.OP_UNARY, t0, out_tensor(node), act=_UNARY[k], dims=(_numel(d0),))
        return
    if k == "Softmax":
        t0, d0 = port(node, 0)
        if not d0:
            raise OpError(SHAPE_MISMATCH)
        ax = a["axis"] + len(d0) if a["axis"] < 0 else a["axis"]
        if ax != len(d0) - 1:
            raise UnsupportedOp("Softmax")  # the HAL softmax normalizes rows of the last dim only
        p.op(G.OP_SOFTMAX, t0, out_tensor(node), dims=(_numel(d0) // d0[-1], d0[-1]))
        return
    if k in ("Reshape", "Flatten"):  # a view: the same device tensor (copy_elements, exec.rs:448-451)
        t0, d0 = port(node, 0)
        if _numel(d0) != _numel(node.dims):
            raise OpError(SIZE_MISMATCH, _numel(node.dims), _numel(d0))
        tid[node.id] = t0
        return
    if k in ("MaxPool2d", "AveragePool2d"):
        t0, d0 = port(node, 0)
        (kh, kw), (sh, sw), (ph, pw) = a["kernel"], a["strides"], a["padding"]
        if len(d0) != 4 or len(node.dims) != 4 or kh == 0 or kw == 0 or sh == 0 or sw == 0:
            raise OpError(SHAPE_MISMATCH)
        n_, c_, h_, w_ = d0
        oh, ow = node.dims[2], node.dims[3]
        if node.dims[:2] != (n_, c_) or h_ + 2 * ph < kh or w_ + 2 * pw < kw or \
                oh != (h_ + 2 * ph - kh) // sh + 1 or ow != (w_ + 2 * pw - kw) // sw + 1:
            raise OpError(SHAPE_MISMATCH)  # pool_geometry (kernels.rs:198-260)
        p.op(G.OP_POOL_NCHW, t0, out_tensor(node), act=int(k == "AveragePool2d"),
             dims=(n_, c_, h_, w_, kh, kw, sh, sw, ph, pw, oh, ow))
        return
    _lower_node2(graph, node, p, tid, const, port, is_init, out_tensor)


def _lower_node2(graph, node, p, tid, const, port, is_init, out_tensor):
    k = node.op.kind
    a = node.op.attrs
    if k == "BatchNorm":
        if len(node.inputs) != 5:
            raise OpError(INVALID)
        t0, d0 = port(node, 0)
        if not all(is_init(node, i) for i in range(1, 5)):
            raise UnsupportedOp("BatchNorm")  # parameters must be initializers (packed into one constant)
        prm = [graph.initializers[graph.nodes[node.inputs[i]].name].data for i in range(1, 5)]
        plen = prm[0].size
        if any(v.size != plen for v in prm):
            raise OpError(SHAPE_MISMATCH)
        n = _numel(d0)
        channel = len(d0) == 4 and plen == d0[1]
        if not channel and plen != n:
            raise OpError(SHAPE_MISMATCH)  # kernels.rs:448-452
        packed = p.const(np.concatenate(prm).astype(np.float32))
        p.op(G.OP_BATCHNORM, t0, out_tensor(node), in1=packed, f0=a["epsilon"],
             dims=(n, plen, int(channel), d0[2] * d0[3] if channel else 0))
        return
    if k == "Concat":
        if len(node.inputs) < 2:
            raise OpError(INVALID)
        od = node.dims
        rank = len(od)
        if rank == 0:
            raise OpError(SHAPE_MISMATCH)
        ax = a["axis"] + rank if a["axis"] < 0 else a["axis"]
        if not 0 <= ax < rank:
            raise OpError(SHAPE_MISMATCH)
        inner = _numel(od[ax + 1:])
        out = out_tensor(node)
        off = 0
        for i in range(len(node.inputs)):
            ti, di = port(node, i)
            if len(di) != rank or any(d != ax and v != od[d] for d, v in enumerate(di)):
                raise OpError(SHAPE_MISMATCH)
            if di[ax] == 0 or inner == 0 or off + di[ax] > od[ax]:
                raise OpError(SHAPE_MISMATCH)
            outer = _numel(di) // (di[ax] * inner)
            p.op(G.OP_CONCAT, ti, out, dims=(outer, di[ax] * inner, od[ax] * inner, off * inner))
            off += di[ax]
        if off != od[ax]:
            raise OpError(SHAPE_MISMATCH)
        return
    if k == "Transpose":
        t0, d0 = port(node, 0)
        perm = list(a["perm"])
        rank = len(d0)
        if len(perm) != rank or sorted(perm) != list(range(rank)) or rank > MAX_RANK or \
                tuple(node.dims) != tuple(d0[i] for i in perm):
            raise OpError(SHAPE_MISMATCH)
        lead = MAX_RANK - rank
        pperm = list(range(lead)) + [lead + i for i in perm]
        p.op(G.OP_TRANSPOSE, t0, out_tensor(node), dims=(*_pad(d0), *pperm))
        return
    if k == "LayerNorm":
        if len(node.inputs) != 3:
            raise OpError(INVALID)
        (t0, d0), (tg, dg), (tb, db) = port(node, 0), port(node, 1), port(node, 2)
        cols = d0[-1]
        if _numel(dg) != cols or _numel(db) != cols:
            raise OpError(SHAPE_MISMATCH)
        p.op(G.OP_LAYERNORM, t0, out_tensor(node), in1=tg, in2=tb, f0=a["epsilon"], dims=(_numel(d0) // cols, cols))
        return
    if k == "Gemm":
        if len(node.inputs) not in (2, 3):
            raise OpError(INVALID)
        (ta, ad), (tb, bd) = port(node, 0), port(node, 1)
        if len(ad) != 2 or len(bd) != 2:
            raise OpError(SHAPE_MISMATCH)
        m, kk = (ad[1], ad[0]) if a["trans_a"] else (ad[0], ad[1])
        kb, n = (bd[1], bd[0]) if a["trans_b"] else (bd[0], bd[1])
        if kk != kb or tuple(node.dims) != (m, n):
            raise OpError(SHAPE_MISMATCH)
        tc = -1
        if len(node.inputs) == 3:
            src = graph.nodes[node.inputs[2]]
            cdims = src.dims
            if _numel(cdims) not in (n, m * n):
                raise OpError(SHAPE_MISMATCH)
            if is_init(node, 2):  # beta * C rounded once, as the Gemm epilogue does per element
                c = graph.initializers[src.name].data
                tc = p.const((np.float32(a["beta"]) * c).astype(np.float32))
            elif a["beta"] == 1.0:
                tc = tid[src.id]
            else:
                raise UnsupportedOp("Gemm")  # a computed C with beta != 1
        p.op(G.OP_GEMM, ta, out_tensor(node), in1=tb, in2=tc, f0=a["alpha"],
             dims=(m, kk, n, int(a["trans_a"]), int(a["trans_b"])))
        return
    raise UnsupportedOp(node.op.name)  # Custom / anything else (exec.rs:527-531)

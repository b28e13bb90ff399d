"""ONNX models as ComputationGraphs: a loader (and a small writer) for the
lowering to the CUDA backend.

No ONNX package exists in this image, so the protobuf wire format is decoded
here directly (varints, length-delimited fields, fixed32/64). Only the fields
the reference's loader reads are kept (crates/tpt-infer-onnx/src/load.rs:161-
523): ModelProto.graph / opset_import, GraphProto node / initializer / input /
output / value_info, NodeProto input / output / name / op_type / attribute,
AttributeProto f / i / s / floats / ints, TensorProto dims / data_type /
float_data / int64_data / raw_data, and the tensor shapes of ValueInfoProto.

The graph is built the way ``graph_from_proto`` builds it (load.rs:161-398):
runtime inputs first (graph inputs that are not initializers, dims from the
value infos, ``[1]`` when unknown), then one Input node per initializer (its
data bound under its name), then the nodes in file order with the operator of
registry.rs:17-80 and the attributes of ``build_operator`` (load.rs:400-523):
``kernel_shape``/``strides``/``pads`` (begin values), ``auto_pad`` SAME_* as
symmetric same padding, GlobalAveragePool as an average pool over the whole
map, the Reshape target from its int64 shape initializer. Output dims come from
the value infos, else from shape inference. Graph outputs are marked by name.

Differences, each because the CUDA backend has the op: ``Gemm`` keeps its
transA/transB/alpha/beta attributes and its C input (the reference drops them,
registry.rs:21), ``LayerNormalization`` becomes the LayerNorm extension
operator (the reference: Custom, registry.rs:62), and Identity/Dropout become
views of their input (the reference: Input nodes, which its runtime cannot
dispatch).
"""
from __future__ import annotations

import struct

import numpy as np

from .lowering import ComputationGraph, Operator

MAX_SUPPORTED_OPSET = 17  # load.rs:92-96


class OnnxError(Exception):
    """OnnxError (load.rs:26-36): Decode / InvalidModel."""


# ------------------------------------------------------------------ wire format
def _varint(b, i):
    r = s = 0
    while True:
        if i >= len(b):
            raise OnnxError("protobuf decode error: truncated varint")
        c = b[i]
        i += 1
        r |= (c & 0x7F) << s
        if c < 0x80:
            return r, i
        s += 7
        if s > 70:
            raise OnnxError("protobuf decode error: varint too long")


def _fields(b):
    """(field number, wire type, value) of one message; value is an int for
    varint / fixed fields and a memoryview for length-delimited ones."""
    i, n = 0, len(b)
    while i < n:
        key, i = _varint(b, i)
        f, wt = key >> 3, key & 7
        if wt == 0:
            v, i = _varint(b, i)
        elif wt == 1:
            if i + 8 > n:
                raise OnnxError("protobuf decode error: truncated fixed64")
            v = int.from_bytes(b[i:i + 8], "little")
            i += 8
        elif wt == 2:
            ln, i = _varint(b, i)
            if i + ln > n:
                raise OnnxError("protobuf decode error: truncated field")
            v = b[i:i + ln]
            i += ln
        elif wt == 5:
            if i + 4 > n:
                raise OnnxError("protobuf decode error: truncated fixed32")
            v = int.from_bytes(b[i:i + 4], "little")
            i += 4
        else:
            raise OnnxError(f"protobuf decode error: wire type {wt}")
        yield f, wt, v


def _sint64(v):
    return v - (1 << 64) if v >= 1 << 63 else v


def _ints(wt, v):
    """A repeated int64 field: one varint, or a packed run."""
    if wt == 0:
        return [_sint64(v)]
    out, i = [], 0
    while i < len(v):
        x, i = _varint(v, i)
        out.append(_sint64(x))
    return out


def _floats(wt, v):
    if wt == 5:
        return [struct.unpack("<f", v.to_bytes(4, "little"))[0]]
    return list(np.frombuffer(bytes(v), "<f4"))


def _str(v):
    return bytes(v).decode("utf-8", "replace")


# ------------------------------------------------------------------ messages
def _tensor(b):
    t = {"dims": [], "data_type": 0, "float_data": [], "int64_data": [], "name": "", "raw": None}
    for f, wt, v in _fields(b):
        if f == 1:
            t["dims"] += _ints(wt, v)
        elif f == 2:
            t["data_type"] = v
        elif f == 4:
            t["float_data"] += _floats(wt, v)
        elif f == 7:
            t["int64_data"] += _ints(wt, v)
        elif f == 8:
            t["name"] = _str(v)
        elif f == 9:
            t["raw"] = bytes(v)
    return t


def _attribute(b):
    a = {"name": "", "f": None, "i": None, "s": None, "floats": [], "ints": [], "t": None}
    for f, wt, v in _fields(b):
        if f == 1:
            a["name"] = _str(v)
        elif f == 2:
            a["f"] = struct.unpack("<f", v.to_bytes(4, "little"))[0]
        elif f == 3:
            a["i"] = _sint64(v)
        elif f == 4:
            a["s"] = _str(v)
        elif f == 5:
            a["t"] = _tensor(v)
        elif f == 7:
            a["floats"] += _floats(wt, v)
        elif f == 8:
            a["ints"] += _ints(wt, v)
    return a


def _node(b):
    n = {"input": [], "output": [], "name": "", "op_type": "", "attribute": []}
    for f, wt, v in _fields(b):
        if f == 1:
            n["input"].append(_str(v))
        elif f == 2:
            n["output"].append(_str(v))
        elif f == 3:
            n["name"] = _str(v)
        elif f == 4:
            n["op_type"] = _str(v)
        elif f == 5:
            n["attribute"].append(_attribute(v))
    return n


def _value_info(b):
    """(name, dims or None): the dims of a tensor type with a shape, a dim
    without a positive value (symbolic, unset or <= 0: a dynamic dim) as 0,
    as vi_dims does (load.rs:562-579); None without a tensor shape."""
    name, dims = "", None
    for f, _, v in _fields(b):
        if f == 1:
            name = _str(v)
        elif f == 2:
            for f2, _, v2 in _fields(v):
                if f2 != 1:
                    continue
                for f3, _, v3 in _fields(v2):
                    if f3 != 2:
                        continue
                    ds = []
                    for f4, _, v4 in _fields(v3):
                        if f4 == 1:
                            val = None
                            for f5, _, v5 in _fields(v4):
                                if f5 == 1:
                                    val = _sint64(v5)
                            ds.append(val)
                    dims = [int(d) if d is not None and d > 0 else 0 for d in ds]
    return name, dims


def _graph(b):
    g = {"node": [], "initializer": [], "input": [], "output": [], "value_info": []}
    for f, _, v in _fields(b):
        if f == 1:
            g["node"].append(_node(v))
        elif f == 5:
            g["initializer"].append(_tensor(v))
        elif f == 11:
            g["input"].append(_value_info(v))
        elif f == 12:
            g["output"].append(_value_info(v))
        elif f == 13:
            g["value_info"].append(_value_info(v))
    return g


def _tensor_f32(t):
    """tensor_f32 / tensor_i64 (load.rs:581-620): FLOAT (1) from float_data or raw
    little-endian bytes, INT64 (7) converted to f32; None for other types."""
    if t["data_type"] == 1:
        if t["raw"] is not None:
            return np.frombuffer(t["raw"], "<f4").astype(np.float32)
        return np.asarray(t["float_data"], np.float32)
    if t["data_type"] == 7:
        if t["raw"] is not None:
            return np.frombuffer(t["raw"], "<i8").astype(np.float32)
        return np.asarray(t["int64_data"], np.int64).astype(np.float32)
    return None


def _tensor_i64(t):
    if t["data_type"] != 7:
        return None
    if t["raw"] is not None:
        return [int(v) for v in np.frombuffer(t["raw"], "<i8")]
    return list(t["int64_data"])


def _same_padding(inp, k, s):
    """load.rs:545-550: symmetric padding that keeps ceil(input / stride) outputs."""
    out = -(-inp // s)
    total = max((out - 1) * s + k - inp, 0)
    return total // 2


def _build_operator(node, inits):
    """registry.rs:17-80 plus build_operator's attributes (load.rs:400-523)."""
    at = {a["name"]: a for a in node["attribute"]}
    op = node["op_type"]

    def ints(name, default):
        a = at.get(name)
        return list(a["ints"]) if a is not None and a["ints"] else list(default)

    def one_i(name, default):
        a = at.get(name)
        return a["i"] if a is not None and a["i"] is not None else default

    def one_f(name, default):
        a = at.get(name)
        return a["f"] if a is not None and a["f"] is not None else default

    strides = ints("strides", [1, 1])[:2]
    pads = ints("pads", [0, 0, 0, 0])[:2]
    kernel = ints("kernel_shape", [0, 0])[:2]
    if op in ("Identity", "Dropout"):
        return Operator("Reshape", {"shape": (), "view": True})
    if op == "MatMul":
        return Operator.matmul()
    if op == "Gemm":
        return Operator.gemm(one_f("alpha", 1.0), one_f("beta", 1.0), bool(one_i("transA", 0)),
                             bool(one_i("transB", 0)))
    if op in ("Add", "Sub", "Mul", "Div", "Relu", "Sigmoid"):
        return Operator(op)
    if op in ("Gelu", "Erf"):
        return Operator("Gelu")
    if op == "Softmax":
        return Operator.softmax(one_i("axis", -1))
    if op == "Flatten":
        return Operator.flatten(one_i("axis", 1))
    if op == "Concat":
        return Operator.concat(one_i("axis", 1))
    if op == "Transpose":
        return Operator.transpose(ints("perm", []))
    if op == "Reshape":
        shape = ints("shape", [])
        if not shape and len(node["input"]) > 1 and node["input"][1] in inits:
            shape = _tensor_i64(inits[node["input"][1]]) or []
        return Operator.reshape(shape)
    if op == "Conv":
        return Operator.conv2d(strides, pads)
    if op == "MaxPool":
        return Operator.max_pool2d(kernel, strides, pads)
    if op == "AveragePool":
        return Operator.average_pool2d(kernel, strides, pads)
    if op == "GlobalAveragePool":
        return Operator.average_pool2d([0, 0], [1, 1], [0, 0])
    if op == "BatchNormalization":
        return Operator.batch_norm(one_f("epsilon", 1e-5))
    if op == "LayerNormalization":
        return Operator.layer_norm(one_f("epsilon", 1e-5))
    return Operator.custom(op)


def _bcast(a, b):
    r = max(len(a), len(b))
    a = [1] * (r - len(a)) + list(a)
    b = [1] * (r - len(b)) + list(b)
    return [max(x, y) if 1 in (x, y) else x for x, y in zip(a, b)]


def _out_dim(inp, pad, kernel, stride):
    """conv_out_dim (shapes.rs:199-217): (input + 2 pad - kernel) / stride + 1
    with the stride taken as at least 1; a kernel that does not fit the padded
    input is InvalidGeometry, which the loader reports as an invalid model
    (load.rs:77-81)."""
    num = inp + 2 * pad - kernel
    if num < 0:
        raise OnnxError("invalid model: shape inference failed: convolution/pooling kernel does not fit the "
                        "(padded) input dimensions")
    return num // max(stride, 1) + 1


def _infer(op, ins):
    """Output dims of a node without a declared shape (the cases of
    crates/tpt-infer-onnx/src/shapes.rs the lowering supports); [1] otherwise."""
    k, a = op.kind, op.attrs
    if not ins:
        return [1]
    x = list(ins[0])
    if k in ("Relu", "Sigmoid", "Gelu", "Softmax", "BatchNorm", "LayerNorm"):
        return x
    if k in ("Add", "Sub", "Mul", "Div") and len(ins) > 1:
        return _bcast(ins[0], ins[1])
    if k == "MatMul" and len(ins) > 1 and len(x) >= 2 and len(ins[1]) >= 2:
        w = ins[1]
        return _bcast(x[:-2], w[:-2]) + [x[-2], w[-1]]
    if k == "Gemm" and len(ins) > 1:
        m = x[1] if a["trans_a"] else x[0]
        n = ins[1][0] if a["trans_b"] else ins[1][1]
        return [m, n]
    if k == "Conv2d" and len(ins) > 1 and len(x) == 4 and len(ins[1]) == 4:
        # conv_shape (shapes.rs:219-248): a dynamic (0) spatial dim stays 0
        w = ins[1]
        (sh, sw), (ph, pw) = a["strides"], a["padding"]
        return [x[0], w[0], 0 if x[2] == 0 else _out_dim(x[2], ph, w[2], sh),
                0 if x[3] == 0 else _out_dim(x[3], pw, w[3], sw)]
    if k in ("MaxPool2d", "AveragePool2d") and len(x) == 4:
        # pool_shape (shapes.rs:250-272): kernel 0 is the global pool
        (kh, kw), (sh, sw), (ph, pw) = a["kernel"], a["strides"], a["padding"]
        if kh == 0:
            return [x[0], x[1], 1, 1]
        return [x[0], x[1], _out_dim(x[2], ph, kh, sh), _out_dim(x[3], pw, kw, sw)]
    if k == "Flatten":
        ax = a["axis"] + len(x) if a["axis"] < 0 else a["axis"]
        return [int(np.prod(x[:ax], dtype=np.int64)), int(np.prod(x[ax:], dtype=np.int64))]
    if k == "Reshape":
        if a.get("view"):
            return x
        shape = list(a["shape"])
        total = int(np.prod(x, dtype=np.int64))
        shape = [x[i] if d == 0 and i < len(x) else d for i, d in enumerate(shape)]
        if -1 in shape:
            known = int(np.prod([d for d in shape if d != -1], dtype=np.int64))
            shape[shape.index(-1)] = total // max(known, 1)
        return shape
    if k == "Transpose":
        perm = a["perm"] or tuple(reversed(range(len(x))))
        return [x[p] for p in perm]
    if k == "Concat":
        ax = a["axis"] + len(x) if a["axis"] < 0 else a["axis"]
        out = list(x)
        out[ax] = sum(d[ax] for d in ins)
        return out
    return [1]


def load_from_bytes(data, max_bytes=1 << 31, max_graph_items=1_000_000):
    """load_from_bytes_with_limits + graph_from_proto (load.rs:116-398)."""
    if len(data) > max_bytes:
        raise OnnxError(f"invalid model: model is {len(data)} bytes, exceeding the {max_bytes}-byte limit")
    mv = memoryview(bytes(data))
    graph, opsets = None, []
    for f, _, v in _fields(mv):
        if f == 7:
            graph = _graph(v)
        elif f == 8:
            dom, ver = "", 0
            for f2, _, v2 in _fields(v):
                if f2 == 1:
                    dom = _str(v2)
                elif f2 == 2:
                    ver = _sint64(v2)
            opsets.append((dom, ver))
    if graph is None:
        raise OnnxError("invalid model: model has no graph")
    if len(graph["node"]) + sum(len(n["attribute"]) for n in graph["node"]) > max_graph_items:
        raise OnnxError("invalid model: too many nodes and attributes")
    if not graph["node"]:
        raise OnnxError("invalid model: graph has no nodes")
    for dom, ver in opsets:
        if dom == "" and ver > MAX_SUPPORTED_OPSET:
            raise OnnxError(f"invalid model: unsupported opset version {ver} for the default domain")
    shapes = {}
    for group in ("input", "output", "value_info"):
        for name, dims in graph[group]:
            if dims is not None:
                shapes.setdefault(name, dims)
    g = ComputationGraph()
    ids = {}
    inits = {t["name"]: t for t in graph["initializer"]}
    for name, _ in graph["input"]:
        if name in inits:
            continue
        ids[name] = g.add_input(shapes.get(name) or [1], name)
    for t in graph["initializer"]:
        if any(d < 0 for d in t["dims"]):
            raise OnnxError(f"invalid model: initializer '{t['name']}' has a negative declared dimension")
        dims = [int(d) for d in t["dims"]] or [1]
        ids[t["name"]] = g.add_input(dims, t["name"])
        vals = _tensor_f32(t)
        if vals is not None:
            if vals.size != int(np.prod(dims, dtype=np.int64)):
                raise OnnxError(f"invalid model: initializer '{t['name']}' declares "
                                f"{int(np.prod(dims, dtype=np.int64))} elements but has {vals.size}")
            g.add_initializer(t["name"], dims, vals)
    for n in graph["node"]:
        op = _build_operator(n, inits)
        ins = []
        for nm in n["input"]:
            if not nm:
                continue
            if nm not in ids:
                ids[nm] = g.add_input([1], nm)
            ins.append(ids[nm])
        if op.kind == "Reshape" and not op.attrs.get("view"):
            ins = ins[:1]  # the shape operand is an attribute here (load.rs:452-462)
        in_dims = [g.nodes[i].dims for i in ins]
        if op.kind == "AveragePool2d" and tuple(op.attrs["kernel"]) == (0, 0) and in_dims and len(in_dims[0]) == 4:
            op.attrs["kernel"] = tuple(in_dims[0][2:])  # GlobalAveragePool
        at = {a["name"]: a for a in n["attribute"]}
        auto = at.get("auto_pad", {}).get("s") if "auto_pad" in at else None
        if auto in ("SAME_UPPER", "SAME_LOWER") and in_dims and len(in_dims[0]) == 4:
            x = in_dims[0]
            if op.kind == "Conv2d" and len(in_dims) > 1 and len(in_dims[1]) == 4:
                kh, kw = in_dims[1][2], in_dims[1][3]
            elif op.kind in ("MaxPool2d", "AveragePool2d"):
                kh, kw = op.attrs["kernel"]
            else:
                kh = kw = None
            if kh is not None:
                sh, sw = op.attrs["strides"]
                op.attrs["padding"] = (_same_padding(x[2], kh, sh), _same_padding(x[3], kw, sw))
        out_name = n["output"][0] if n["output"] else ""
        dims = shapes.get(out_name) or _infer(op, in_dims)
        nid = g.add_node(op, ins, dims, n["name"])
        if out_name:
            ids[out_name] = nid
    marked = False
    for name, _ in graph["output"]:
        if name in ids:
            g.mark_output(ids[name])
            marked = True
    if not marked:  # infer_outputs: nodes nothing reads
        used = {i for nd in g.nodes for i in nd.inputs}
        for nd in g.nodes:
            if nd.id not in used and nd.op.kind != "Input":
                g.mark_output(nd.id)
    return g


def load(path):
    """load (load.rs:106-114)."""
    with open(path, "rb") as f:
        return load_from_bytes(f.read())


# ------------------------------------------------------------------ writer
def _enc_varint(v):
    v &= (1 << 64) - 1
    out = bytearray()
    while True:
        c = v & 0x7F
        v >>= 7
        if v:
            out.append(c | 0x80)
        else:
            out.append(c)
            return bytes(out)


def _key(f, wt):
    return _enc_varint(f << 3 | wt)


def _ld(f, payload):
    payload = payload.encode() if isinstance(payload, str) else bytes(payload)
    return _key(f, 2) + _enc_varint(len(payload)) + payload


def _vi(f, name, dims):
    dim_msgs = b"".join(_ld(1, _key(1, 0) + _enc_varint(d)) for d in dims)
    tensor_type = _key(1, 0) + _enc_varint(1) + _ld(2, dim_msgs)  # elem_type FLOAT, shape
    return _ld(f, _ld(1, name) + _ld(2, _ld(1, tensor_type)))


def _attr_ints(name, vals):
    return _ld(5, _ld(1, name) + _ld(8, b"".join(_enc_varint(int(v)) for v in vals)) + _key(20, 0) +
               _enc_varint(7))


def _attr_i(name, v):
    return _ld(5, _ld(1, name) + _key(3, 0) + _enc_varint(int(v)) + _key(20, 0) + _enc_varint(2))


def _attr_f(name, v):
    return _ld(5, _ld(1, name) + _key(2, 5) + struct.pack("<f", float(v)) + _key(20, 0) + _enc_varint(1))


def _tensor_msg(name, dims, data, dtype=1):
    raw = np.ascontiguousarray(data, "<f4" if dtype == 1 else "<i8").tobytes()
    return (_ld(1, b"".join(_enc_varint(int(d)) for d in dims)) + _key(2, 0) + _enc_varint(dtype) + _ld(8, name) +
            _ld(9, raw))


def save_bytes(graph: ComputationGraph, opset=17):
    """A ComputationGraph as ONNX bytes (ModelProto, ir_version 8): every node's
    output is named ``t<id>`` and declared in value_info with its dims; runtime
    inputs keep their names; initializers are raw little-endian f32."""
    names = {}
    for n in graph.nodes:
        names[n.id] = n.name if n.op.kind == "Input" else f"t{n.id}"
    body = bytearray()
    extra_inits = []
    for n in graph.nodes:
        k, a = n.op.kind, n.op.attrs
        if k == "Input":
            continue
        ins = [names[i] for i in n.inputs]
        attrs = b""
        op_type = {"Conv2d": "Conv", "MaxPool2d": "MaxPool", "AveragePool2d": "AveragePool",
                   "BatchNorm": "BatchNormalization", "LayerNorm": "LayerNormalization"}.get(k, k)
        if k == "Custom":
            op_type = a["name"]
        if k == "Conv2d":
            attrs = _attr_ints("strides", a["strides"]) + _attr_ints("pads", list(a["padding"]) * 2)
        elif k in ("MaxPool2d", "AveragePool2d"):
            attrs = (_attr_ints("kernel_shape", a["kernel"]) + _attr_ints("strides", a["strides"]) +
                     _attr_ints("pads", list(a["padding"]) * 2))
        elif k in ("Softmax", "Flatten", "Concat"):
            attrs = _attr_i("axis", a["axis"])
        elif k == "Transpose":
            attrs = _attr_ints("perm", a["perm"])
        elif k in ("BatchNorm", "LayerNorm"):
            attrs = _attr_f("epsilon", a["epsilon"])
        elif k == "Gemm":
            attrs = (_attr_f("alpha", a["alpha"]) + _attr_f("beta", a["beta"]) + _attr_i("transA", a["trans_a"]) +
                     _attr_i("transB", a["trans_b"]))
        elif k == "Reshape":
            sname = f"t{n.id}_shape"
            extra_inits.append(_tensor_msg(sname, [len(n.dims)], np.asarray(n.dims, np.int64), dtype=7))
            ins.append(sname)
        node = b"".join(_ld(1, s) for s in ins) + _ld(2, names[n.id]) + _ld(3, n.name or f"node{n.id}") + \
            _ld(4, op_type) + attrs
        body += _ld(1, node)
    for name, init in graph.initializers.items():
        body += _ld(5, _tensor_msg(name, init.dims, init.data))
    for t in extra_inits:
        body += _ld(5, t)
    for nid in graph.inputs():
        body += _vi(11, names[nid], graph.nodes[nid].dims)
    for nid in graph.outputs:
        body += _vi(12, names[nid], graph.nodes[nid].dims)
    for n in graph.nodes:
        if n.op.kind != "Input":
            body += _vi(13, names[n.id], n.dims)
    body = _ld(2, "tpt_graph") + bytes(body)
    model = _key(1, 0) + _enc_varint(8) + _ld(2, "tpt_infer_b200") + _ld(7, body) + \
        _ld(8, _ld(1, "") + _key(2, 0) + _enc_varint(opset))
    return model


def save(graph, path):
    with open(path, "wb") as f:
        f.write(save_bytes(graph))

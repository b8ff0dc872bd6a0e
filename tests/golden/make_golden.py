"""Extracts the reference's MatMulNBits (and GatherBlockQuantized) operator fixtures into
small ``.npz`` golden files that travel with this repository.

The fixtures are the reference's own known-answer tests: ``test/fixtures/ops/<case>/`` holds
``model.onnx`` (B, scales, zero points and bias as initializers), ``in_0.bin`` (A) and
``out_0.bin`` (Y recorded by ONNX Runtime on the CPU with graph optimizations off). They were
made by ``test/support/make_op_fixtures.py:140-165`` (the five small cases) and ``:1584-1593``
(``MatMulNBits_b4_bs256_packed``), and the reference checks them with the tolerance
``1e-4 + 1e-3 * max|Y|`` of ``test/transmuter/ops_test.exs:582-598``.

``onnx`` is not installed here, so a protobuf wire-format reader of ~60 lines decodes the few
fields that the fixtures use (ModelProto.graph, GraphProto.node/initializer,
NodeProto.input/output/op_type/attribute, AttributeProto.name/i, TensorProto
dims/data_type/raw_data/float_data).

Run once in a container that has the reference checkout::

    python tests/golden/make_golden.py /path/to/transmuter

It writes ``tests/golden/<case>.npz``. Nothing at test time reads the reference checkout.
"""

import json
import os
import sys

import numpy as np

CASES = [
    "MatMulNBits_b4_bs16_packed",
    "MatMulNBits_b4_bs32_none_bias",
    "MatMulNBits_b8_bs32_packed",
    "MatMulNBits_b4_bs16_float",
    "MatMulNBits_b2_bs16_packed",
    "MatMulNBits_b4_bs256_packed",
    "GatherBlockQuantized_b4",
    "GatherBlockQuantized_b8",
]

# TensorProto.DataType -> numpy
ONNX_DTYPES = {1: np.float32, 2: np.uint8, 3: np.int8, 6: np.int32, 7: np.int64, 10: np.float16, 11: np.float64}
NX_DTYPES = {"f32": np.float32, "f16": np.float16, "s64": np.int64, "u8": np.uint8}


def _varint(buf, i):
    shift = value = 0
    while True:
        byte = buf[i]
        i += 1
        value |= (byte & 0x7F) << shift
        shift += 7
        if byte < 0x80:
            return value, i


def fields(buf):
    """Yields (field number, wire type, value) of one protobuf message. Length-delimited
    values are bytes; varints are ints; fixed32/fixed64 are raw bytes."""
    i = 0
    while i < len(buf):
        key, i = _varint(buf, i)
        num, wire = key >> 3, key & 7
        if wire == 0:
            value, i = _varint(buf, i)
        elif wire == 1:
            value, i = buf[i:i + 8], i + 8
        elif wire == 2:
            size, i = _varint(buf, i)
            value, i = buf[i:i + size], i + size
        elif wire == 5:
            value, i = buf[i:i + 4], i + 4
        else:
            raise ValueError(f"unsupported wire type {wire}")
        yield num, wire, value


def tensor(buf):
    dims, dtype, raw, floats, name = [], None, None, [], ""
    for num, wire, value in fields(buf):
        if num == 1:
            if wire == 2:  # packed repeated int64
                j = 0
                while j < len(value):
                    d, j = _varint(value, j)
                    dims.append(d)
            else:
                dims.append(value)
        elif num == 2:
            dtype = value
        elif num == 4:
            floats.append(np.frombuffer(value, np.float32) if wire == 2 else np.frombuffer(value, np.float32))
        elif num == 8:
            name = value.decode()
        elif num == 9:
            raw = value
    np_dtype = ONNX_DTYPES[dtype]
    data = np.frombuffer(raw, np_dtype) if raw is not None else np.concatenate(floats).astype(np_dtype)
    return name, data.reshape(dims).copy()


def node(buf):
    out = {"input": [], "output": [], "op_type": "", "attrs": {}}
    for num, _wire, value in fields(buf):
        if num == 1:
            out["input"].append(value.decode())
        elif num == 2:
            out["output"].append(value.decode())
        elif num == 4:
            out["op_type"] = value.decode()
        elif num == 5:
            name, ival = None, None
            for anum, _aw, aval in fields(value):
                if anum == 1:
                    name = aval.decode()
                elif anum == 3:
                    ival = aval
            out["attrs"][name] = ival
    return out


def model(path):
    with open(path, "rb") as f:
        buf = f.read()
    graph = next(v for n, _w, v in fields(buf) if n == 7)
    nodes, inits = [], {}
    for num, _wire, value in fields(graph):
        if num == 1:
            nodes.append(node(value))
        elif num == 5:
            name, data = tensor(value)
            inits[name] = data
    return nodes, inits


def extract(reference, case):
    d = os.path.join(reference, "test", "fixtures", "ops", case)
    with open(os.path.join(d, "meta.json")) as f:
        meta = json.load(f)
    nodes, inits = model(os.path.join(d, "model.onnx"))
    (n,) = nodes
    out = {"op_type": np.array(n["op_type"]), "inputs": np.array(n["input"])}
    for key, value in n["attrs"].items():
        out["attr_" + key] = np.array(value, np.int64)
    for name, data in inits.items():
        out["init_" + name] = data
    for spec in meta["inputs"]:
        raw = np.fromfile(os.path.join(d, spec["file"]), NX_DTYPES[spec["dtype"]])
        out["in_" + spec["name"]] = raw.reshape(spec["shape"])
    for spec in meta["outputs"]:
        raw = np.fromfile(os.path.join(d, spec["file"]), NX_DTYPES[spec["dtype"]])
        out["out_" + spec["name"]] = raw.reshape(spec["shape"])
    return out


def main():
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_golden.py <checkout of georgeguimaraes/transmuter>")
    reference = sys.argv[1]
    here = os.path.dirname(os.path.abspath(__file__))
    for case in CASES:
        out = extract(reference, case)
        np.savez(os.path.join(here, case + ".npz"), **out)
        print(case, {k: getattr(v, "shape", v) for k, v in out.items()})


if __name__ == "__main__":
    main()

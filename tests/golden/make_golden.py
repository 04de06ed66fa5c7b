"""Regenerates the golden fixtures in this directory from the reference's
own ORT-oracle fixtures (CrispStrobe/onnx_runtime_dart, test/fixtures/<case>/
{model.onnx, case.json}, produced by its tool/gen_fixtures.py:891-925 and
:114-120 with native onnxruntime).

Usage (needs the reference checkout; run once, output is committed):

    python tests/golden/make_golden.py /path/to/onnx_runtime_dart

For every hot-path case it decodes the single-node ONNX graph with a small
protobuf wire-format reader (the `onnx` package is not needed), and writes
``<case>.npz`` holding the graph inputs (``in_<name>``), the initializers
(``init_<name>``), the node's op type / attributes / input order (as a JSON
string under ``meta``) and the ORT-computed output (``expected``).
"""
from __future__ import annotations

import json
import os
import struct
import sys

import numpy as np

CASES = [
    "matmulnbits_basic",
    "matmulnbits_zeropoints",
    "matmulnbits_partial_block",
    "gemm_transB_bias",
    "matmul_batched",
    # device ArgMax / ArgMin over the last axis (the lm_head -> ArgMax step
    # of greedy decoding), pinned to the reference's ORT fixtures
    "argmax_axis1",
    "argmax_nan",
    "argmin_nokeep_last",
    # the int8 dynamic-quantisation path: DynamicQuantizeLinear and
    # MatMulInteger (scalar / per-column zero points, u8 x i8, batched)
    "dynamicquantizelinear",
    "matmulinteger_nozp",
    "matmulinteger_percol_bzp",
    "matmulinteger_u8i8",
    "matmulinteger_batched",
    # the attention ops around the projections of a decoder step
    "gqa_causal",
    "gqa_kvcache",
    "gqa_kvcache_bias",
    "gqa_kvcache_rotary",
    "mha_no_bias",
    "mha_with_bias",
    "rotary_embedding",
    "sdpa_pattern",  # MatMul/Div/Add/Softmax/MatMul, fused to _FusedSDPA
    # candidate selection after lm_head (top-k sampling)
    "topk_largest",
    "topk_smallest_axis0",
]

_ONNX_DTYPES = {1: np.float32, 2: np.uint8, 3: np.int8, 6: np.int32, 7: np.int64,
                10: np.float16, 11: np.float64}


def _varint(buf, i):
    shift = v = 0
    while True:
        b = buf[i]
        i += 1
        v |= (b & 0x7F) << shift
        if b < 0x80:
            return v, i
        shift += 7


def _fields(buf):
    """Yields (field_number, wire_type, value) of one protobuf message."""
    i = 0
    while i < len(buf):
        key, i = _varint(buf, i)
        fn, wt = key >> 3, key & 7
        if wt == 0:
            v, i = _varint(buf, i)
        elif wt == 1:
            v = buf[i:i + 8]
            i += 8
        elif wt == 2:
            ln, i = _varint(buf, i)
            v = buf[i:i + ln]
            i += ln
        elif wt == 5:
            v = buf[i:i + 4]
            i += 4
        else:
            raise ValueError(f"unsupported wire type {wt}")
        yield fn, wt, v


def _packed_varints(buf):
    out, i = [], 0
    while i < len(buf):
        v, i = _varint(buf, i)
        out.append(v)
    return out


def _tensor(buf):
    """TensorProto: dims=1, data_type=2, float_data=4, int32_data=5,
    int64_data=7, name=8, raw_data=9."""
    dims, dtype, name, raw = [], None, "", None
    floats, ints32, ints64 = [], [], []
    for fn, wt, v in _fields(buf):
        if fn == 1:
            dims += _packed_varints(v) if wt == 2 else [v]
        elif fn == 2:
            dtype = v
        elif fn == 4:
            floats += list(struct.unpack(f"<{len(v) // 4}f", v)) if wt == 2 else \
                [struct.unpack("<f", v)[0]]
        elif fn == 5:
            ints32 += _packed_varints(v) if wt == 2 else [v]
        elif fn == 7:
            ints64 += _packed_varints(v) if wt == 2 else [v]
        elif fn == 8:
            name = v.decode()
        elif fn == 9:
            raw = bytes(v)
    npdt = _ONNX_DTYPES[dtype]
    if raw is not None:
        arr = np.frombuffer(raw, dtype=npdt).copy()
    elif floats:
        arr = np.array(floats, dtype=npdt)
    elif ints32:
        arr = np.array(ints32, dtype=np.int64).astype(npdt)
    else:
        arr = np.array(ints64, dtype=npdt)
    return name, arr.reshape(dims)


def _attribute(buf):
    """AttributeProto: name=1, f=2, i=3."""
    name, val = "", None
    for fn, wt, v in _fields(buf):
        if fn == 1:
            name = v.decode()
        elif fn == 2:
            val = struct.unpack("<f", v)[0]
        elif fn == 3:
            val = v - (1 << 64) if v >= (1 << 63) else v
    return name, val


def _node(buf):
    """NodeProto: input=1, output=2, op_type=4, attribute=5, domain=7."""
    node = {"inputs": [], "outputs": [], "op_type": "", "attrs": {}, "domain": ""}
    for fn, _, v in _fields(buf):
        if fn == 1:
            node["inputs"].append(v.decode())
        elif fn == 2:
            node["outputs"].append(v.decode())
        elif fn == 4:
            node["op_type"] = v.decode()
        elif fn == 5:
            k, a = _attribute(v)
            node["attrs"][k] = a
        elif fn == 7:
            node["domain"] = v.decode()
    return node


def parse_model(path):
    """ModelProto.graph=7; GraphProto.node=1, initializer=5."""
    data = open(path, "rb").read()
    graph = next(v for fn, _, v in _fields(data) if fn == 7)
    nodes, inits = [], {}
    for fn, _, v in _fields(graph):
        if fn == 1:
            nodes.append(_node(v))
        elif fn == 5:
            name, arr = _tensor(v)
            inits[name] = arr
    return nodes, inits


def main(ref_root):
    out_dir = os.path.dirname(os.path.abspath(__file__))
    for case in CASES:
        d = os.path.join(ref_root, "test", "fixtures", case)
        nodes, inits = parse_model(os.path.join(d, "model.onnx"))
        cj = json.load(open(os.path.join(d, "case.json")))
        arrays = {}
        for k, v in cj["inputs"].items():
            arrays["in_" + k] = np.array(v["data"], dtype=v["dtype"]).reshape(v["shape"])
        for k, v in inits.items():
            arrays["init_" + k] = v
        outs = list(cj["expected"].items())
        for ok, ov in outs:  # every output; the only one also as "expected"
            arr = np.array(ov["data"], dtype=ov["dtype"]).reshape(ov["shape"])
            arrays["expected_" + ok] = arr
            if len(outs) == 1:
                arrays["expected"] = arr
        # one node, or (a pattern the reference fuses) the whole node list
        meta = dict(nodes[0]) if len(nodes) == 1 else {"nodes": nodes, "op_type": "pattern"}
        meta["source"] = f"test/fixtures/{case}"
        arrays["meta"] = np.array(json.dumps(meta))
        np.savez(os.path.join(out_dir, case + ".npz"), **arrays)
        print(case, {k: v.shape for k, v in arrays.items()}, meta.get("attrs"))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <reference checkout>")
    main(sys.argv[1])

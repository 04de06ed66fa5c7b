"""Maps the reference's attention fixtures (tests/golden/{gqa_*, mha_*,
rotary_embedding, sdpa_pattern}.npz) onto the arguments of the attention
ops, as the reference's dispatch reads them (lib/src/onnx_graph.dart:
978-1000 for GroupQueryAttention / MultiHeadAttention / RotaryEmbedding,
:355-386 for the Softmax pattern fused to _FusedSDPA)."""
import numpy as np

GQA_CASES = ["gqa_causal", "gqa_kvcache", "gqa_kvcache_bias", "gqa_kvcache_rotary"]
MHA_CASES = ["mha_no_bias", "mha_with_bias"]


def _inputs(g):
    """name -> array over the graph inputs and initializers."""
    d = {}
    for k, v in g.items():
        if k.startswith("in_"):
            d[k[3:]] = v
        elif k.startswith("init_"):
            d[k[5:]] = v
    return d


def _arg(node, vals, idx):
    names = node["inputs"]
    if idx >= len(names) or names[idx] == "":
        return None
    return vals[names[idx]]


def gqa_args(g):
    """(q, k, v, kwargs) for a GroupQueryAttention fixture; inputs 3/4 past
    K/V, 7/8 cos/sin caches, 10 the attention bias (seqlens_k and
    total_sequence_length are not read, as in the reference)."""
    node, vals = g["meta"], _inputs(g)
    a = node["attrs"]
    kw = dict(num_heads=int(a["num_heads"]), kv_num_heads=int(a["kv_num_heads"]),
              scale=a.get("scale"), do_rotary=bool(a.get("do_rotary", 0)),
              rotary_interleaved=bool(a.get("rotary_interleaved", 0)),
              past_key=_arg(node, vals, 3), past_value=_arg(node, vals, 4),
              cos_cache=_arg(node, vals, 7), sin_cache=_arg(node, vals, 8),
              attention_bias=_arg(node, vals, 10))
    return _arg(node, vals, 0), _arg(node, vals, 1), _arg(node, vals, 2), kw


def mha_args(g):
    node, vals = g["meta"], _inputs(g)
    a = node["attrs"]
    kw = dict(num_heads=int(a["num_heads"]), scale=a.get("scale"),
              attention_bias=_arg(node, vals, 5))
    return _arg(node, vals, 0), _arg(node, vals, 1), _arg(node, vals, 2), kw


def rotary_args(g):
    node, vals = g["meta"], _inputs(g)
    a = node["attrs"]
    return ([_arg(node, vals, i) for i in range(4)],
            dict(interleaved=bool(a.get("interleaved", 0)), num_heads=int(a.get("num_heads", 0)),
                 rotary_dim=int(a.get("rotary_embedding_dim", 0))))


def sdpa_args(g):
    """The fused node's inputs (A, B, V, mask) and float32 scale: the
    fixture is MatMul -> Div(sqrt_d) -> Add(mask) -> Softmax -> MatMul, which
    the reference folds with scale = float32(1 / sqrt_d)."""
    nodes, vals = g["meta"]["nodes"], _inputs(g)
    mm1, div, add, _, mm2 = nodes
    assert [n["op_type"] for n in nodes] == ["MatMul", "Div", "Add", "Softmax", "MatMul"]
    c = float(vals[div["inputs"][1]])
    mask_name = add["inputs"][1] if add["inputs"][0] == div["outputs"][0] else add["inputs"][0]
    return (vals[mm1["inputs"][0]], vals[mm1["inputs"][1]], vals[mm2["inputs"][1]],
            vals[mask_name], float(np.float32(1.0 / c)))

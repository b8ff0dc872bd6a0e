"""The sibling-matmul merge of Transmuter's loader for packed MatMulNBits weights: a Python mirror
of ``Fusion.matmuls/2`` (lib/transmuter/fusion.ex:430-540) over tq4 handles.

The reference merges the matmuls of a moved model that read one input (q, k and v; gate and up)
into one matmul over the weights concatenated along N plus a ``Split`` of its output, and does so
only for float {N, K} weights (``mergeable?/3``, :466-473). Here the weights stay packed on the
GPU: a group's handles are concatenated row-wise by ``tq4_weight_merge``, so one GEMV streams the
whole group's rows. The grouping follows the reference:

- a node merges when it is a MatMulNBits whose A input is not empty, whose optional inputs
  (zero points, g_idx, bias) are all empty after the move, whose weight is read by no other node,
  and whose weight is a packed handle;
- nodes group by (A input, dequantize type, K, and the packed layout: bits, block_size, scale
  and zero-point types), the reference's ``merge_key/2`` (:480-484) with the layout added,
  because only handles of one layout concatenate;
- groups of at least two nodes merge; the merged node keeps the first node's name and inputs with
  the merged weight's name (``<first weight>:merged``) and N; a Split node with the groups' N
  sizes restores the original outputs (:490-530).
"""

from collections import Counter
from dataclasses import replace

from .deferred import ArgumentError
from .quantized import Node, PackedWeight


def dependencies(node):
    """The inputs a node reads (``Transmuter.dependencies/1``): its non-empty input names."""
    return [x for x in node.input if x]


def mergeable(node, weights, uses):
    """``mergeable?/3`` for packed weights."""
    if node.op_type != "MatMulNBits" or len(node.input) < 2:
        return False
    a, w, rest = node.input[0], node.input[1], node.input[2:]
    return (a != "" and all(x == "" for x in rest) and uses.get(w, 0) == 1
            and isinstance(weights.get(w), PackedWeight))


def merge_key(node, weights):
    w = weights[node.input[1]]
    d = w.desc
    return (node.op_type, node.input[0], str(w.dtype), w.k, w.bits, w.block_size, d.scale_dtype, d.zp_kind, d.zp_dtype)


def matmuls(nodes, weights, outputs=(), merge=PackedWeight.merge):
    """Returns (nodes, weights) with every group of sibling MatMulNBits merged. ``weights`` maps
    weight names to handles; merged parts are removed from it (the caller closes them) and the
    merged handle is added. ``merge`` builds the merged weight from a list of parts."""
    uses = Counter([x for n in nodes for x in dependencies(n)] + list(outputs))
    groups = {}
    for n in nodes:
        if mergeable(n, weights, uses):
            groups.setdefault(merge_key(n, weights), []).append(n)
    groups = [g for g in groups.values() if len(g) >= 2]
    weights = dict(weights)
    replacements = {}
    for group in groups:
        first = group[0]
        parts = [weights[n.input[1]] for n in group]
        sizes = [p.n for p in parts]
        name = first.input[1] + ":merged"
        if name in weights:
            raise ArgumentError(f"the model already has a param {name}")
        output = first.output[0] + ":merged"
        attrs = dict(first.attribute, N=sum(sizes))
        merged = replace(first, input=[first.input[0], name] + list(first.input[2:]), output=[output],
                         attribute=attrs)
        merged.attribute["transmuter.fused"] = [n.name for n in group]
        split = Node("Split", {"axis": -1, "split": sizes}, [output], [n.output[0] for n in group],
                     name=f"{first.name}:split")
        weights[name] = merge(parts)
        for n in group:
            weights.pop(n.input[1], None)
        replacements[id(first)] = [merged, split]
        for n in group[1:]:
            replacements[id(n)] = []
    out = []
    for n in nodes:
        out.extend(replacements.get(id(n), [n]))
    return out, weights


def split(y, sizes):
    """The Split node after a merged matmul: Y's last axis cut into the parts' N."""
    import torch
    return list(torch.split(y, list(sizes), dim=-1))

"""Host logic of the packed sibling-matmul merge (transmuter_b200/fusion.py, the packed form of
Fusion.matmuls/2, lib/transmuter/fusion.ex:430-540), on CPU with stand-in weights: which nodes
group, the merged node and its Split, and what stays unmerged."""

from transmuter_b200 import _lib, fusion
from transmuter_b200.quantized import Node, PackedWeight


def fake_weight(k, n, bits=4, bs=32, zp_kind=0):
    w = PackedWeight.__new__(PackedWeight)
    w.k, w.n, w.bits, w.block_size, w.dtype = k, n, bits, bs, "f32"
    w.desc = _lib.WeightDesc()
    w.desc.K, w.desc.N, w.desc.bits, w.desc.block_size = k, n, bits, bs
    w.desc.scale_dtype, w.desc.zp_kind, w.desc.zp_dtype = _lib.F32, zp_kind, _lib.U8
    w._handle = None
    return w


def node(name, a, w, out, extra=()):
    return Node("MatMulNBits", {"K": 1024, "N": 0, "bits": 4, "block_size": 32}, [a, w, *extra], [out], name=name)


def fake_merge(parts):
    return fake_weight(parts[0].k, sum(p.n for p in parts))


def test_q_k_v_and_gate_up_merge_into_one_node_and_a_split_each():
    weights = {"wq": fake_weight(1024, 2048), "wk": fake_weight(1024, 1024), "wv": fake_weight(1024, 1024),
               "wg": fake_weight(1024, 3072), "wu": fake_weight(1024, 3072), "wo": fake_weight(2048, 1024)}
    nodes = [node("q", "x", "wq", "q_out"), node("k", "x", "wk", "k_out"), node("v", "x", "wv", "v_out"),
             node("o", "attn", "wo", "o_out"),
             node("gate", "h", "wg", "g_out"), node("up", "h", "wu", "u_out")]
    out, w = fusion.matmuls(nodes, weights, merge=fake_merge)
    names = [(n.op_type, n.name) for n in out]
    assert names == [("MatMulNBits", "q"), ("Split", "q:split"), ("MatMulNBits", "o"),
                     ("MatMulNBits", "gate"), ("Split", "gate:split")]
    qkv, split = out[0], out[1]
    assert qkv.input == ["x", "wq:merged"] and qkv.output == ["q_out:merged"]
    assert qkv.attribute["N"] == 4096 and qkv.attribute["transmuter.fused"] == ["q", "k", "v"]
    assert split.input == ["q_out:merged"] and split.output == ["q_out", "k_out", "v_out"]
    assert split.attribute == {"axis": -1, "split": [2048, 1024, 1024]}
    assert set(w) == {"wq:merged", "wo", "wg:merged"} and w["wq:merged"].n == 4096 and w["wg:merged"].n == 6144


def test_what_does_not_merge():
    weights = {"a": fake_weight(1024, 64), "b": fake_weight(1024, 64), "c": fake_weight(512, 64),
               "d": fake_weight(1024, 64, bs=64), "e": fake_weight(1024, 64), "f": fake_weight(1024, 64),
               "g": fake_weight(1024, 64)}
    nodes = [node("a", "x", "a", "ya", extra=("", "", "", "bias")),  # a bias input
             node("b", "x", "b", "yb"), node("c", "x", "c", "yc"),  # another K
             node("d", "x", "d", "yd"),                              # another block size
             node("e", "y", "e", "ye"),                              # alone on its input
             node("f", "z", "f", "yf"), node("g", "z", "g", "yg"),
             Node("Add", {}, ["f", "yb"], ["sum"])]                  # weight f read by another node
    out, w = fusion.matmuls(nodes, weights, merge=fake_merge)
    assert [n.name for n in out] == ["a", "b", "c", "d", "e", "f", "g", ""]
    assert w.keys() == weights.keys()


def test_merged_graph_gives_the_unmerged_outputs():
    """fusion_test.exs:396-430: two 4-bit MatMulNBits nodes read x (K 1024, N 32 and 16, block 32,
    no zero points, B an iota pattern, constant scales). The merged node and its Split give the
    outputs of the graph without the rewrite, within the test's tolerance (atol = rtol = 1e-4).
    Evaluated here with the oracle, the merged weight being the row concatenation of the parts'
    B and scales (the layout tq4_weight_merge builds on the device, where the GPU tests check it
    bit for bit)."""
    import numpy as np
    from oracle import matmul_nbits as o

    def packed(n, factor):
        return ((np.arange(n * 32 * 16).reshape(n, 32, 16) * factor) % 256).astype(np.uint8)

    weights = {}
    for name, b, s in (("bq", packed(32, 7), 0.01), ("bk", packed(16, 13), 0.02)):
        w = fake_weight(1024, b.shape[0])
        w.host = (b, np.full(b.shape[0] * 32, s, np.float32))
        weights[name] = w

    def merge(parts):
        w = fake_weight(parts[0].k, sum(p.n for p in parts))
        w.host = tuple(np.concatenate([p.host[i] for p in parts]) for i in range(2))
        return w

    attrs = {"K": 1024, "bits": 4, "block_size": 32}
    nodes = [Node("MatMulNBits", dict(attrs, N=32), ["x", "bq"], ["q"], name="q"),
             Node("MatMulNBits", dict(attrs, N=16), ["x", "bk"], ["k"], name="k")]
    x = ((np.arange(2 * 1024) % 17.0) - 8.0).astype(np.float32).reshape(1, 2, 1024)

    def run(graph, ws):
        env = {"x": x}
        for n in graph:
            if n.op_type == "MatMulNBits":
                b, s = ws[n.input[1]].host
                env[n.output[0]] = o.matmul_nbits(n.attribute, env[n.input[0]], b, s)[0]
            else:  # Split along the last axis
                cuts = np.cumsum(n.attribute["split"])[:-1]
                env.update(zip(n.output, np.split(env[n.input[0]], cuts, axis=-1)))
        return env

    fused, fw = fusion.matmuls(nodes, weights, outputs=["q", "k"], merge=merge)
    assert [n.op_type for n in fused] == ["MatMulNBits", "Split"]
    merged = fw["bq:merged"]
    wq = o.dequantize_weight(*weights["bq"].host, None, 1024, 32, 4, 32, "f32")
    wk = o.dequantize_weight(*weights["bk"].host, None, 1024, 16, 4, 32, "f32")
    np.testing.assert_array_equal(o.dequantize_weight(*merged.host, None, 1024, 48, 4, 32, "f32"),
                                  np.concatenate([wq, wk]))
    want, got = run(nodes, weights), run(fused, fw)
    for name in ("q", "k"):
        assert got[name].shape == want[name].shape == (1, 2, {"q": 32, "k": 16}[name])
        np.testing.assert_allclose(got[name], want[name], atol=1e-4, rtol=1e-4)

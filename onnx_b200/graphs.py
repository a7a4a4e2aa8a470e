"""Graph definitions: the node-list form of an ONNX model that the executor runs.

A ``GraphDef`` mirrors what ``Model.Load`` produces in the reference
(src/Lokad.Onnx.Backend/Model.cs:30-63): nodes in file order with string
tensor names and typed attributes, a name -> initializer map, and the graph's
input/output names.  The builders produce the benchmark workloads with seeded
synthetic weights:

* ``mnist8``  -- the topology of the reference's test model
  tests/Lokad.Onnx.Backend.Tests/models/mnist-8.onnx (12 nodes, opset 8);
* ``e5_encoder`` -- a BERT-style encoder shaped like multilingual-e5-small,
  written with the same decomposed ops an ONNX export of that model uses
  (Gather embeddings, ReduceMean-based LayerNorm, Erf GELU, MatMul+Add
  projections, Reshape/Transpose head split, Softmax with an additive mask),
  mean-pooled over the attention mask.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass, field

import numpy as np


@dataclass
class Node:
    op: str
    inputs: list
    outputs: list
    attrs: dict = field(default_factory=dict)


@dataclass
class GraphDef:
    nodes: list
    initializers: dict
    inputs: list
    outputs: list
    opset: int = 13


def from_json(path_json: str, arrays: dict, prefix: str = "init/") -> GraphDef:
    """Load a node list written by tests/golden/make_mnist8_fixture.py."""
    with open(path_json) as f:
        g = json.load(f)
    nodes = [Node(n["op"], n["inputs"], n["outputs"], n["attrs"]) for n in g["nodes"]]
    inits = {k[len(prefix):]: np.asarray(v) for k, v in arrays.items() if k.startswith(prefix)}
    return GraphDef(nodes, inits, g["inputs"], g["outputs"], g["opset"])


def mnist8(seed: int = 0) -> GraphDef:
    """mnist-8 topology with N(0, 0.1) weights."""
    rng = np.random.default_rng(seed)
    w = lambda *s: (rng.standard_normal(s) * 0.1).astype(np.float32)
    inits = {
        "Parameter193": w(16, 4, 4, 10),
        "Parameter193_reshape1_shape": np.array([256, 10], np.int64),
        "Parameter5": w(8, 1, 5, 5),
        "Parameter6": w(8, 1, 1),
        "Parameter87": w(16, 8, 5, 5),
        "Parameter88": w(16, 1, 1),
        "Pooling160_Output_0_reshape0_shape": np.array([1, 256], np.int64),
        "Parameter194": w(1, 10),
    }
    conv = {"kernel_shape": [5, 5], "strides": [1, 1], "auto_pad": "SAME_UPPER", "group": 1,
            "dilations": [1, 1]}
    N = Node
    nodes = [
        N("Reshape", ["Parameter193", "Parameter193_reshape1_shape"], ["Parameter193_reshape1"]),
        N("Conv", ["Input3", "Parameter5"], ["Convolution28_Output_0"], dict(conv)),
        N("Add", ["Convolution28_Output_0", "Parameter6"], ["Plus30_Output_0"]),
        N("Relu", ["Plus30_Output_0"], ["ReLU32_Output_0"]),
        N("MaxPool", ["ReLU32_Output_0"], ["Pooling66_Output_0"],
          {"kernel_shape": [2, 2], "strides": [2, 2], "pads": [0, 0, 0, 0], "auto_pad": "NOTSET"}),
        N("Conv", ["Pooling66_Output_0", "Parameter87"], ["Convolution110_Output_0"], dict(conv)),
        N("Add", ["Convolution110_Output_0", "Parameter88"], ["Plus112_Output_0"]),
        N("Relu", ["Plus112_Output_0"], ["ReLU114_Output_0"]),
        N("MaxPool", ["ReLU114_Output_0"], ["Pooling160_Output_0"],
          {"kernel_shape": [3, 3], "strides": [3, 3], "pads": [0, 0, 0, 0], "auto_pad": "NOTSET"}),
        N("Reshape", ["Pooling160_Output_0", "Pooling160_Output_0_reshape0_shape"],
          ["Pooling160_Output_0_reshape0"]),
        N("MatMul", ["Pooling160_Output_0_reshape0", "Parameter193_reshape1"], ["Times212_Output_0"]),
        N("Add", ["Times212_Output_0", "Parameter194"], ["Plus214_Output_0"]),
    ]
    return GraphDef(nodes, inits, ["Input3"], ["Plus214_Output_0"], opset=8)


E5_SMALL = dict(layers=12, hidden=384, heads=12, ffn=1536, vocab=250037, max_pos=512, eps=1e-12)


def e5_encoder(layers=12, hidden=384, heads=12, ffn=1536, vocab=250037, max_pos=512,
               seq=128, eps=1e-12, seed=0, std=0.02) -> GraphDef:
    """BERT-style post-LayerNorm encoder shaped like multilingual-e5-small,
    random-init N(0, std) weights.

    Inputs: input_ids, attention_mask, token_type_ids -- int64 [B, seq].
    Output: ``sentence_embedding`` [B, hidden], the attention-mask mean pool
    of the last hidden state (``last_hidden_state`` is also an output)."""
    rng = np.random.default_rng(seed)
    H, dh = hidden, hidden // heads
    g = lambda *s: (rng.standard_normal(s, dtype=np.float32) * std).astype(np.float32)
    inits = {}
    nodes = []
    N = lambda op, i, o, **a: nodes.append(Node(op, list(i), list(o), dict(a)))
    c = lambda name, arr: inits.__setitem__(name, arr)

    c("word_embeddings", g(vocab, H))
    c("position_embeddings", g(max_pos, H))
    c("token_type_embeddings", g(1, H))
    c("position_ids", np.arange(seq, dtype=np.int64).reshape(1, seq))
    c("one", np.array(1.0, np.float32))
    c("two", np.array(2.0, np.float32))
    c("half", np.array(0.5, np.float32))
    c("sqrt2", np.array(np.sqrt(2.0), np.float32))
    c("eps", np.array(eps, np.float32))
    c("scale", np.array(np.sqrt(dh), np.float32))
    c("mask_min", np.array(np.finfo(np.float32).min, np.float32))
    c("axes_last", np.array([-1], np.int64))
    c("axes_1", np.array([1], np.int64))
    c("axes_2", np.array([2], np.int64))
    c("heads_shape", np.array([0, 0, heads, dh], np.int64))
    c("merge_shape", np.array([0, 0, H], np.int64))

    def layernorm(x, p):
        c(p + ".gamma", (1.0 + g(H)).astype(np.float32))
        c(p + ".beta", g(H))
        N("ReduceMean", [x, "axes_last"], [p + "/mean"])
        N("Sub", [x, p + "/mean"], [p + "/d"])
        N("Pow", [p + "/d", "two"], [p + "/d2"])
        N("ReduceMean", [p + "/d2", "axes_last"], [p + "/var"])
        N("Add", [p + "/var", "eps"], [p + "/ve"])
        N("Sqrt", [p + "/ve"], [p + "/std"])
        N("Div", [p + "/d", p + "/std"], [p + "/n"])
        N("Mul", [p + "/n", p + ".gamma"], [p + "/y"])
        N("Add", [p + "/y", p + ".beta"], [p + "/out"])
        return p + "/out"

    def linear(x, p, k, n):
        c(p + ".weight", g(k, n))
        c(p + ".bias", g(n))
        N("MatMul", [x, p + ".weight"], [p + "/mm"])
        N("Add", [p + "/mm", p + ".bias"], [p + "/out"])
        return p + "/out"

    # embeddings
    N("Gather", ["word_embeddings", "input_ids"], ["emb/word"], axis=0)
    N("Gather", ["token_type_embeddings", "token_type_ids"], ["emb/type"], axis=0)
    N("Add", ["emb/word", "emb/type"], ["emb/wt"])
    N("Gather", ["position_embeddings", "position_ids"], ["emb/pos"], axis=0)
    N("Add", ["emb/wt", "emb/pos"], ["emb/sum"])
    x = layernorm("emb/sum", "emb/ln")

    # extended attention mask: (1 - mask[:, None, None, :]) * float32.min
    N("Unsqueeze", ["attention_mask", "axes_1"], ["mask/u1"])
    N("Unsqueeze", ["mask/u1", "axes_2"], ["mask/u2"])
    N("Cast", ["mask/u2"], ["mask/f"], to=1)
    N("Sub", ["one", "mask/f"], ["mask/inv"])
    N("Mul", ["mask/inv", "mask_min"], ["mask/add"])

    for l in range(layers):
        p = f"l{l}"
        q = linear(x, p + ".q", H, H)
        k = linear(x, p + ".k", H, H)
        v = linear(x, p + ".v", H, H)
        N("Reshape", [q, "heads_shape"], [p + "/q4"])
        N("Transpose", [p + "/q4"], [p + "/qt"], perm=[0, 2, 1, 3])
        N("Reshape", [k, "heads_shape"], [p + "/k4"])
        N("Transpose", [p + "/k4"], [p + "/kt"], perm=[0, 2, 3, 1])
        N("Reshape", [v, "heads_shape"], [p + "/v4"])
        N("Transpose", [p + "/v4"], [p + "/vt"], perm=[0, 2, 1, 3])
        N("MatMul", [p + "/qt", p + "/kt"], [p + "/s"])
        N("Div", [p + "/s", "scale"], [p + "/ss"])
        N("Add", [p + "/ss", "mask/add"], [p + "/sm"])
        N("Softmax", [p + "/sm"], [p + "/p"], axis=-1)
        N("MatMul", [p + "/p", p + "/vt"], [p + "/ctx"])
        N("Transpose", [p + "/ctx"], [p + "/ctxt"], perm=[0, 2, 1, 3])
        N("Reshape", [p + "/ctxt", "merge_shape"], [p + "/ctx2"])
        o = linear(p + "/ctx2", p + ".o", H, H)
        N("Add", [o, x], [p + "/r1"])
        x1 = layernorm(p + "/r1", p + ".ln1")
        f = linear(x1, p + ".ffn1", H, ffn)
        N("Div", [f, "sqrt2"], [p + "/ga"])
        N("Erf", [p + "/ga"], [p + "/gb"])
        N("Add", [p + "/gb", "one"], [p + "/gc"])
        N("Mul", [f, p + "/gc"], [p + "/gd"])
        N("Mul", [p + "/gd", "half"], [p + "/ge"])
        f2 = linear(p + "/ge", p + ".ffn2", ffn, H)
        N("Add", [f2, x1], [p + "/r2"])
        x = layernorm(p + "/r2", p + ".ln2")

    # masked mean pool
    N("Unsqueeze", ["attention_mask", "axes_last"], ["pool/u"])
    N("Cast", ["pool/u"], ["pool/m"], to=1)
    N("Mul", [x, "pool/m"], ["pool/xm"])
    N("ReduceSum", ["pool/xm", "axes_1"], ["pool/sum"], keepdims=0)
    N("ReduceSum", ["pool/m", "axes_1"], ["pool/cnt"], keepdims=0)
    N("Div", ["pool/sum", "pool/cnt"], ["sentence_embedding"])
    return GraphDef(nodes, inits, ["input_ids", "attention_mask", "token_type_ids"],
                    ["sentence_embedding", x], opset=18)


def e5_inputs(batch, seq=128, vocab=250037, seed=0):
    """Synthetic e5 inputs: uniform token ids, an
    attention mask of ones with a random right-padded tail per row (tail
    length uniform in [0, seq-1]), token types all zero."""
    rng = np.random.default_rng(seed + 1)
    ids = rng.integers(0, vocab, size=(batch, seq), dtype=np.int64)
    tail = rng.integers(0, seq, size=batch)
    mask = np.ones((batch, seq), np.int64)
    for b in range(batch):
        if tail[b]:
            mask[b, seq - tail[b]:] = 0
    return {"input_ids": ids, "attention_mask": mask,
            "token_type_ids": np.zeros((batch, seq), np.int64)}


def e5_flops_per_seq(layers=12, hidden=384, ffn=1536, seq=128):
    """Algorithmic FLOPs per sequence: projections, FFN and the two attention
    products (2 FLOP per multiply-add)."""
    return layers * (2 * seq * hidden * 4 * hidden + 2 * 2 * seq * hidden * ffn
                     + 2 * 2 * seq * seq * hidden)


def resnet50(num_classes=1000, seed=0, onnx_ops=False) -> GraphDef:
    """ResNet-50 v1: stride on the first 1x1 of each downsampling bottleneck,
    Kaiming-normal conv weights, global average pool, final 2048 x
    num_classes classifier.

    onnx_ops=False: BatchNorm folded into each conv's weight scale and bias
    (the folded BN scale is 0.2 on the last conv of each residual branch and
    0.5 on projection shortcuts, which keeps activations O(1) through the 16
    residual sums as trained BNs do), global average pool as ReduceMean over
    H and W, classifier as MatMul + bias Add -- only ops the reference
    dispatches.

    onnx_ops=True: the graph as an ONNX export of torchvision's ResNet-50
    lays it out -- Conv without bias -> BatchNormalization (seeded
    scale/B/mean/var, same per-branch damping) -> Relu, GlobalAveragePool,
    Flatten, Gemm(transB=1) -- the ops the reference names but cannot run.

    Convs carry explicit strides/pads; run them with the attributes applied
    (ComputationalGraph(..., honor_conv_attrs=True)), which the reference's
    Conv dispatch does not do (Node.cs:137-138)."""
    rng = np.random.default_rng(seed)
    inits, nodes = {}, []
    cnt = [0]

    def conv(x, cin, cout, k, s, pad, relu, gamma=1.0):
        i = cnt[0]
        cnt[0] += 1
        w, b = f"conv{i}.w", f"conv{i}.b"
        attrs = {"kernel_shape": [k, k], "strides": [s, s], "pads": [pad] * 4, "auto_pad": "NOTSET", "group": 1,
                 "dilations": [1, 1]}
        y = f"conv{i}.y"
        if not onnx_ops:
            std = gamma * np.sqrt(2.0 / (cin * k * k))
            inits[w] = (rng.standard_normal((cout, cin, k, k), dtype=np.float32) * std).astype(np.float32)
            inits[b] = (rng.standard_normal(cout, dtype=np.float32) * 0.01).astype(np.float32)
            nodes.append(Node("Conv", [x, w, b], [y], attrs))
        else:
            std = np.sqrt(2.0 / (cin * k * k))
            inits[w] = (rng.standard_normal((cout, cin, k, k), dtype=np.float32) * std).astype(np.float32)
            bn = f"bn{i}"
            mean = (rng.standard_normal(cout, dtype=np.float32) * 0.1).astype(np.float32)
            var = rng.uniform(0.5, 1.5, cout).astype(np.float32)
            inits[bn + ".scale"] = (gamma * np.sqrt(var + 1e-5) * rng.uniform(0.9, 1.1, cout)).astype(np.float32)
            inits[bn + ".B"] = (rng.standard_normal(cout, dtype=np.float32) * 0.01).astype(np.float32)
            inits[bn + ".mean"] = mean
            inits[bn + ".var"] = var
            nodes.append(Node("Conv", [x, w], [y + ".pre"], attrs))
            nodes.append(Node("BatchNormalization", [y + ".pre", bn + ".scale", bn + ".B", bn + ".mean", bn + ".var"],
                              [y], {"epsilon": 1e-5}))
        if relu:
            nodes.append(Node("Relu", [y], [y + ".relu"]))
            return y + ".relu"
        return y

    x = conv("data", 3, 64, 7, 2, 3, True)
    nodes.append(Node("MaxPool", [x], ["pool0"], {"kernel_shape": [3, 3], "strides": [2, 2], "pads": [1, 1, 1, 1],
                                                  "auto_pad": "NOTSET"}))
    x, cin = "pool0", 64
    for stage, (blocks, width) in enumerate([(3, 64), (4, 128), (6, 256), (3, 512)]):
        for blk in range(blocks):
            s = 2 if (blk == 0 and stage > 0) else 1
            cout = width * 4
            h = conv(x, cin, width, 1, s, 0, True)
            h = conv(h, width, width, 3, 1, 1, True)
            h = conv(h, width, cout, 1, 1, 0, False, gamma=0.2)
            sc = conv(x, cin, cout, 1, s, 0, False, gamma=0.5) if (blk == 0) else x
            name = f"res{stage}_{blk}"
            nodes.append(Node("Add", [h, sc], [name + ".sum"]))
            nodes.append(Node("Relu", [name + ".sum"], [name]))
            x, cin = name, cout
    fc_w = (rng.standard_normal((2048, num_classes), dtype=np.float32) * np.sqrt(1.0 / 2048)).astype(np.float32)
    if not onnx_ops:
        inits["gap_axes"] = np.array([2, 3], np.int64)
        nodes.append(Node("ReduceMean", [x, "gap_axes"], ["gap"], {"keepdims": 0}))
        inits["fc.w"] = fc_w
        inits["fc.b"] = np.zeros(num_classes, np.float32)
        nodes.append(Node("MatMul", ["gap", "fc.w"], ["fc.mm"]))
        nodes.append(Node("Add", ["fc.mm", "fc.b"], ["logits"]))
    else:
        nodes.append(Node("GlobalAveragePool", [x], ["gap"]))
        nodes.append(Node("Flatten", ["gap"], ["flat"], {"axis": 1}))
        inits["fc.weight"] = np.ascontiguousarray(fc_w.T)  # [num_classes, 2048] as torch stores it
        inits["fc.bias"] = (rng.standard_normal(num_classes, dtype=np.float32) * 0.01).astype(np.float32)
        nodes.append(Node("Gemm", ["flat", "fc.weight", "fc.bias"], ["logits"],
                          {"alpha": 1.0, "beta": 1.0, "transB": 1}))
    return GraphDef(nodes, inits, ["data"], ["logits"], opset=18)


def resnet50_flops_per_img(h=224, w=224):
    """Conv + FC FLOPs of resnet50() per image (2 per multiply-add)."""
    g = resnet50()
    shapes = {"data": (3, h, w)}
    total = 0
    for n in g.nodes:
        if n.op == "Conv":
            c, hh, ww = shapes[n.inputs[0]]
            wt = g.initializers[n.inputs[1]]
            k, s, p = n.attrs["kernel_shape"][0], n.attrs["strides"][0], n.attrs["pads"][0]
            ho, wo = (hh + 2 * p - k) // s + 1, (ww + 2 * p - k) // s + 1
            total += 2 * ho * wo * wt.shape[0] * c * k * k
            shapes[n.outputs[0]] = (wt.shape[0], ho, wo)
        elif n.op == "MaxPool":
            c, hh, ww = shapes[n.inputs[0]]
            shapes[n.outputs[0]] = (c, (hh + 2 - 3) // 2 + 1, (ww + 2 - 3) // 2 + 1)
        elif n.op in ("Relu", "Add") and n.inputs[0] in shapes:
            shapes[n.outputs[0]] = shapes[n.inputs[0]]
    return total + 2 * 2048 * 1000

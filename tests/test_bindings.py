"""CPU checks of the reference-facing bindings: the C# P/Invoke file
(bindings/csharp/Native.cs) declares exactly the entry points of
include/lonnx.h with the same argument counts, and the Python ctypes table
(onnx_b200/_native.py) covers every one of them too."""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _split_args(s):
    s = s.strip()
    if not s or s == "void":
        return []
    depth, cur, out = 0, "", []
    for ch in s:
        if ch in "(<[":
            depth += 1
        elif ch in ")>]":
            depth -= 1
        if ch == "," and depth == 0:
            out.append(cur)
            cur = ""
        else:
            cur += ch
    out.append(cur)
    return [a.strip() for a in out]


def header_functions():
    src = open(os.path.join(ROOT, "include", "lonnx.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return {m.group(1): len(_split_args(m.group(2)))
            for m in re.finditer(r"LONNX_API\s+[^;()]*?\b(lonnx_\w+)\s*\(([^)]*)\)\s*;", src)}


def csharp_functions():
    src = open(os.path.join(ROOT, "bindings", "csharp", "Native.cs")).read()
    return {m.group(1): len(_split_args(m.group(2)))
            for m in re.finditer(r"\[DllImport\(Lib\)\]\s*public static extern [\w\*]+ (lonnx_\w+)\(([^)]*)\);", src,
                                 flags=re.S)}


def test_csharp_pinvoke_matches_header():
    h, cs = header_functions(), csharp_functions()
    assert len(h) > 40
    assert sorted(set(h) - set(cs)) == [], "declared in lonnx.h but not bound in Native.cs"
    assert sorted(set(cs) - set(h)) == [], "bound in Native.cs but not declared in lonnx.h"
    wrong = {n: (h[n], cs[n]) for n in h if h[n] != cs[n]}
    assert wrong == {}, f"argument counts differ (header, C#): {wrong}"


def test_ctypes_table_covers_header():
    src = open(os.path.join(ROOT, "onnx_b200", "_native.py")).read()
    table = set(re.findall(r'"(lonnx_\w+)":\s*\(', src))
    missing = sorted(set(header_functions()) - table)
    assert missing == [], f"no ctypes signature for {missing}"


def test_csharp_provider_covers_cpu_provider_ops():
    """Every op of the reference's SupportedOps (CPUExecutionProvider.cs:24-50)
    has a CUDAExecutionProvider method and a Node.ExecuteCUDA case."""
    ops = ["Reshape", "Add", "Div", "Sub", "Mul", "Pow", "Conv", "Relu", "MaxPool", "MatMul", "Sqrt", "Erf",
           "Transpose", "Constant", "Cast", "Concat", "Shape", "Gather", "Slice", "Unsqueeze", "ReduceSum",
           "ReduceMean", "ReduceMax", "Softmax"]
    prov = open(os.path.join(ROOT, "bindings", "csharp", "CUDAExecutionProvider.cs")).read()
    node = open(os.path.join(ROOT, "bindings", "csharp", "Node.CUDA.cs")).read()
    for op in ops:
        assert re.search(rf"public static OpResult {op}\(", prov), op
        assert f"OpType.{op} =>" in node, op

"""IR JSON + meta.json front-end (the reference's L1 contract).

Follows compile.py's ABI helpers:

* the IR file is an Emmy ``Graph`` dict whose KernelOp node stores its body
  as ``repr()`` text in ``op_fields.body`` (compile.py:3170-3172);
* the KernelOp entry name is ``op_fields.name`` (compile.py:320-324);
* ``meta.json`` next to the IR supplies the kernel record matched on
  ``entry``, or the only record (compile.py:302-311);
* parameter order is ``meta.arg_order``, else inputs then outputs
  (compile.py:314-317);
* shapes/dtypes merge graph outputs, KernelOp tensors, meta args and Smem
  declarations in that order (compile.py:273-299).

The body text is decoded with :mod:`ast` (never ``eval``): calls of known IR
class names build :mod:`emmy_ptx_compiler_b200.ir` nodes, ``dtype('float32')``
becomes the dtype name, and ``float('inf')`` style calls become floats.
"""

from __future__ import annotations

import ast
import json
from pathlib import Path

from . import ir
from .errors import UnsupportedIR


def _conv(node: ast.AST):
    if isinstance(node, ast.Constant):
        return node.value
    if isinstance(node, (ast.Tuple, ast.List)):
        return tuple(_conv(e) for e in node.elts)
    if isinstance(node, ast.Dict):
        return {_conv(k): _conv(v) for k, v in zip(node.keys, node.values)}
    if isinstance(node, ast.UnaryOp) and isinstance(node.op, (ast.USub, ast.UAdd)):
        v = _conv(node.operand)
        if not isinstance(v, (int, float)):
            raise UnsupportedIR(f"unary sign on non-number in IR text: {ast.dump(node)}")
        return -v if isinstance(node.op, ast.USub) else v
    if isinstance(node, ast.Call):
        if isinstance(node.func, ast.Name):
            fname = node.func.id
        elif isinstance(node.func, ast.Attribute):
            fname = node.func.attr
        else:
            raise UnsupportedIR(f"unsupported call in IR text: {ast.dump(node.func)}")
        args = [_conv(a) for a in node.args]
        kwargs = {k.arg: _conv(k.value) for k in node.keywords}
        if fname == "dtype":
            return str(args[0]) if args else None
        if fname == "float":
            return float(args[0])
        if fname == "int":
            return int(args[0])
        cls = ir.NODE_CLASSES.get(fname)
        if cls is None:
            raise UnsupportedIR(f"unknown IR node {fname!r}")
        try:
            return cls(*args, **kwargs)
        except TypeError as exc:
            raise UnsupportedIR(f"bad {fname} in IR text: {exc}") from exc
    if isinstance(node, ast.Name):
        if node.id in ("None", "True", "False"):
            return {"None": None, "True": True, "False": False}[node.id]
        if node.id in ("inf", "nan"):
            return float(node.id)
        raise UnsupportedIR(f"unknown name {node.id!r} in IR text")
    raise UnsupportedIR(f"unsupported syntax in IR text: {type(node).__name__}")


def decode_body(text: str):
    try:
        tree = ast.parse(text.strip(), mode="eval")
    except SyntaxError as exc:
        raise UnsupportedIR(f"IR body is not a node expression: {exc}") from exc
    return _conv(tree.body)


class GraphInfo:
    """The decoded pieces of one IR JSON document."""

    def __init__(self, raw: dict, kop: ir.KernelOp, constants: dict[str, object]):
        self.raw = raw
        self.kop = kop
        self.constants = constants


def load_graph(raw: dict) -> GraphInfo:
    nodes = raw.get("nodes") or {}
    tensors: dict[str, ir.Tensor] = {}
    for nd in nodes.values():
        for out in nd.get("outputs") or []:
            if out.get("name"):
                tensors[out["name"]] = ir.Tensor(out["name"], tuple(int(x) for x in out.get("shape") or ()),
                                                 out.get("dtype") or "f32")
    kop = None
    constants: dict[str, object] = {}
    for name, nd in nodes.items():
        kind = nd.get("op")
        fields = nd.get("op_fields") or {}
        if kind == "KernelOp" and kop is None:
            body: list = []
            for text in fields.get("body") or []:
                b = decode_body(text)
                body.extend(b if isinstance(b, tuple) else (b,))
            ins = {i: tensors.get(i, ir.Tensor(i)) for i in nd.get("inputs") or []}
            outs = {o["name"]: tensors[o["name"]] for o in nd.get("outputs") or [] if o.get("name")}
            kop = ir.KernelOp(fields.get("name", name), tuple(body), ins, outs)
        elif kind == "ConstantOp":
            constants[fields.get("name", name)] = fields.get("value")
    if kop is None:
        raise UnsupportedIR("no KernelOp in IR")
    return GraphInfo(raw, kop, constants)


def load_meta_kernel(ir_path: Path, entry: str) -> dict | None:
    meta_path = Path(ir_path).parent / "meta.json"
    if not meta_path.is_file():
        return None
    meta = json.loads(meta_path.read_text(encoding="utf-8"))
    kernels = meta.get("kernels") or []
    for k in kernels:
        if k.get("entry") == entry:
            return k
    return kernels[0] if len(kernels) == 1 else None


def arg_order_for(kop: ir.KernelOp, meta_kernel: dict | None) -> list[str]:
    if meta_kernel and meta_kernel.get("arg_order"):
        return list(meta_kernel["arg_order"])
    return list(kop.inputs) + list(kop.outputs)


def load_shapes(raw: dict | None, kop: ir.KernelOp, meta_kernel: dict | None
                ) -> tuple[dict[str, tuple[int, ...]], dict[str, str]]:
    shapes: dict[str, tuple[int, ...]] = {}
    dtypes: dict[str, str] = {}
    for node in ((raw or {}).get("nodes") or {}).values():
        for out in node.get("outputs") or []:
            name = out.get("name")
            if name and out.get("shape") is not None:
                shapes[name] = tuple(int(x) for x in out["shape"])
                dtypes[name] = out.get("dtype") or "f32"
    for mapping in (kop.inputs, kop.outputs):
        for name, tensor in mapping.items():
            if name not in shapes:
                sh = tuple(int(d) for d in (getattr(tensor, "shape", ()) or ()))
                if sh:
                    shapes[name] = sh
            dtypes.setdefault(name, ir.dtype_name(getattr(tensor, "dtype", None)) or "f32")
    if meta_kernel:
        for arg in meta_kernel.get("args") or []:
            name = arg.get("name")
            if name and arg.get("shape") is not None:
                shapes.setdefault(name, tuple(int(x) for x in arg["shape"]))
                dtypes.setdefault(name, arg.get("dtype") or "f32")
    for sm in ir.walk(kop.body):
        if isinstance(sm, ir.Smem):
            shapes[sm.name] = tuple(int(e) for e in sm.extents)
            dtypes[sm.name] = "f32" if sm.dtype in ("float", "float32", "") else sm.dtype
    return shapes, dtypes

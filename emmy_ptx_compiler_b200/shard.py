"""Split one KernelOp over the GPUs of a node: the KernelOp each GPU runs on
its own contiguous part of the data.

A KernelOp shards when one loop axis ``a`` can be cut into contiguous
pieces that need no data from one another:

* **rows** - ``a`` is a Tile axis and every Write indexes its output's first
  dimension with ``a`` (pointwise chains, row reductions, the GEMM's M).
  GPU ``d`` runs the same KernelOp with ``a``'s extent cut to its rows; every
  buffer whose first dimension is indexed by ``a`` holds only those rows.
  Outputs are final; nothing is exchanged.
* **partial** - every output is a scalar (a full-array reduction) and ``a``
  is the loop axis that walks the reduced input.  GPU ``d`` reduces its
  slice; the per-GPU results are then combined with the reduction's own
  operator (the one exchange on the path).

No data moves to make a shard: a GPU's buffers are views of (or copies of)
rows ``[lo, hi)`` of the whole problem, and the shard's KernelOp indexes them
from 0.  Which GPU owns which rows is ``split(extent, parts, part)``: as even
as possible, contiguous, in rank order.
"""

from __future__ import annotations

from dataclasses import dataclass, field

from . import ir
from .errors import UnsupportedIR


def split(extent: int, parts: int, part: int) -> tuple[int, int]:
    """Rows ``[lo, hi)`` of ``extent`` owned by ``part`` of ``parts``."""
    if parts <= 0 or not 0 <= part < parts:
        raise ValueError(f"part {part} of {parts}")
    return extent * part // parts, extent * (part + 1) // parts


@dataclass
class Shard:
    kop: ir.KernelOp
    shapes: dict
    axis: str
    mode: str            # "rows" | "partial"
    extent: int          # the axis' extent in the whole problem
    lo: int
    hi: int
    buffers: list[str] = field(default_factory=list)   # buffers cut along their first dimension
    combine: str | None = None                          # "partial": the reduction operator


def _first_index_var(index) -> str | None:
    if not index:
        return None
    ix = index[0]
    return ix.name if isinstance(ix, ir.Var) else None


def _axis_extents(body) -> dict[str, int]:
    out: dict[str, int] = {}
    for s in ir.walk(body):
        if isinstance(s, ir.Tile):
            for a in s.axes:
                out[a.name] = a.size
        elif isinstance(s, (ir.Loop, ir.StridedLoop)):
            out[s.axis.name] = s.axis.size
    return out


def shard_axis(kop: ir.KernelOp, shapes: dict) -> tuple[str, str, str | None]:
    """(axis, mode, combine op) of ``kop``, or UnsupportedIR when it does not shard."""
    body = ir.body_stmts(kop.body)
    tiles = [s for s in body if isinstance(s, ir.Tile)]
    if len(tiles) != 1 or len(body) != 1:
        raise UnsupportedIR("only a KernelOp that is one Tile shards")
    tile = tiles[0]
    smem = {s.name for s in ir.walk(tile.body) if isinstance(s, ir.Smem)}
    writes = [s for s in ir.walk(tile.body) if isinstance(s, ir.Write) and s.output not in smem]
    if not writes or any(s.atomic for s in writes):
        raise UnsupportedIR("no plain Write to shard")
    tile_axes = [a.name for a in tile.axes]
    firsts = {_first_index_var(s.index) for s in writes}
    if len(firsts) == 1 and next(iter(firsts)) in tile_axes:
        return next(iter(firsts)), "rows", None
    if all(len(tuple(shapes.get(s.output, ()))) == 0 or tuple(shapes.get(s.output, ())) == (1,) for s in writes):
        loops = [s for s in ir.walk(tile.body) if isinstance(s, ir.StridedLoop)]
        accs = [s for s in ir.walk(tile.body) if isinstance(s, ir.Accum)]
        ops = {ir.op_name(a.op) for a in accs}
        if len(loops) == 1 and len(ops) == 1 and ops <= {"add", "sum", "max", "maximum", "min", "minimum"}:
            return loops[0].axis.name, "partial", next(iter(ops))
    raise UnsupportedIR("no axis indexes the first dimension of every output")


def _rebuild(node, axis: str, extent: int):
    """A copy of ``node`` with every Axis named ``axis`` given ``extent``."""
    if isinstance(node, ir.Axis):
        return ir.Axis(node.name, ir.Dim(extent)) if node.name == axis else node
    if isinstance(node, tuple):
        return tuple(_rebuild(x, axis, extent) for x in node)
    if isinstance(node, ir.Node) and not isinstance(node, (ir.Expr, ir.Dim, ir.DataType, ir.ElementwiseImpl)):
        vals = {f: _rebuild(getattr(node, f), axis, extent) for f in node.FIELDS}
        return type(node)(**vals)
    return node


def shard_kernel(kop: ir.KernelOp, shapes: dict, parts: int, part: int, axis: str | None = None) -> Shard:
    """The KernelOp and shapes GPU ``part`` of ``parts`` runs (see module doc)."""
    found, mode, combine = shard_axis(kop, shapes)
    axis = axis or found
    extent = _axis_extents(kop.body).get(axis)
    if extent is None:
        raise UnsupportedIR(f"no loop axis {axis!r}")
    lo, hi = split(extent, parts, part)
    if hi == lo:
        raise UnsupportedIR(f"{parts} parts of {extent} leave part {part} empty")
    # buffers whose first dimension is indexed by the axis in every access
    seen: dict[str, bool] = {}
    for s in ir.walk(kop.body):
        if isinstance(s, (ir.Load, ir.Write)):
            buf = s.input if isinstance(s, ir.Load) else s.output
            ok = _first_index_var(s.index) == axis and tuple(shapes.get(buf, ()))[:1] == (extent,)
            seen[buf] = seen.get(buf, True) and ok
    cut = sorted(b for b, ok in seen.items() if ok)
    if mode == "partial" and len(cut) != 1:
        raise UnsupportedIR("a partial reduction must stream exactly one input along the axis")
    new_shapes = dict(shapes)
    for b in cut:
        new_shapes[b] = (hi - lo,) + tuple(shapes[b])[1:]
    body = _rebuild(tuple(kop.body), axis, hi - lo)
    k2 = ir.KernelOp(kop.name, body, dict(kop.inputs), dict(kop.outputs))
    return Shard(k2, new_shapes, axis, mode, extent, lo, hi, cut, combine)

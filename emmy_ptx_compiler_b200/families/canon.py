"""Canonical forms of scheduled IRs, so the fast families see through a schedule.

Emmy can stage a matmul's operands through shared memory with ``cp.async``
(compile.py:2288-2319 lowers the copies): each block copies a tile of A and a
tile of B into shared buffers, waits, synchronises and runs a short k loop over
the staged tiles.  The arithmetic is still ``acc = fma(a, b, acc)`` over k in
ascending order, so the result is the naive matmul's bit for bit.  The staging
only changes where each operand is read from.

``staged_matmul`` proves that and returns the equivalent naive-matmul IR
(the shape tools/make_proxy_set.py:338-365 builds), which the GEMM family then
lowers.  It answers None, and the IR keeps its own schedule, unless every step
of the proof holds:

* the structure is one Tile; then ``Init acc``; then a k-tile loop holding
  the copies, a barrier, an inner loop of two shared-memory loads, a multiply
  and an add Accum, and a barrier; then an epilogue and one ``Write C[r, c]``.
  The copies are ``CpAsyncCopy`` of f32 (optionally under a Cond on thread
  coordinates) followed by ``cp.async.wait_group 0``, or plain copies: a
  global ``Load`` whose value a shared ``Write`` stores unchanged;
* every index expression is affine in the Tile axes and the two loop
  variables (``+``, ``-``, ``*`` by a literal).  The trailing Tile axes that
  make up one thread block index the threads; the leading ones index blocks;
* within one block, at k tile 0, every shared element a thread reads was
  copied by exactly one thread, from ``A[r, kk]`` (or ``B[kk, c]``), where
  r and c are the row and column that thread writes;
* each block axis shifts the copies' sources by exactly the shift it gives
  the written row or column, and the k-tile loop shifts them by one k tile.
  For affine maps the base point and these shifts determine every point;
* the blocks tile C exactly once (two block axes: one row-tile axis, one
  column-tile axis), and k tiles times the inner extent is K.
"""

from __future__ import annotations

from itertools import product

from .. import ir

F32 = ir.DataType("f32", "float32", 4)
_CMP = {"<": lambda a, b: a < b, "<=": lambda a, b: a <= b, ">": lambda a, b: a > b,
        ">=": lambda a, b: a >= b, "==": lambda a, b: a == b, "!=": lambda a, b: a != b}


def _affine(e) -> bool:
    if isinstance(e, ir.Literal):
        return isinstance(e.value, int) and not isinstance(e.value, bool)
    if isinstance(e, ir.Var):
        return True
    if isinstance(e, ir.BinaryExpr):
        if e.op in ("+", "-"):
            return _affine(e.left) and _affine(e.right)
        if e.op == "*":
            return (_affine(e.left) and _affine(e.right)
                    and (isinstance(e.left, ir.Literal) or isinstance(e.right, ir.Literal)))
    return False


def _ev(e, env: dict) -> int:
    if isinstance(e, ir.Literal):
        return int(e.value)
    if isinstance(e, ir.Var):
        return env[e.name]
    a, b = _ev(e.left, env), _ev(e.right, env)
    return a + b if e.op == "+" else (a - b if e.op == "-" else a * b)


def _flat(index, shape, env) -> int:
    if len(index) != len(shape):
        raise ValueError("index rank")
    out = 0
    for ix, ext in zip(index, shape):
        out = out * int(ext) + _ev(ix, env)
    return out


def _vars(exprs) -> set[str]:
    out: set[str] = set()
    for e in exprs:
        out |= e.var_names() if isinstance(e, ir.Expr) else set()
    return out


def _launch_threads(tile, meta) -> int:
    if tile.block_threads:
        return int(tile.block_threads)
    b = (meta or {}).get("block") or []
    n = 1
    for x in b:
        n *= int(x)
    return n if b else 0


def staged_matmul(kop: ir.KernelOp, shapes: dict, dtypes: dict, meta: dict | None) -> ir.KernelOp | None:
    try:
        return _staged_matmul(kop, shapes, dtypes, meta)
    except (KeyError, ValueError, AttributeError, TypeError, ZeroDivisionError):
        return None


def _staged_matmul(kop, shapes, dtypes, meta):
    body = ir.body_stmts(kop.body)
    if len(body) != 1 or not isinstance(body[0], ir.Tile):
        return None
    tile = body[0]
    if tile.aux_threads or tile.raster_group:
        return None
    axes = [(a.name, a.size) for a in tile.axes]
    nthr = _launch_threads(tile, meta)
    split, acc_n = len(axes), 1
    while split > 0 and acc_n < nthr:
        split -= 1
        acc_n *= axes[split][1]
    if not nthr or acc_n != nthr:
        return None
    block_axes, thread_axes = axes[:split], axes[split:]
    smem = {s.name: tuple(int(x) for x in s.extents) for s in ir.walk(tile.body) if isinstance(s, ir.Smem)}
    stmts = [s for s in ir.body_stmts(tile.body) if not isinstance(s, ir.Smem)]
    loops = [s for s in stmts if isinstance(s, ir.Loop)]
    if len(loops) != 1 or any(isinstance(s, ir.StridedLoop) for s in stmts):
        return None
    kt_loop = loops[0]
    li = stmts.index(kt_loop)
    pre, post = stmts[:li], stmts[li + 1:]
    kl = list(ir.body_stmts(kt_loop.body))
    inner = [s for s in kl if isinstance(s, ir.Loop)]
    if len(inner) != 1:
        return None
    kk_loop = inner[0]
    head, tail = kl[:kl.index(kk_loop)], kl[kl.index(kk_loop) + 1:]
    # copies, commit, wait 0, barrier ... k loop ... barrier
    if not head or not (isinstance(head[-1], ir.Sync) and not head[-1].warp and not head[-1].barrier_id):
        return None
    if len(tail) != 1 or not (isinstance(tail[0], ir.Sync) and not tail[0].warp and not tail[0].barrier_id):
        return None
    copies, waited, asyncs = [], False, False
    staged = list(head[:-1])
    i = 0
    while i < len(staged):
        s = staged[i]
        if isinstance(s, ir.CpAsyncCopy) and not waited:
            copies.append((_Copy.of_async(s), None))
            asyncs = True
        elif (isinstance(s, ir.Cond) and not s.else_body and not waited
              and all(isinstance(t, ir.CpAsyncCopy) for t in s.body)):
            copies += [(_Copy.of_async(t), s.cond) for t in s.body]
            asyncs = True
        elif isinstance(s, ir.CpAsyncCommit) and not waited:
            pass
        elif isinstance(s, ir.CpAsyncWait) and int(s.group) == 0:
            waited = True
        elif isinstance(s, ir.Load) and i + 1 < len(staged) and not waited:
            # a plain copy: one element loaded from global memory, stored unchanged into shared memory
            cp = _Copy.of_pair(s, staged[i + 1])
            if cp is None:
                return None
            copies.append((cp, None))
            i += 1
        else:
            return None
        i += 1
    if not copies or (asyncs and not waited):
        return None
    kb = list(ir.body_stmts(kk_loop.body))
    if len(kb) != 4 or not all(isinstance(s, ir.Load) for s in kb[:2]):
        return None
    la, lb, mul, accum = kb
    if not (isinstance(mul, ir.Assign) and ir.op_name(mul.op) == "multiply" and len(mul.args) == 2
            and isinstance(accum, ir.Accum) and ir.op_name(accum.op) in ("add", "sum")
            and accum.value == mul.name and accum.base in (None, accum.name)
            and len(la.names) == 1 and len(lb.names) == 1 and set(mul.args) == {la.names[0], lb.names[0]}
            and la.input in smem and lb.input in smem and la.input != lb.input):
        return None
    seed = 0.0
    for s in pre:
        if isinstance(s, ir.Init) and s.name == accum.name:
            seed = float(s.identity)
        else:
            return None
    writes = [s for s in ir.walk(post) if isinstance(s, ir.Write)]
    if len(writes) != 1 or not post or writes[0] is not post[-1] or writes[0].atomic or len(writes[0].values) != 1:
        return None
    out = writes[0]
    if len(out.index) != 2 or not all(_affine(e) for e in out.index):
        return None
    M, N = (int(x) for x in shapes[out.output])
    # the copies: f32 only, affine, sources are the two global operands
    src_of = {}
    for cp, cond in copies:
        if cp.lane_index is not None or cp.smem not in smem or cp.src in smem:
            return None
        if ir.canon_dtype(dtypes.get(cp.src)) != "f32" or int(cp.nbytes) % 4:
            return None
        if not all(_affine(e) for e in tuple(cp.smem_index) + tuple(cp.src_index)):
            return None
        if _vars(cp.smem_index) - {a for a, _ in thread_axes}:
            return None
        if _vars(cp.src_index) - {a for a, _ in axes} - {kt_loop.axis.name}:
            return None
        if cond is not None:
            if not (isinstance(cond, ir.BinaryExpr) and cond.op in _CMP and _affine(cond.left)
                    and _affine(cond.right)) or _vars((cond,)) - {a for a, _ in thread_axes}:
                return None
        src_of.setdefault(cp.smem, cp.src)
        if src_of[cp.smem] != cp.src:
            return None
    if set(src_of) != {la.input, lb.input}:
        return None
    ga, gb = src_of[la.input], src_of[lb.input]
    KT, KK = kt_loop.axis.size, kk_loop.axis.size
    K = KT * KK
    if ga == gb or tuple(shapes[ga]) != (M, K) or tuple(shapes[gb]) != (K, N):
        return None
    thread_vars = {a for a, _ in thread_axes}
    if (_vars(la.index) | _vars(lb.index)) - thread_vars - {kk_loop.axis.name}:
        return None
    if not all(_affine(e) for e in tuple(la.index) + tuple(lb.index)):
        return None
    if _vars(out.index) - {a for a, _ in axes}:
        return None
    # one block at k tile 0: who copies what
    base = {a: 0 for a, _ in block_axes}
    base[kt_loop.axis.name] = 0
    writer: dict[tuple[str, int], int] = {}
    threads = [dict(zip([a for a, _ in thread_axes], t)) for t in product(*[range(e) for _, e in thread_axes])]
    for t in threads:
        env = {**base, **t}
        for cp, cond in copies:
            if cond is not None and not _CMP[cond.op](_ev(cond.left, env), _ev(cond.right, env)):
                continue
            s0 = _flat(cp.smem_index, smem[cp.smem], env)
            g0 = _flat(cp.src_index, shapes[cp.src], env)
            for e in range(int(cp.nbytes) // 4):
                key = (cp.smem, s0 + e)
                if key in writer or not 0 <= s0 + e < _size(smem[cp.smem]):
                    return None
                writer[key] = g0 + e
    # rows and columns each thread writes, and the reads it makes
    for t in threads:
        env = {**base, **t}
        r, c = _ev(out.index[0], env), _ev(out.index[1], env)
        for kk in range(KK):
            env[kk_loop.axis.name] = kk
            ga_flat = writer.get((la.input, _flat(la.index, smem[la.input], env)))
            gb_flat = writer.get((lb.input, _flat(lb.index, smem[lb.input], env)))
            if ga_flat != r * K + kk or gb_flat != kk * N + c:
                return None
    # shifts: every block axis moves the copies' sources as it moves the written cell,
    # the k-tile loop moves them one k tile along
    t0 = {**base, **threads[0]}

    def delta(exprs, shape, var):
        return _flat(exprs, shape, {**t0, var: 1}) - _flat(exprs, shape, t0)
    rows_axis = cols_axis = None
    for a, ext in block_axes:
        dr = _ev(out.index[0], {**t0, a: 1}) - _ev(out.index[0], t0)
        dc = _ev(out.index[1], {**t0, a: 1}) - _ev(out.index[1], t0)
        for cp, _ in copies:
            want = dr * K if cp.src == ga else dc
            if delta(cp.src_index, shapes[cp.src], a) != want:
                return None
        if dr and not dc:
            rows_axis = (a, ext, dr)
        elif dc and not dr:
            cols_axis = (a, ext, dc)
        else:
            return None
    for cp, _ in copies:
        want = KK if cp.src == ga else KK * N
        if delta(cp.src_index, shapes[cp.src], kt_loop.axis.name) != want:
            return None
    # the blocks tile C exactly once
    if len(block_axes) != 2 or rows_axis is None or cols_axis is None:
        return None
    cells = {(_ev(out.index[0], {**base, **t}), _ev(out.index[1], {**base, **t})) for t in threads}
    tr, tc = rows_axis[2], cols_axis[2]
    if cells != {(r, c) for r in range(tr) for c in range(tc)} or len(threads) != tr * tc:
        return None
    if rows_axis[1] * tr != M or cols_axis[1] * tc != N:
        return None
    # epilogue: row / column vectors indexed exactly as the output, and pointwise statements
    names = {a for a, _ in axes} | {kt_loop.axis.name, kk_loop.axis.name}
    ci, cj, ck = _fresh("i", names), _fresh("j", names), _fresh("k", names)
    row_txt, col_txt = out.index[0].pretty(), out.index[1].pretty()
    epi = []
    for s in post[:-1]:
        if isinstance(s, ir.Load):
            if len(s.index) != 1 or s.input in smem:
                return None
            txt = s.index[0].pretty()
            if txt == col_txt:
                epi.append(ir.Load(names=s.names, input=s.input, index=(ir.Var(cj),), dtype=s.dtype))
            elif txt == row_txt:
                epi.append(ir.Load(names=s.names, input=s.input, index=(ir.Var(ci),), dtype=s.dtype))
            else:
                return None
        elif isinstance(s, (ir.Assign, ir.Let)) and not (s.reads() & names):
            epi.append(s)
        else:
            return None
    a_name, b_name = la.names[0], lb.names[0]
    canon = ir.Tile(axes=(ir.Axis(ci, ir.Dim(M)), ir.Axis(cj, ir.Dim(N))), body=(
        ir.Init(accum.name, seed, dtype=F32),
        ir.Loop(axis=ir.Axis(ck, ir.Dim(K)), body=(
            ir.Load(names=(a_name,), input=ga, index=(ir.Var(ci), ir.Var(ck)), dtype=la.dtype),
            ir.Load(names=(b_name,), input=gb, index=(ir.Var(ck), ir.Var(cj)), dtype=lb.dtype),
            ir.Assign(mul.name, mul.op, mul.args, mul.dtype),
            ir.Accum(accum.name, accum.value, accum.op, accum.dtype, axes=(ck,)),
        )),
        *epi,
        ir.Write(output=out.output, index=(ir.Var(ci), ir.Var(cj)), values=out.values, value_dtype=out.value_dtype),
    ))
    return ir.KernelOp(name=kop.name, body=(canon,), inputs=kop.inputs, outputs=kop.outputs)


class _Copy:
    """One staging copy: shared buffer and index, global source and index, bytes."""

    def __init__(self, smem, smem_index, src, src_index, nbytes, lane_index=None):
        self.smem, self.smem_index = smem, tuple(smem_index)
        self.src, self.src_index = src, tuple(src_index)
        self.nbytes, self.lane_index = int(nbytes), lane_index

    @classmethod
    def of_async(cls, s) -> "_Copy":
        return cls(s.smem, s.smem_index, s.src, s.src_index, s.nbytes, s.lane_index)

    @classmethod
    def of_pair(cls, ld, wr) -> "_Copy | None":
        if not (isinstance(wr, ir.Write) and not wr.atomic and len(ld.names) == 1 and len(wr.values) == 1
                and wr.values[0] == ld.names[0]):
            return None
        if ir.canon_dtype(ld.dtype) not in (None, "f32") or ir.canon_dtype(wr.value_dtype) not in (None, "f32"):
            return None
        return cls(wr.output, wr.index, ld.input, ld.index, 4)


def _size(shape) -> int:
    n = 1
    for x in shape:
        n *= int(x)
    return n


def _fresh(stem: str, used: set[str]) -> str:
    k = 0
    while f"_c{stem}{k}" in used:
        k += 1
    return f"_c{stem}{k}"

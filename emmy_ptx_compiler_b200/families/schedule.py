"""Schedule family: any block-cooperative KernelOp, lowered statement by
statement in the schedule Emmy chose, with the reference's thread model.

The other families recognise a computation (a pointwise chain, a reduction, a
GEMM, a fused row pass, naive attention) and generate their own sm_100a
schedule for it.  This family is the drop-in for every other KernelOp the
reference lowers.  It keeps the IR's own schedule:

* thread ids as the reference's prologue builds them (compile.py:1010-1077):
  the linear thread index of the (up to 3-D) block, the linear block index,
  ``gid = cta * nthreads + tid``, ``lane = tid & 31``, ``warp = tid >> 5``,
  and the ``threadIdx.*``/``blockIdx.*``/``blockDim.*`` builtins;
* each ``Tile`` (compile.py:1520-1629): axes decoded row-major from ``gid``
  (the first axis undivided), raster groups, ``aux_threads``, and the guard
  for leftover threads.  It is a branch around the body, or a predicate on
  memory accesses when the body holds barriers, shuffles or async copies;
* ``Loop`` / ``StridedLoop`` in order with accumulator seeding
  (compile.py:1769-1783, 1813-1914), ``Cond``, ``Select``, the Assign op
  table and both FMA contractions (shared with the other families);
* ``Smem`` buffers (``__shared__``), ``Sync`` (``bar.sync``), ``WarpShuffle``
  (``shfl.sync.bfly`` steps from length/2 down, then the combine Assigns,
  compile.py:2213-2231), ``TreeHalve`` (smem halving steps with a barrier
  after each, compile.py:2233-2276);
* ``CpAsyncCopy`` / ``CpAsyncCommit`` / ``CpAsyncWait`` (``cp.async.ca|cg``,
  compile.py:2288-2319, 1460-1465) and ``ZeroPrologue`` (compile.py:2890-2913).

Arithmetic follows the reference instruction for instruction, so results match
its PTX bit for bit where the arithmetic is IEEE-exact.  The exception is the
reference's warp-reduce rewrite of single-warp 32-trip loops (compile.py:743-806),
which changes its summation order; that is not mirrored here.  The tensor-core
and TMA nodes (``MmaSyncPtx``, ``LdmatrixLoad``, ``TmaLoad``, mbarriers,
``Wgmma*``) are sm_90 forms and stay unsupported: ``wgmma`` does not exist on
sm_100a.
"""

from __future__ import annotations

from dataclasses import dataclass

from .. import ir
from ..cgen import DEVICE_PRELUDE, Emitter, carry_slot, ctype, f32_lit, fusable_products, identity_of, lit_int
from ..errors import UnsupportedIR
from .common import KernelSource, LaunchPlan, ParamSpec, launch_record_source
from .common import c_ident as _c

SUPPORTED = (ir.Tile, ir.Smem, ir.Sync, ir.WarpShuffle, ir.TreeHalve, ir.Load, ir.Write, ir.Assign,
             ir.Accum, ir.Init, ir.Let, ir.Loop, ir.StridedLoop, ir.Cond, ir.Select, ir.ZeroPrologue,
             ir.CpAsyncCopy, ir.CpAsyncCommit, ir.CpAsyncWait, ir.Pre, ir.Carry)
COLLECTIVE = (ir.Sync, ir.TreeHalve, ir.WarpShuffle, ir.CpAsyncCopy, ir.CpAsyncCommit, ir.CpAsyncWait)
STATIC_SMEM_MAX = 48 * 1024
_SMEM_BYTES = {"f32": 4, "float": 4, "float32": 4, "i32": 4, "u32": 4, "s32": 4, "int": 4, "u64": 8,
               "i64": 8, "f16": 2, "bf16": 2, "half": 2}
_SMEM_CTYPE = {4: "float", 8: "unsigned long long", 2: "unsigned short"}


@dataclass
class SchedPlan:
    smem: list          # ir.Smem declarations, in order
    tiles: int


def unsupported_nodes(kop: ir.KernelOp) -> list[str]:
    return sorted({type(s).__name__ for s in ir.walk(kop.body) if not isinstance(s, SUPPORTED)})


def match(kop: ir.KernelOp, shapes: dict, dtypes: dict) -> SchedPlan | None:
    top = ir.body_stmts(kop.body)
    if not top or unsupported_nodes(kop):
        return None
    smem, seen = [], set()
    for s in ir.walk(kop.body):
        if isinstance(s, ir.Smem):
            if s.name in seen:
                continue
            seen.add(s.name)
            smem.append(s)
    return SchedPlan(smem, sum(isinstance(s, ir.Tile) for s in top))


class SchedEmitter(Emitter):
    """The shared Emitter plus the block-cooperative statements."""

    def __init__(self, shapes: dict, dtypes: dict, ptrs: dict[str, str], load_hook=None, write_hook=None,
                 indent: str = "    ", smem: set[str] | None = None, active: str | None = None):
        super().__init__(shapes, dtypes, ptrs, load_hook, write_hook, indent)
        self.custom_hooks = (load_hook, write_hook)
        self.smem = smem or set()
        self.active = active
        self.counter = [0]
        # Pre / Carry (compile.py:2860-2888): (carrier, slot) -> C variable of the
        # Carry emitted last, and each carrier's seed; resolved in emission order
        self.carry_vals: dict[tuple[str, str], str] = {}
        self.carry_seed: dict[str, float] = {}
        self.carry_var: dict[int, str] = {}
        self.carry_prod: dict[str, tuple] = {}

    def _child(self) -> "SchedEmitter":
        # a child with the default hooks binds its own (its environment holds the loop variables)
        c = SchedEmitter(self.shapes, self.dtypes, self.ptrs, *self.custom_hooks,
                         indent=self.ind + "    ", smem=self.smem, active=self.active)
        c.declared = self.declared
        c.tmp = self.tmp + 1000
        c.fusable = self.fusable
        c.products = self.products
        c.ftype = self.ftype
        c.row_divisors = self.row_divisors
        c.counter = self.counter
        c.carry_vals = self.carry_vals
        c.carry_seed = self.carry_seed
        c.carry_var = self.carry_var
        c.carry_prod = self.carry_prod
        c.env = dict(self.env)
        return c

    def uid(self, stem: str) -> str:
        self.counter[0] += 1
        return f"_{stem}{self.counter[0]}"

    # thread builtins are bound in the environment under their own names
    def expr(self, e):
        if isinstance(e, ir.Builtin):
            if e.name in self.env:
                return self.env[e.name]
            raise UnsupportedIR(f"unknown thread builtin {e.name!r}")
        return super().expr(e)

    # memory accesses of leftover threads are predicated off (compile.py:1541-1549)
    def _default_load(self, s: ir.Load, k: int):
        kind, code = super()._default_load(s, k)
        if self.active:
            zero = "0.0f" if kind == "f32" else "0LL"
            return kind, f"({self.active} ? {code} : {zero})"
        return kind, code

    def _default_write(self, s: ir.Write, k: int, kind: str, code: str) -> str:
        line = super()._default_write(s, k, kind, code)
        return f"if ({self.active}) {{ {line} }}" if self.active else line

    def stmt(self, s) -> None:
        if isinstance(s, ir.Smem):
            return                                    # declared once at the top of the kernel
        if isinstance(s, ir.Sync):
            self.emit(_sync_code(s.barrier_id, s.count, s.warp))
            return
        if isinstance(s, ir.Loop):
            ext = s.axis.size
            if ext > 0:
                self._loop(s.axis.name, "0LL", f"{ext}LL", "1LL", s.body, s.seed)
            return
        if isinstance(s, ir.StridedLoop):
            end = (self.index_code(s.end) if s.end is not None else f"{s.axis.size}LL")
            self._loop(s.axis.name, self.index_code(s.start), end, self.index_code(s.step), s.body, s.seed)
            return
        if isinstance(s, ir.WarpShuffle):
            self._warp_shuffle(s)
            return
        if isinstance(s, ir.TreeHalve):
            self._tree_halve(s)
            return
        if isinstance(s, ir.CpAsyncCopy):
            self._cp_async(s)
            return
        if isinstance(s, ir.CpAsyncCommit):
            self.emit('asm volatile("cp.async.commit_group;" ::: "memory");')
            return
        if isinstance(s, ir.CpAsyncWait):
            self.emit(f'asm volatile("cp.async.wait_group {int(s.group)};" ::: "memory");')
            return
        if isinstance(s, ir.ZeroPrologue):
            self._zero_prologue(s)
            return
        if isinstance(s, ir.Carry):
            self.carry_seed[s.name] = float(s.seed)
            var = self._carry_decl(s)
            self.emit(f"{var} = {self.as_f32(s.value)};")
            self.carry_vals[(s.name, carry_slot(s.index))] = var
            self.env[s.name] = ("f32", var)
            # a carried plain product stays foldable into the add/sub that reads it back
            prod = self.products.get(s.value) if isinstance(s.value, str) else None
            if prod is not None:
                self.carry_prod[var] = prod
            else:
                self.carry_prod.pop(var, None)
            return
        if isinstance(s, ir.Pre):
            key = (s.carrier, carry_slot(s.index))
            src = self.carry_vals.get(key) or self.carry_vals.get((s.carrier, "_"))
            self.assign(s.name, "f32", src if src is not None else f32_lit(self.carry_seed.get(s.carrier, 0.0)))
            if src is not None and src in self.carry_prod:
                self.products[s.name] = self.carry_prod[src]
            return
        super().stmt(s)

    def _carry_decl(self, s) -> str:
        """One function-scope variable per Carry statement (declared before any
        enclosing loop or branch, so later Pre statements can read it)."""
        if id(s) not in self.carry_var:
            self.carry_var[id(s)] = self.declare(f"__carry{len(self.carry_var)}_{s.name}", "f32")
        return self.carry_var[id(s)]

    def _defines(self, s) -> list[tuple[str, str]]:
        if isinstance(s, (ir.Pre, ir.Carry)):
            return [(s.name, "f32")]
        return super()._defines(s)

    def _predeclare(self, body) -> None:
        for t in ir.walk(body):
            if isinstance(t, ir.Carry):
                self._carry_decl(t)
                continue
            for nm, kind in self._defines(t):
                self.declare(nm, kind)
            if isinstance(t, (ir.WarpShuffle, ir.TreeHalve)):
                for nm in tuple(t.state) + tuple(t.state_b):
                    self.declare(nm, "f32")

    def _loop(self, var: str, start: str, end: str, step: str, body, seed: bool) -> None:
        if seed:
            # accumulators of the body start at their identity before the loop (compile.py:1769-1783)
            for t in ir.body_stmts(body):
                if isinstance(t, ir.Accum) and t.name not in self.env:
                    dt = ir.dtype_name(t.dtype)
                    if dt in (None, "", *ir.F32_NAMES):
                        self.assign(t.name, "f32", f32_lit(identity_of(t.op)))
                    else:
                        self.assign(t.name, "int", f"{int(identity_of(t.op))}LL")
        self._predeclare(body)
        iv = self.uid("i")
        self.emit(f"for (long long {iv} = {start}; {iv} < {end}; {iv} += {step}) {{")
        inner = self._child()
        inner.env[var] = ("int", iv)
        inner.run(body)
        self.lines.extend(inner.lines)
        self.emit("}")
        for k, v in inner.env.items():
            if k != var and (k not in self.env or v[1] in self.declared.values()):
                self.env[k] = v

    def _warp_shuffle(self, s: ir.WarpShuffle) -> None:
        mask = self.uid("mask")
        self.emit(f"const unsigned {mask} = __activemask();")
        step = int(s.length) // 2
        while step > 0:
            for st, sb in zip(s.state, s.state_b):
                self.assign(sb, "f32", f"__shfl_xor_sync({mask}, {self.as_f32(st)}, {step})")
            for asn in s.combine_states:
                self.stmt(asn)
            step >>= 1

    def _slot(self, s: ir.TreeHalve, tid: str, extra: int) -> str:
        base = f"({tid} + {extra})" if extra else f"({tid})"
        if s.inner is not None:
            iv, scale = s.inner
            return f"({base} * {int(scale)}LL + {self.as_int(iv)})"
        return base

    def _tree_halve(self, s: ir.TreeHalve) -> None:
        tid = self.as_int(s.tid_var)
        for nm in tuple(s.state) + tuple(s.state_b):
            self.declare(nm, "f32")
        step = int(s.length) // 2
        while step > 0:
            self.emit(f"if (({tid}) < {step}) {{")
            inner = self._child()
            for buf, st, sb in zip(s.bufs, s.state, s.state_b):
                inner.assign(st, "f32", f"{self.ptrs[buf]}[{self._slot(s, tid, 0)}]")
                inner.assign(sb, "f32", f"{self.ptrs[buf]}[{self._slot(s, tid, step)}]")
            for asn in s.combine_states:
                inner.stmt(asn)
            for buf, st in zip(s.bufs, s.state):
                inner.emit(f"{self.ptrs[buf]}[{self._slot(s, tid, 0)}] = {inner.as_f32(st)};")
            self.lines.extend(inner.lines)
            self.emit("}")
            self.emit(_sync_code(s.barrier_id, s.barrier_count, False))
            step >>= 1
        for buf, st in zip(s.bufs, s.state):
            root = self.as_int(s.inner[0]) if s.inner is not None else "0"
            self.assign(st, "f32", f"{self.ptrs[buf]}[{root}]")

    def _cp_async(self, s) -> None:
        didx = self.flat_index(s.smem, s.smem_index)
        if s.lane_index is not None:
            cols = int(self.shapes[s.smem][-1])
            didx = f"({didx} + ({self.index_code(s.lane_index[0])}) * {cols}LL + ({self.index_code(s.lane_index[1])}))"
        sidx = self.flat_index(s.src, s.src_index)
        n = int(s.nbytes)
        q = "cg" if n == 16 else "ca"
        line = (f'asm volatile("cp.async.{q}.shared.global [%0], [%1], {n};" :: '
                f'"r"((unsigned)__cvta_generic_to_shared(&{self.ptrs[s.smem]}[{didx}])), '
                f'"l"(&{self.ptrs[s.src]}[{sidx}]) : "memory");')
        self.emit(f"if ({self.active}) {{ {line} }}" if self.active else line)

    def _zero_prologue(self, s) -> None:
        if int(s.words) <= 0 or s.dst not in self.ptrs:
            return
        zi = self.uid("z")
        self.emit(f"for (long long {zi} = emmy_gid; {zi} < {int(s.words)}LL; "
                  f"{zi} += (long long)emmy_nthr * emmy_ncta)")
        self.emit(f"    reinterpret_cast<unsigned int *>({self.ptrs[s.dst]})[{zi}] = 0u;")


def _sync_code(barrier_id, count, warp) -> str:
    if warp:
        return "__syncwarp();"
    bid = int(barrier_id or 0)
    if bid == 0:
        return "__syncthreads();"
    if int(count or 0) > 0:
        return f'asm volatile("bar.sync {bid}, {int(count)};" ::: "memory");'
    return f'asm volatile("bar.sync {bid};" ::: "memory");'


def _launch_threads(meta: dict) -> int:
    b = list(meta.get("block") or [])
    out = 1
    for x in b:
        out *= int(x)
    return out if b else 0


def generate(kop: ir.KernelOp, plan: SchedPlan, shapes: dict, dtypes: dict, args: list[str],
             scalars: dict[str, str], written: set[str], meta: dict | None = None,
             device_fn: str | None = None) -> KernelSource:
    """The KernelOp in its own schedule.  With ``device_fn`` the code is a
    ``static __device__`` function of that name taking the same parameters
    (no prelude, no launch record), for a module that already has them."""
    meta = meta or {}
    shapes = dict(shapes)
    dtypes = dict(dtypes)
    params: list[ParamSpec] = []
    ptrs: dict[str, str] = {}
    sig: list[str] = []
    for name in args:
        if name in scalars:
            sig.append(f"{ctype(scalars[name])} p_{_c(name)}")
            params.append(ParamSpec(name, "scalar", scalars[name]))
            continue
        dt = ir.canon_dtype(dtypes.get(name))
        const = "" if name in written else "const "
        sig.append(f"{const}{ctype(dt)}* __restrict__ p_{_c(name)}")
        ptrs[name] = f"p_{_c(name)}"
        params.append(ParamSpec(name, "ptr", dt))
    scalar_env = {n: (("f32", f"p_{_c(n)}") if scalars[n] == "f32" else ("int", f"(long long)p_{_c(n)}"))
                  for n in scalars}
    # shared buffers: static below 48 KiB, else one dynamic region
    decl, offsets, total = [], {}, 0
    for sm in plan.smem:
        dt = ir.dtype_name(sm.dtype) or "f32"
        nb = _SMEM_BYTES.get(dt, 4)
        count = 1
        for x in sm.extents:
            count *= int(x)
        align = max(16, int(sm.align or 0))
        total = -(-total // align) * align
        offsets[sm.name] = (total, nb, count, align)
        total += nb * max(1, count)
        shapes[sm.name] = tuple(int(x) for x in sm.extents)
        dtypes[sm.name] = "f32" if nb == 4 and dt in ir.F32_NAMES else ("u32" if nb == 4 else dt)
        ptrs[sm.name] = f"s_{_c(sm.name)}"
    dyn = total if total > STATIC_SMEM_MAX else 0
    for sm in plan.smem:
        off, nb, count, align = offsets[sm.name]
        cty = _SMEM_CTYPE[nb] if not (nb == 4 and dtypes[sm.name] != "f32") else "unsigned int"
        if dyn:
            decl.append(f"    {cty} *const s_{_c(sm.name)} = reinterpret_cast<{cty} *>(emmy_dsm + {off});")
        else:
            decl.append(f"    __shared__ __align__({align}) {cty} s_{_c(sm.name)}[{max(1, count)}];")
    lines: list[str] = [] if device_fn else [DEVICE_PRELUDE]
    w = lines.append
    if device_fn:
        w(f"static __device__ void {device_fn}(" + ", ".join(sig) + ") {")
    else:
        w(f'extern "C" __global__ void {kop.name}(' + ", ".join(sig) + ") {")
    if dyn:
        w("    extern __shared__ __align__(128) unsigned char emmy_dsm[];")
    lines.extend(decl)
    # the reference's thread ids (compile.py:1010-1077)
    w("    const int emmy_tid = (int)((threadIdx.z * blockDim.y + threadIdx.y) * blockDim.x + threadIdx.x);")
    w("    const int emmy_nthr = (int)(blockDim.x * blockDim.y * blockDim.z);")
    w("    const int emmy_cta = (int)((blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x);")
    w("    const int emmy_ncta = (int)(gridDim.x * gridDim.y * gridDim.z);")
    w("    const long long emmy_gid = (long long)emmy_cta * emmy_nthr + emmy_tid;")
    w("    (void)emmy_nthr; (void)emmy_ncta; (void)emmy_gid;")
    base_env = dict(scalar_env)
    base_env.update({
        "_tid": ("int", "(long long)emmy_tid"), "_gid": ("int", "emmy_gid"), "_cta": ("int", "(long long)emmy_cta"),
        "_ntid": ("int", "(long long)emmy_nthr"), "_ncta": ("int", "(long long)emmy_ncta"),
        "lane": ("int", "(long long)(emmy_tid & 31)"), "warp": ("int", "(long long)(emmy_tid >> 5)"),
        "threadIdx.x": ("int", "(long long)threadIdx.x"), "threadIdx.y": ("int", "(long long)threadIdx.y"),
        "threadIdx.z": ("int", "(long long)threadIdx.z"), "blockDim.x": ("int", "(long long)blockDim.x"),
        "blockDim.y": ("int", "(long long)blockDim.y"), "blockDim.z": ("int", "(long long)blockDim.z"),
        "blockIdx.x": ("int", "(long long)blockIdx.x"), "blockIdx.y": ("int", "(long long)blockIdx.y"),
        "blockIdx.z": ("int", "(long long)blockIdx.z"),
    })
    smem_names = set(offsets)
    fus = fusable_products(kop.body)
    launch_block = _launch_threads(meta)
    first_n = None
    # statements outside any Tile run in every thread (compile.py:1077-1095); one scope for the kernel
    top_em = SchedEmitter(shapes, dtypes, ptrs, indent="    ", smem=smem_names)
    top_em.fusable = fus
    top_em.env.update(base_env)
    top_em._predeclare(tuple(t for t in ir.body_stmts(kop.body) if not isinstance(t, ir.Tile)))
    loose: list = []

    def flush_loose() -> None:
        if loose:
            top_em.run(tuple(loose))
            loose.clear()
        lines.extend(top_em.lines)
        top_em.lines = []

    for ti, top in enumerate(ir.body_stmts(kop.body)):
        if isinstance(top, ir.Smem):
            continue
        if not isinstance(top, ir.Tile):
            loose.append(top)
            continue
        flush_loose()
        tile = top
        extents = [a.size for a in tile.axes]
        n = 1
        for x in extents:
            n *= x
        first_n = first_n if first_n is not None else n
        cells = int(tile.block_threads) if tile.block_threads is not None else launch_block
        aux = int(tile.aux_threads or 0)
        w("    {")
        gid = "emmy_gid"
        if aux:
            bt = int(tile.block_threads or cells or 0)
            w(f"    const long long emmy_gid_t{ti} = (long long)emmy_cta * {bt}LL + (emmy_tid % {bt});")
            gid = f"emmy_gid_t{ti}"
        guard = aux != 0 or not cells or n % int(cells) != 0
        collective = any(isinstance(s, COLLECTIVE) for s in ir.walk(tile.body))
        active = None
        ind = "        "
        if guard and collective:
            active = f"emmy_active{ti}"
            w(f"        const bool {active} = {gid} < {n}LL;")
        elif guard:
            w(f"        if ({gid} < {n}LL) {{")
            ind = "            "
        em = top_em._child()
        em.declared = dict(top_em.declared)    # the tile's own scope
        em.ind = ind
        em.active = active
        if aux:
            em.env["_gid"] = ("int", gid)
        _bind_axes(em, tile, extents, gid)
        em.run(tile.body)
        lines.extend(em.lines)
        if guard and not collective:
            w("        }")
        w("    }")
    flush_loose()
    w("}")
    grid = tuple(int(x) for x in (meta.get("grid") or [])) or None
    block = tuple(int(x) for x in (meta.get("block") or [])) or None
    if block is None:
        first_tile = next((s for s in ir.body_stmts(kop.body) if isinstance(s, ir.Tile)), None)
        block = (int(first_tile.block_threads or 128) if first_tile is not None else 1, 1, 1)
    block = (tuple(block) + (1, 1))[:3]
    if grid is None:
        nthr = block[0] * block[1] * block[2]
        grid = (max(1, -(-(first_n or 1) // nthr)), 1, 1)
    grid = (tuple(grid) + (1, 1))[:3]
    launch = LaunchPlan(grid=grid, block=block, smem=dyn)
    if not device_fn:
        lines.append(launch_record_source("schedule", launch, params))
    notes = {"kernel": "schedule", "tiles": plan.tiles, "smem_static": 0 if dyn else total, "smem_dynamic": dyn}
    return KernelSource(entry=kop.name, source="\n".join(lines), launch=launch, params=params,
                        family="schedule", notes=notes)


def _bind_axes(em: SchedEmitter, tile: ir.Tile, extents: list[int], gid: str) -> None:
    """Tile axes from the thread id (compile.py:1556-1625)."""
    strides = [1] * len(extents)
    acc = 1
    for i in range(len(extents) - 1, -1, -1):
        strides[i] = acc
        acc *= extents[i]
    raster = None
    if tile.raster_group and tile.raster_axes:
        names = [a.name for a in tile.axes]
        if tile.raster_axes[0] in names and tile.raster_axes[1] in names:
            mi, ni = names.index(tile.raster_axes[0]), names.index(tile.raster_axes[1])
            if ni == mi + 1:
                gi, oi = (mi, ni) if tile.raster_orient == "m" else (ni, mi)
                g_eff = min(int(tile.raster_group), extents[gi])
                if extents[gi] > 1 and extents[oi] > 1 and g_eff > 1:
                    raster = (gi, oi, g_eff, mi, ni)
    a_code = b_code = None
    for i, axis in enumerate(tile.axes):
        s, ext = strides[i], extents[i]
        if raster is not None:
            gi, oi, g, mi, ni = raster
            if i == mi:
                ea, eb = extents[gi], extents[oi]
                sn = strides[ni]
                sub = gid if sn == 1 else f"({gid} / {sn}LL)"
                if mi != 0:
                    sub = f"({sub} % {ea * eb}LL)"
                geb = g * eb
                if ea % g == 0:
                    a_code = f"(({sub} / {geb}LL) * {g}LL + ({sub} % {g}LL))"
                    b_code = f"(({sub} % {geb}LL) / {g}LL)"
                else:
                    rs = em.uid("rsz")
                    rg = em.uid("rgrp")
                    em.emit(f"const long long {rg} = {sub} / {geb}LL;")
                    em.emit(f"const long long {rs} = ({ea}LL - {rg} * {g}LL) < {g}LL ? ({ea}LL - {rg} * {g}LL) : {g}LL;")
                    a_code = f"({rg} * {g}LL + (({sub} % {geb}LL) % {rs}))"
                    b_code = f"(({sub} % {geb}LL) / {rs})"
                em.bind_const(axis.name, "int", a_code if i == gi else b_code)
                continue
            if i == ni:
                em.bind_const(axis.name, "int", a_code if i == gi else b_code)
                continue
        if ext == 1:
            em.bind_const(axis.name, "int", "0LL")
            continue
        term = gid if s == 1 else f"({gid} / {s}LL)"
        em.bind_const(axis.name, "int", term if i == 0 else f"({term} % {ext}LL)")


__all__ = ["SchedPlan", "match", "generate", "unsupported_nodes", "lit_int"]

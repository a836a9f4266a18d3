"""Pieces shared by the kernel families: launch plans, parameter specs and the
launch record every emitted module carries (layout: include/emmy_launch_record.h)."""

from __future__ import annotations

from dataclasses import dataclass, field

SM_COUNT = 148  # B200: 2 dies x 74 SMs

FAMILY_ID = {"pointwise": 1, "reduction": 2, "gemm": 3, "rownorm": 4, "attention": 5, "schedule": 6}
PARAM_KIND = {"ptr": 0, "f32": 1, "i32": 2}


@dataclass
class LaunchPlan:
    grid: tuple[int, int, int]
    block: tuple[int, int, int]
    smem: int = 0
    cluster: tuple[int, int, int] = (1, 1, 1)
    # fill_waves > 0: the loader sets grid[0] = fill_waves x resident CTAs per SM
    # x SMs (a multiple of grid_quantum); grid[0] here is the fallback estimate
    fill_waves: int = 0
    grid_quantum: int = 1
    # unit ranges: the kernel takes (range_begin, range_end) after the tensor maps
    range_total: int = 0          # 0 = no range parameters
    range_align: int = 1
    range_bytes: list[int] = field(default_factory=list)  # per arg_order parameter
    # grid_units: a launch over a unit range runs min(grid[0], units in the range / grid_quantum) CTAs
    grid_units: bool = False
    # cooperative: the loader launches every CTA at once (cooperative launch) or fails
    cooperative: bool = False

FLAG_FILL_GRID = 0x100
FLAG_RANGE = 0x200
FLAG_GRID_UNITS = 0x400
FLAG_COOPERATIVE = 0x800


@dataclass
class ParamSpec:
    name: str
    kind: str  # "ptr" | "scalar"
    dtype: str


@dataclass
class TmapSpec:
    src_param: int
    dtype: int       # CUtensorMapDataType
    dims: list[int]  # innermost first
    strides: list[int]  # bytes, dims 1..rank-1
    box: list[int]
    swizzle: int     # CUtensorMapSwizzle
    l2_promotion: int = 2  # CU_TENSOR_MAP_L2_PROMOTION_L2_128B


@dataclass
class KernelSource:
    entry: str
    source: str
    launch: LaunchPlan
    params: list[ParamSpec]
    family: str
    notes: dict = field(default_factory=dict)
    tmaps: list[TmapSpec] = field(default_factory=list)


def launch_record_source(family: str, launch: LaunchPlan, params: list[ParamSpec],
                         tmaps: list[TmapSpec] | None = None) -> str:
    """C++ definition of the module's ``emmy_launch_record`` and ``emmy_status``."""
    tmaps = tmaps or []
    kinds = []
    for p in params:
        if p.kind == "ptr":
            kinds.append(PARAM_KIND["ptr"])
        elif p.dtype == "f32":
            kinds.append(PARAM_KIND["f32"])
        else:
            kinds.append(PARAM_KIND["i32"])
    if len(kinds) > 32:
        raise ValueError("more than 32 kernel parameters")
    kinds += [0] * (32 - len(kinds))
    tm_src = []
    for t in tmaps:
        dims = list(t.dims) + [1] * (5 - len(t.dims))
        strides = list(t.strides) + [0] * (4 - len(t.strides))
        box = list(t.box) + [1] * (5 - len(t.box))
        tm_src.append("{%du, %du, %du, %du, {%s}, {%s}, {%s}, %du, {0u, 0u, 0u}}" % (
            t.src_param, t.dtype, len(t.dims), t.swizzle,
            ", ".join(f"{d}ull" for d in dims), ", ".join(f"{s}ull" for s in strides),
            ", ".join(f"{b}u" for b in box), t.l2_promotion))
    while len(tm_src) < 4:
        tm_src.append("{0u, 0u, 0u, 0u, {0ull, 0ull, 0ull, 0ull, 0ull}, {0ull, 0ull, 0ull, 0ull}, "
                      "{0u, 0u, 0u, 0u, 0u}, 0u, {0u, 0u, 0u}}")
    g, b = launch.grid, launch.block
    flags = int(launch.cluster[0])
    if launch.range_total:
        flags |= FLAG_RANGE
        if launch.grid_units:
            flags |= FLAG_GRID_UNITS
    if launch.cooperative:
        flags |= FLAG_COOPERATIVE
    rbytes = list(launch.range_bytes) + [0] * (32 - len(launch.range_bytes))
    if launch.fill_waves:
        flags |= FLAG_FILL_GRID
        g = (launch.fill_waves, g[1], g[2])
    return (
        "\n#include \"emmy_launch_record.h\"\n"
        "extern \"C\" __device__ unsigned int emmy_status = 0u;\n"
        "extern \"C\" __device__ const EmmyLaunchRecord emmy_launch_record = {\n"
        f"    EMMY_LR_MAGIC, EMMY_LR_VERSION, {FAMILY_ID[family]}u, {flags}u,\n"
        f"    {{{g[0]}u, {g[1]}u, {g[2]}u}}, {{{b[0]}u, {b[1]}u, {b[2]}u}}, {launch.smem}u, {len(params)}u,\n"
        "    {" + ", ".join(f"{k}u" for k in kinds) + "},\n"
        f"    {len(tmaps)}u, {max(1, int(launch.grid_quantum))}u,\n"
        "    {" + ",\n     ".join(tm_src) + "},\n"
        f"    {int(launch.range_total)}ull, {max(1, int(launch.range_align))}u, 0u,\n"
        "    {" + ", ".join(f"{int(x)}ull" for x in rbytes) + "}\n"
        "};\n"
    )


def c_ident(name: str) -> str:
    """An IR name as a C identifier fragment (every other character becomes '_')."""
    import re
    return re.sub(r"[^A-Za-z0-9_]", "_", name)

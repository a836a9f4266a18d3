"""The C-ABI library loads without a GPU and exports every declared symbol (CPU only)."""

from __future__ import annotations

import ctypes
import re

from conftest import REPO


def _declared() -> list[str]:
    text = (REPO / "include" / "emmy_b200.h").read_text()
    return sorted(set(re.findall(r"^(?:int|const char \*)\s*(emmy_\w+)\(", text, re.M)))


def test_library_exports_every_declared_symbol():
    from emmy_ptx_compiler_b200 import runtime
    lib = ctypes.CDLL(str(runtime.lib()._name))
    declared = _declared()
    assert len(declared) >= 25
    for name in declared:
        assert hasattr(lib, name), name
    assert sorted(runtime.EXPORTED) == declared


def test_version_and_error_paths_without_driver():
    """No compute: only calls that must fail cleanly when there is no GPU."""
    import torch
    from emmy_ptx_compiler_b200 import runtime
    lib = runtime.lib()
    assert lib.emmy_version().startswith(b"emmy_b200")
    if torch.cuda.is_available():
        return
    rc = lib.emmy_launch(None, None, 0, None, None, 0)
    assert rc == -3  # EMMY_ERR_INVALID
    buf = ctypes.create_string_buffer(256)
    assert lib.emmy_last_error(buf, 256) == -3
    assert b"NULL" in buf.value
    rc = lib.emmy_alloc(0, 16, ctypes.byref(ctypes.c_uint64()))
    assert rc == -8  # EMMY_ERR_NOT_INIT


def test_launch_record_layout_matches_header():
    """Python's record emitter and the C header agree on field count/order."""
    from emmy_ptx_compiler_b200.families.common import LaunchPlan, ParamSpec, launch_record_source
    src = launch_record_source("pointwise", LaunchPlan((1, 1, 1), (256, 1, 1)), [ParamSpec("x", "ptr", "f32")])
    assert "EMMY_LR_MAGIC" in src and "emmy_status" in src
    hdr = (REPO / "include" / "emmy_launch_record.h").read_text()
    assert "uint32_t param_kind[EMMY_LR_MAX_PARAMS];" in hdr


def test_new_entry_points_reject_bad_arguments_without_a_gpu():
    """emmy_launch_ex needs explicit geometry; graphs need a caller stream and a
    graph; run_host and graph_end need their pointers.  All refuse with
    EMMY_ERR_INVALID before any driver call."""
    import torch
    from emmy_ptx_compiler_b200 import runtime
    lib = runtime.lib()
    if torch.cuda.is_available():
        return
    u32x3 = (ctypes.c_uint32 * 3)(1, 1, 1)
    assert lib.emmy_launch_ex(None, None, 0, u32x3, u32x3, 0, 0) == -3
    assert lib.emmy_graph_begin(0, 0) == -3                 # the legacy default stream cannot be recorded
    assert lib.emmy_graph_end(0, 1, None) == -3
    assert lib.emmy_graph_launch(None, 1) == -3
    assert lib.emmy_graph_destroy(None) == 0                # destroying nothing is fine
    assert lib.emmy_run_host(None, None, None, None, 0, 0) == -3
    buf = ctypes.create_string_buffer(256)
    lib.emmy_last_error(buf, 256)
    assert b"NULL" in buf.value
    # a negative or oversized parameter count is refused before anything reads the tables
    mods = (ctypes.c_void_p * 1)(ctypes.c_void_p(16))
    words = (ctypes.c_uint64 * 1)(0)
    rows = (ctypes.POINTER(ctypes.c_uint64) * 1)(words)
    for bad in (-1, 65, 1 << 30):
        assert lib.emmy_launch_sharded(mods, 1, rows, bad, None) == -3
        lib.emmy_last_error(buf, 256)
        assert b"parameters" in buf.value

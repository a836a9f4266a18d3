from emmy._core import (  # noqa: F401
    Accum, Assign, Carry, Cond, Init, Let, Load, Loop, Pre, StridedLoop, Write, ZeroPrologue,
)

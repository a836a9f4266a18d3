from emmy._core import (  # noqa: F401
    BinaryExpr, Builtin, CastExpr, FlatIndex, FuncCallExpr, Literal, SimplifyCtx, TernaryExpr, Var,
)

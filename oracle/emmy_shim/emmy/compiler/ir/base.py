from emmy._core import ConstantOp, InputOp  # noqa: F401

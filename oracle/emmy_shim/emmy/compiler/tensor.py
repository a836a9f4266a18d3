from emmy._core import Tensor  # noqa: F401

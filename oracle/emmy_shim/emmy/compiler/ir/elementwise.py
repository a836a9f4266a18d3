from emmy._core import ElementwiseImpl  # noqa: F401

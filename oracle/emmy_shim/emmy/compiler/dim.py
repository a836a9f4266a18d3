from emmy._core import Dim  # noqa: F401

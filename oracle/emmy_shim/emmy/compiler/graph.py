from emmy._core import Graph, Node  # noqa: F401

from emmy._core import Select, SelectBranch  # noqa: F401

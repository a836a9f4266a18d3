"""GEMM family (placeholder while the tcgen05 kernel is written)."""


def match(kop, shapes, dtypes):
    return None


def generate(*a, **k):
    raise NotImplementedError

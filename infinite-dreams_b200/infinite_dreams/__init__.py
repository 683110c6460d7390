"""B200 (sm_100a) FP16 GEMM kernel bank with the reference's package surface.

Mirrors infinite_dreams/__init__.py of the reference (:9-12): the compiled
operator module ``infinite_dreams_ext`` is imported lazily on first access.
Put ``infinite-dreams_b200/`` on ``sys.path`` in place of the reference's
checkout and ``from infinite_dreams import infinite_dreams_ext`` works as
before.
"""
import importlib

import torch as _torch  # noqa: F401

__all__ = ["infinite_dreams_ext"]


def __getattr__(name: str):
    if name == "infinite_dreams_ext":
        return importlib.import_module(".infinite_dreams_ext", __name__)
    raise AttributeError(name)

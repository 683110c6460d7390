"""Packaging for the infinite_dreams package and its sm_100a kernel bank.

The reference hooked its generator into setup.py (setup.py:22-46): generate
the bank sources, then hand every bank file to torch's BuildExtension.  Here
both ``build_ext`` (``python setup.py build_ext --inplace``, the in-tree
build) and ``build_py`` (``pip install .``) run build.py: the generator
writes csrc/generated/, nvcc compiles each translation unit in parallel for
sm_100a, and the objects are linked into infinite_dreams/_lib/libgemm_sm100.so,
which ships as package data.  Unchanged translation units are not rebuilt.
"""
import importlib.util
import os
from pathlib import Path

from setuptools import setup
from setuptools.command.build_ext import build_ext
from setuptools.command.build_py import build_py

HERE = Path(__file__).resolve().parent


def _build_bank() -> None:
    spec = importlib.util.spec_from_file_location("infinite_dreams_bank_build", HERE / "build.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    jobs = int(os.environ.get("INFINITE_DREAMS_BUILD_JOBS", "0")) or None
    mod.build(jobs=jobs)
    mod.build_torch_ext()


class BuildBankExt(build_ext):
    """build_ext without Python extension modules: builds the C-ABI kernel bank."""

    def run(self):
        _build_bank()


class BuildPyWithBank(build_py):
    def run(self):
        _build_bank()
        super().run()


setup(
    name="infinite_dreams",
    version="0.1.0",
    description="sm_100a (B200) FP16 GEMM kernel bank with a C ABI, DE tuner and per-shape dispatch",
    packages=["infinite_dreams"],
    package_dir={"": "."},
    package_data={"infinite_dreams": ["_lib/libgemm_sm100.so", "_torch_ext*.so", "dispatch_table.json"]},
    python_requires=">=3.10",
    install_requires=["numpy", "torch"],
    cmdclass={"build_ext": BuildBankExt, "build_py": BuildPyWithBank},
)

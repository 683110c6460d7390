"""Builds libgemm_sm100.so (the C-ABI kernel bank) in-tree for sm_100a.

Replaces the reference's build path (setup.py:22-46 running the generator
then torch's BuildExtension over every bank file).  Here the generator runs
first, then every translation unit (one per generated bank file plus the C
ABI) is compiled by nvcc in parallel and linked into one shared library at
``infinite_dreams/_lib/libgemm_sm100.so``.  The library is self-contained
(static CUDA runtime, driver entry points looked up at run time), so it
loads without torch.

The torch binding (csrc/torch_ext.cpp -> infinite_dreams/_torch_ext*.so) is
built after the library and links to it.

Usage:  python infinite-dreams_b200/build.py [--jobs N] [--force] [--verbose-ptxas]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path
from typing import List

PKG_ROOT = Path(__file__).resolve().parent
CSRC = PKG_ROOT / "csrc"
GEN = CSRC / "generated"
BUILD = PKG_ROOT / "_build"
LIB_DIR = PKG_ROOT / "infinite_dreams" / "_lib"
LIB = LIB_DIR / "libgemm_sm100.so"
INCLUDE = PKG_ROOT.parent / "include"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O2",
                           "--expt-relaxed-constexpr", "-I", str(CSRC), "-I", str(INCLUDE)]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the kernel bank needs the CUDA toolkit to build")
    return cand


def sources() -> List[Path]:
    return [CSRC / "gemm_capi.cu", CSRC / "gemm_noalloc.cu"] + sorted(GEN.glob("gemm_bank_*.cu"))


def headers_digest() -> str:
    h = hashlib.sha256()
    for p in sorted(list(CSRC.glob("*.cuh")) + list(GEN.glob("*.inc")) + list(INCLUDE.glob("*.h"))):
        h.update(p.name.encode())
        h.update(p.read_bytes())
    h.update(" ".join(NVCC_FLAGS).encode())
    return h.hexdigest()


def compile_one(src: Path, obj: Path, digest: str, force: bool, ptxas_v: bool) -> str:
    stamp = obj.with_suffix(".stamp")
    key = hashlib.sha256(src.read_bytes() + digest.encode()).hexdigest()
    if not force and obj.exists() and stamp.exists() and stamp.read_text() == key:
        return f"up to date: {src.name}"
    cmd = [nvcc()] + NVCC_FLAGS + (["-Xptxas", "-v"] if ptxas_v else []) + ["-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    stamp.write_text(key)
    return f"compiled: {src.name}" + (("\n" + r.stderr) if ptxas_v else "")


def build(jobs: int | None = None, force: bool = False, ptxas_v: bool = False, quiet: bool = False) -> Path:
    sys.path.insert(0, str(PKG_ROOT))
    from infinite_dreams import gen_gemm_bank  # noqa: E402

    gen_gemm_bank.write()
    BUILD.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    digest = headers_digest()
    srcs = sources()
    objs = [BUILD / (s.stem + ".o") for s in srcs]
    jobs = jobs or max(1, min(len(srcs), os.cpu_count() or 1))
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        for msg in ex.map(lambda so: compile_one(so[0], so[1], digest, force, ptxas_v), zip(srcs, objs)):
            if not quiet:
                print(msg)
    link_key = hashlib.sha256(b"".join(o.read_bytes() for o in objs)).hexdigest()
    link_stamp = BUILD / "link.stamp"
    if force or not LIB.exists() or not link_stamp.exists() or link_stamp.read_text() != link_key:
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc()] + ARCH_FLAGS + ["-shared", "-o", str(tmp)] + [str(o) for o in objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
        link_stamp.write_text(link_key)
        if not quiet:
            print(f"linked: {LIB}")
    return LIB


def torch_ext_path() -> Path:
    import sysconfig
    return PKG_ROOT / "infinite_dreams" / ("_torch_ext" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_torch_ext(force: bool = False, quiet: bool = False) -> Path:
    """Compiles csrc/torch_ext.cpp (the torch binding of the C ABI) against
    the installed torch and links it to libgemm_sm100.so through $ORIGIN."""
    import sysconfig

    import torch
    from torch.utils import cpp_extension as ce

    src = CSRC / "torch_ext.cpp"
    out = torch_ext_path()
    key = hashlib.sha256(src.read_bytes() + (INCLUDE / "gemm_sm100.h").read_bytes() +
                         torch.__version__.encode() + sysconfig.get_config_var("EXT_SUFFIX").encode()).hexdigest()
    stamp = BUILD / "torch_ext.stamp"
    if not force and out.exists() and stamp.exists() and stamp.read_text() == key:
        if not quiet:
            print(f"up to date: {out.name}")
        return out
    cuda_inc = str(Path(nvcc()).resolve().parent.parent / "include")
    incs = ce.include_paths() + [cuda_inc, sysconfig.get_paths()["include"]]
    libdirs = [str(Path(torch.__file__).parent / "lib")]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = (["g++", "-O2", "-fPIC", "-shared", "-std=c++17", "-DTORCH_EXTENSION_NAME=_torch_ext",
            "-DTORCH_API_INCLUDE_EXTENSION_H", f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-w"] +
           [f"-I{d}" for d in incs] + [str(src), "-o", str(out) + ".tmp"] +
           [f"-L{d}" for d in libdirs] + ["-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python", "-lc10_cuda",
                                          "-ltorch_cuda", f"-L{LIB_DIR}", "-lgemm_sm100",
                                          "-Wl,-rpath,$ORIGIN/_lib"])
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"torch extension build failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    os.replace(str(out) + ".tmp", out)
    BUILD.mkdir(parents=True, exist_ok=True)
    stamp.write_text(key)
    if not quiet:
        print(f"built: {out}")
    return out


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    args = ap.parse_args()
    build(args.jobs, args.force, args.verbose_ptxas)
    build_torch_ext(args.force)


if __name__ == "__main__":
    main()

"""Build recipe: libmfcuda.so (sm_100a kernels + C ABI), libminfer_host.so (C++
host runtime) and the oracle libraries.

Everything is built in-tree (minfer_b200/lib, oracle/_build, oracle/_ref) so
the shared objects travel with the working tree. Objects are rebuilt only when
a source or header is newer than the target.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
HOST = CSRC / "host"
INCLUDE = ROOT / "include"
OBJ = PKG / "_build"
LIB = PKG / "lib"
ORACLE = ROOT / "oracle"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
                     f"-I{INCLUDE}", f"-I{CSRC}"]
CXX_FLAGS = ["-std=c++17", "-O3", "-march=x86-64-v3", "-fPIC", "-Wall", "-Wextra", "-Wno-unused-parameter",
             f"-I{INCLUDE}", f"-I{HOST}"]

CUDA_SOURCES = ["capi.cu", "attention.cu", "attn_noalloc.cu", "gemv_f32.cu", "gemv_f16.cu", "gemv_bf16.cu",
                "gemv_tma_f32.cu", "gemv_tma_f16.cu", "gemv_tma_bf16.cu",
                "gemv_tp_f32.cu", "gemv_tp_f16.cu", "gemv_tp_bf16.cu", "prefill.cu", "prefill_moe.cu"]
HOST_SOURCES = ["gguf.cpp", "sampler.cpp", "model.cpp", "capi_model.cpp", "tokenizer.cpp", "chat_template.cpp"]

LIBMFCUDA = LIB / "libmfcuda.so"
LIBHOST = LIB / "libminfer_host.so"


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def cxx() -> str:
    # the image may export CXX as a wrapper; the system g++ is what we test with
    return os.environ.get("MF_CXX") or shutil.which("g++") or "g++"


def _newer(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps if d.exists())


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("build step failed: " + " ".join(cmd[:3]) + " ...")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def build_cuda(force: bool = False, jobs: int = 8) -> Path:
    OBJ.mkdir(exist_ok=True)
    LIB.mkdir(exist_ok=True)
    hdrs = _headers()
    todo = []
    objs = []
    for src in CUDA_SOURCES:
        s = CSRC / src
        o = OBJ / (src + ".o")
        objs.append(o)
        if force or _newer(o, [s] + hdrs):
            todo.append([nvcc(), *NVCC_FLAGS, "-c", str(s), "-o", str(o)])
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        list(ex.map(_run, todo))
    if force or todo or _newer(LIBMFCUDA, objs):
        _run([nvcc(), *ARCH, "-shared", "-o", str(LIBMFCUDA), *map(str, objs), "-lcuda"])
    return LIBMFCUDA


def build_host(force: bool = False, jobs: int = 8) -> Path:
    OBJ.mkdir(exist_ok=True)
    hdrs = sorted(HOST.glob("*.hpp")) + sorted(HOST.glob("*.inc")) + sorted(INCLUDE.glob("*.h"))
    todo, objs = [], []
    for src in HOST_SOURCES:
        s = HOST / src
        o = OBJ / (src + ".o")
        objs.append(o)
        if force or _newer(o, [s] + hdrs):
            todo.append([cxx(), *CXX_FLAGS, "-c", str(s), "-o", str(o)])
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        list(ex.map(_run, todo))
    if force or todo or _newer(LIBHOST, objs + [LIBMFCUDA]):
        _run([cxx(), "-shared", "-o", str(LIBHOST), *map(str, objs), f"-L{LIB}", "-lmfcuda",
              "-Wl,-rpath,$ORIGIN"])
    return LIBHOST


def _reference(reference: str | None) -> str | None:
    # the reference checkout: the argument, else $MF_REFERENCE; none by default
    return reference or os.environ.get("MF_REFERENCE") or None


def build_oracle(reference: str | None = None) -> None:
    """The oracle restatement always; the reference's own CPU path when a
    reference checkout is given (argument or $MF_REFERENCE) and present."""
    targets = ["port"]
    ref = _reference(reference)
    if ref and Path(ref, "src", "ops", "kernels.cpp").exists():
        targets.append("ref")
    _run(["make", "-s", "-C", str(ORACLE), *([f"REF={ref}"] if ref else []), *targets])


def build_integration(reference: str | None = None) -> None:
    """minfer's own host loop linked against the CUDA runtime
    (integration/cuda_backend.cpp), where a reference checkout is given."""
    ref = _reference(reference)
    if ref and Path(ref, "src", "base", "model.cpp").exists():
        _run(["make", "-s", "-C", str(ROOT / "integration"), f"REF={ref}"])


def build_all(force: bool = False, oracle: bool = True, reference: str | None = None) -> None:
    build_cuda(force)
    build_host(force)
    if oracle:
        build_oracle(reference)
        build_integration(reference)


if __name__ == "__main__":
    # python -m minfer_b200.build [--force] [--no-oracle] [--reference DIR]
    ref = sys.argv[sys.argv.index("--reference") + 1] if "--reference" in sys.argv else None
    build_all(force="--force" in sys.argv, oracle="--no-oracle" not in sys.argv, reference=ref)
    print("built", LIBMFCUDA, LIBHOST)

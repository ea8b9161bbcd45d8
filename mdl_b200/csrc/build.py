"""Ahead-of-time build of the mdl_b200 native extension (sm_100a only).

Every ``*.cu`` file under this directory is compiled by nvcc with
``-gencode arch=compute_100a,code=sm_100a``; ``bindings.cpp`` (the only
translation unit that includes torch headers) is compiled by the host
compiler; the objects are linked into ``mdl_b200/_mdl_C.so`` next to the
package, so the built library travels with the source tree. A content hash of
all sources and flags is stored beside the library; a rebuild happens only
when that hash changes (file times are not trusted, since copies of the tree
do not keep them).
"""

from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PKG = CSRC.parent
BUILD_DIR = PKG / "_build"
LIB_NAME = "_mdl_C"
LIB_PATH = PKG / f"{LIB_NAME}.so"
STAMP_PATH = PKG / f"{LIB_NAME}.stamp"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _cuda_home() -> Path:
    env = os.environ.get("CUDA_HOME") or os.environ.get("CUDA_PATH")
    if env:
        return Path(env)
    nvcc = shutil.which("nvcc")
    if nvcc:
        return Path(nvcc).resolve().parent.parent
    return Path("/usr/local/cuda")


def _torch_paths() -> tuple[list[str], list[str], bool]:
    import torch
    from torch.utils import cpp_extension

    includes = [p for p in cpp_extension.include_paths() if "cuda" not in p.lower() or "torch" in p]
    libs = [str(Path(torch.__file__).parent / "lib")]
    return includes, libs, bool(torch._C._GLIBCXX_USE_CXX11_ABI)


def _sources() -> tuple[list[Path], list[Path], list[Path]]:
    cu = sorted(CSRC.glob("*.cu"))
    cpp = sorted(CSRC.glob("*.cpp"))
    headers = sorted(list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")))
    return cu, cpp, headers


def _nvcc_flags(cuda: Path) -> list[str]:
    return [
        str(cuda / "bin" / "nvcc"),
        *ARCH_FLAGS,
        "-O3",
        "-lineinfo",
        "-std=c++17",
        "--expt-relaxed-constexpr",
        "-Xcompiler",
        "-fPIC",
        "-Xptxas",
        "-v",
        f"-I{CSRC}",
        f"-I{cuda / 'include'}",
    ]


def _source_hash(extra: list[str]) -> str:
    cu, cpp, headers = _sources()
    digest = hashlib.sha256()
    for path in [*cu, *cpp, *headers, Path(__file__)]:
        digest.update(path.name.encode())
        digest.update(path.read_bytes())
    for item in extra:
        digest.update(item.encode())
    return digest.hexdigest()


def is_up_to_date() -> bool:
    if not LIB_PATH.exists() or not STAMP_PATH.exists():
        return False
    return STAMP_PATH.read_text().strip() == _source_hash(ARCH_FLAGS)


def _run(cmd: list[str], log: Path) -> None:
    result = subprocess.run(cmd, capture_output=True, text=True)
    log.write_text(" ".join(cmd) + "\n" + result.stdout + result.stderr)
    if result.returncode != 0:
        sys.stderr.write(result.stdout + result.stderr)
        raise RuntimeError(f"build step failed: {' '.join(cmd[:3])} ... (log: {log})")


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every kernel for sm_100a and link the extension library."""

    if not force and is_up_to_date():
        return LIB_PATH
    cuda = _cuda_home()
    includes, libdirs, cxx11_abi = _torch_paths()
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    cu, cpp, _headers = _sources()
    jobs: list[tuple[list[str], Path]] = []
    objects: list[Path] = []
    for src in cu:
        obj = BUILD_DIR / (src.stem + ".cu.o")
        objects.append(obj)
        jobs.append(([*_nvcc_flags(cuda), "-c", str(src), "-o", str(obj)], BUILD_DIR / (src.stem + ".cu.log")))
    py_inc = sysconfig.get_paths()["include"]
    for src in cpp:
        obj = BUILD_DIR / (src.stem + ".cpp.o")
        objects.append(obj)
        cmd = [
            os.environ.get("CXX", "g++"),
            "-O2",
            "-std=c++17",
            "-fPIC",
            f"-D_GLIBCXX_USE_CXX11_ABI={int(cxx11_abi)}",
            f"-DTORCH_EXTENSION_NAME={LIB_NAME}",
            "-DTORCH_API_INCLUDE_EXTENSION_H",
            f"-I{CSRC}",
            f"-I{cuda / 'include'}",
            f"-I{py_inc}",
            *[f"-I{p}" for p in includes],
            "-c",
            str(src),
            "-o",
            str(obj),
        ]
        jobs.append((cmd, BUILD_DIR / (src.stem + ".cpp.log")))
    with ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 4))) as pool:
        futures = [pool.submit(_run, cmd, log) for cmd, log in jobs]
        for future in futures:
            future.result()
    link = [
        os.environ.get("CXX", "g++"),
        "-shared",
        "-o",
        str(LIB_PATH),
        *[str(o) for o in objects],
        *[f"-L{p}" for p in libdirs],
        f"-L{cuda / 'lib64'}",
        "-lc10",
        "-ltorch",
        "-ltorch_cpu",
        "-ltorch_python",
        "-lc10_cuda",
        "-ltorch_cuda",
        "-lcudart_static",
        "-ldl",
        "-lrt",
        "-lpthread",
        *[f"-Wl,-rpath,{p}" for p in libdirs],
    ]
    _run(link, BUILD_DIR / "link.log")
    STAMP_PATH.write_text(_source_hash(ARCH_FLAGS))
    if verbose:
        for log in sorted(BUILD_DIR.glob("*.cu.log")):
            print(log.read_text())
    return LIB_PATH


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(path)

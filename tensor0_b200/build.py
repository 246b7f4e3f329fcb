"""Build recipe for the sm_100a engine library (``_lib/libtensor0_b200.so``).

Compiles every CUDA / C++ source under ``csrc/`` with nvcc for
``compute_100a/sm_100a`` and links a shared library with the static CUDA
runtime, so the library loads on hosts without a GPU driver (the CPU test
suite checks its exported symbols there).

``build_xla()`` links the XLA FFI handler library
(``_lib/libtensor0_b200_xla.so``, source ``xla/handlers.cu``) on top of it.
It needs the XLA FFI headers (``xla/ffi/api/ffi.h``): from
``TENSOR0_XLA_FFI_INCLUDE``, an installed jaxlib, or the jaxlib 0.11.2 copy
that the reference vendors (``crates/tensor0-py/vendor/jaxlib-0.11.2/include``
under ``TENSOR0_REFERENCE``, default ``/root/reference``).  Without them it
builds nothing and returns None.
"""

from __future__ import annotations

import os
import shutil
import subprocess
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
CSRC = PACKAGE / "csrc"
OUT = PACKAGE / "_lib"
BUILD = PACKAGE / "_build"
LIBRARY = OUT / "libtensor0_b200.so"
XLA_SOURCE = PACKAGE / "xla" / "handlers.cu"
XLA_LIBRARY = OUT / "libtensor0_b200_xla.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "--expt-relaxed-constexpr", "-DNDEBUG"]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found; the CUDA 12.9 toolkit is required to build tensor0_b200")
    return path


def sources() -> list[Path]:
    return sorted([*CSRC.glob("*.cu"), *CSRC.glob("*.cpp")])


def _stale(target: Path, inputs: list[Path]) -> bool:
    if not target.exists():
        return True
    stamp = target.stat().st_mtime
    return any(path.stat().st_mtime > stamp for path in inputs)


def build(verbose: bool = False, jobs: int | None = None) -> Path:
    """Compile and link the library if any source or header changed."""
    compiler = nvcc()
    OUT.mkdir(exist_ok=True)
    BUILD.mkdir(exist_ok=True)
    headers = [*CSRC.glob("*.h"), *CSRC.glob("*.cuh"), PACKAGE.parent / "include" / "tensor0_b200.h"]
    objects = []
    commands = []
    for source in sources():
        obj = BUILD / (source.name + ".o")
        objects.append(obj)
        if _stale(obj, [source, *headers, Path(__file__)]):
            language = ["-x", "cu"]
            commands.append([compiler, *language, *ARCH, *NVCC_FLAGS, "-I", str(CSRC),
                             "-I", str(PACKAGE.parent / "include"), "-c", str(source), "-o", str(obj)])

    def run(command: list[str]) -> None:
        if verbose:
            print(" ".join(command), flush=True)
        subprocess.run(command, check=True)

    with ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 1)) as pool:
        list(pool.map(run, commands))
    if commands or _stale(LIBRARY, objects):
        run([compiler, *ARCH, "-shared", "--cudart=static", "-o", str(LIBRARY), *map(str, objects)])
    return LIBRARY


def xla_ffi_include() -> Path | None:
    """The directory holding ``xla/ffi/api/ffi.h``, or None."""
    candidates = []
    if os.environ.get("TENSOR0_XLA_FFI_INCLUDE"):
        candidates.append(Path(os.environ["TENSOR0_XLA_FFI_INCLUDE"]))
    try:
        import jaxlib  # noqa: F401  (absent in this image; used where installed)
        candidates.append(Path(jaxlib.__file__).parent / "include")
    except ImportError:
        pass
    reference = Path(os.environ.get("TENSOR0_REFERENCE", "/root/reference"))
    candidates.append(reference / "crates" / "tensor0-py" / "vendor" / "jaxlib-0.11.2" / "include")
    for candidate in candidates:
        if (candidate / "xla" / "ffi" / "api" / "ffi.h").is_file():
            return candidate
    return None


def build_xla(verbose: bool = False) -> Path | None:
    """Link the XLA FFI handler library if its headers are available."""
    include = xla_ffi_include()
    if include is None:
        return None
    library = build(verbose=verbose)
    inputs = [XLA_SOURCE, PACKAGE.parent / "include" / "tensor0_b200.h",
              PACKAGE.parent / "include" / "tensor0_b200_xla.h", library, Path(__file__)]
    if _stale(XLA_LIBRARY, inputs):
        command = [nvcc(), "-x", "cu", *ARCH, *NVCC_FLAGS, "-diag-suppress", "940,2473",
                   "-I", str(PACKAGE.parent / "include"), "-isystem", str(include),
                   "-shared", "--cudart=static", str(XLA_SOURCE), "-o", str(XLA_LIBRARY),
                   "-L", str(OUT), "-ltensor0_b200", "-Xlinker", "-rpath,$ORIGIN"]
        if verbose:
            print(" ".join(command), flush=True)
        subprocess.run(command, check=True)
    return XLA_LIBRARY


if __name__ == "__main__":
    print(build(verbose=True))
    print(build_xla(verbose=True))

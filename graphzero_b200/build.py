"""In-tree build of libgraphzero_b200.so (nvcc, sm_100a) and the oracle.

Usage: python graphzero_b200/build.py [--force]
(run as a file: importing the package itself needs the built library)

The CUDA library is compiled per translation unit (in parallel) into
graphzero_b200/_build/ and linked into graphzero_b200/libgraphzero_b200.so.
Objects are rebuilt when a source or any header under csrc/ or include/ is
newer than the object.
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
BUILD = PKG / "_build"
LIB = PKG / "libgraphzero_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
              f"-I{ROOT / 'include'}", f"-I{CSRC}", "--expt-relaxed-constexpr"]
# The search kernels rely on explicitly rounded IEEE operations; keep the
# compiler from contracting anything else in that unit either.
PER_FILE = {"mcts.cu": ["-fmad=false"]}


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _headers() -> list[Path]:
    return list(CSRC.glob("*.h")) + list((ROOT / "include").glob("*.h"))


def _stale(out: Path, deps: list[Path]) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, force: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    if force or _stale(obj, [src] + _headers()):
        cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *PER_FILE.get(src.name, []), "-c", str(src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj


def build_library(force: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, force), srcs))
    if force or _stale(LIB, objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-ldl", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


def reference_dir() -> Path | None:
    """The reference checkout whose rule functions oracle/_ref is compiled
    from: $GZ_REFERENCE_DIR, else a `reference` directory beside this
    repository; None when neither exists."""
    cand = os.environ.get("GZ_REFERENCE_DIR") or str(ROOT.parent / "reference")
    return Path(cand) if (Path(cand) / "games" / "connect4" / "connect4.cu").exists() else None


def build_oracle() -> None:
    """Build the CPU oracle (test infrastructure) and, where the reference tree
    is present, its rule functions under oracle/_ref."""
    cmd = ["make", "-s", "-C", str(ROOT / "oracle")]
    ref = reference_dir()
    if ref is not None:
        cmd.append(f"REF={ref}")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{r.stdout}\n{r.stderr}")


def main(argv: list[str]) -> int:
    force = "--force" in argv
    print(build_library(force))
    build_oracle()
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))

"""Build the C-ABI CUDA library for sm_100a in-tree.

    python moss-tts-optimized_b200/build.py [--verbose]

Compiles every ``csrc/*.cu`` with ``nvcc -gencode arch=compute_100a,code=sm_100a``
(objects in ``_build/``, in parallel) and links ``moss_tts/_runtime/libmoss_tts_b200.so``.
The library links the CUDA runtime statically and exports only the ``mt_*``
entry points declared in ``include/moss_tts_b200.h``; it has no torch dependency.
"""
import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
OUT = HERE / "moss_tts" / "_runtime" / "libmoss_tts_b200.so"
BUILD = HERE / "_build"
INCLUDE = HERE.parent / "include"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
         "-Xptxas", "-v", "--expt-relaxed-constexpr", f"-I{INCLUDE}"]


def nvcc() -> str:
    for cand in (os.environ.get("MOSS_TTS_NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; set MOSS_TTS_NVCC or CUDA_HOME")


def _compile(src: Path, verbose: bool) -> tuple[Path, str]:
    obj = BUILD / (src.stem + ".o")
    cmd = [nvcc(), *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    log = res.stdout + res.stderr
    if res.returncode:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{log}")
    return obj, log


def up_to_date() -> bool:
    if not OUT.exists():
        return False
    newest = max(p.stat().st_mtime for p in list(CSRC.glob("*")) + list(INCLUDE.glob("*.h")))
    return OUT.stat().st_mtime >= newest


def build(verbose: bool = False, force: bool = False) -> Path:
    if not force and up_to_date():
        return OUT
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    with cf.ThreadPoolExecutor(max_workers=max(1, min(len(sources), os.cpu_count() or 1))) as ex:
        results = list(ex.map(lambda s: _compile(s, verbose), sources))
    logs = "\n".join(log for _, log in results)
    (BUILD / "ptxas.log").write_text(logs)
    if verbose:
        print(logs)
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", *[str(o) for o, _ in results],
           "-o", str(tmp)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode:
        raise RuntimeError(f"link failed:\n{res.stdout}{res.stderr}")
    tmp.replace(OUT)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    path = build(args.verbose, args.force)
    print(path)
    sys.exit(0)

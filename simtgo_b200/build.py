"""Builds libsimtgo_b200.so in-tree with nvcc for sm_100a.

    python -m simtgo_b200.build          # incremental
    python -m simtgo_b200.build --force  # rebuild everything

Each csrc/*.cu is compiled to simtgo_b200/_build/<name>.o (in parallel, only
when it or a header changed), then linked with -ldl into
simtgo_b200/libsimtgo_b200.so. The device headers a tile graph's specialised
kernel is compiled from at run time (tile_jit.cu, NVRTC) are written into
_build/rtc_headers.inc as string literals first, so they travel inside the
library. The library links the CUDA runtime
statically, so it needs only libcuda.so.1 at run time.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import pathlib
import subprocess
import sys

PKG = pathlib.Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libsimtgo_b200.so"

NVCC = os.environ.get("NVCC", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--fmad=false", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-Wall", "-I", str(ROOT / "include"), "-I", str(BUILD),
         "--expt-relaxed-constexpr",
         "-Xptxas", "-warn-spills"]


def _headers():
    return sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) +
                  list((ROOT / "include").glob("*.h")))


def _compile(src: pathlib.Path, force: bool, verbose: bool) -> pathlib.Path:
    obj = BUILD / (src.stem + ".o")
    deps = [src] + _headers()
    if not force and obj.exists() and obj.stat().st_mtime >= max(d.stat().st_mtime for d in deps):
        return obj
    cmd = [NVCC, *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    if verbose or "spill" in r.stderr.lower() and "0 bytes spill" not in r.stderr:
        sys.stderr.write(r.stderr)
    return obj


# The headers NVRTC needs for a specialised tile kernel, by the names
# tile_kernel.cuh includes them under.
RTC_HEADERS = ["tile_kernel.cuh", "common.cuh", "exact.cuh", "tma.cuh"]
RTC_INC = BUILD / "rtc_headers.inc"
_DELIM = "SIMTGO_RTC"


def _write_rtc_headers(force: bool) -> None:
    srcs = [CSRC / h for h in RTC_HEADERS]
    if not force and RTC_INC.exists() and RTC_INC.stat().st_mtime >= max(
            p.stat().st_mtime for p in srcs):
        return
    out = ["// Written by simtgo_b200/build.py from csrc/: the device headers of a",
           "// specialised tile kernel, for NVRTC. Do not edit.",
           f"const int kRtcHeaderCount = {len(srcs)};",
           "const char* const kRtcHeaderNames[] = {" + ", ".join(f'"{h}"' for h in RTC_HEADERS)
           + "};",
           "const char* const kRtcHeaderSources[] = {"]
    for p in srcs:
        text = p.read_text()
        if f"){_DELIM}" in text:
            raise RuntimeError(f"{p.name} contains the raw-string delimiter")
        out.append(f'R"{_DELIM}({text}){_DELIM}",')
    out.append("};")
    tmp = RTC_INC.with_suffix(".tmp")
    tmp.write_text("\n".join(out) + "\n")
    os.replace(tmp, RTC_INC)


def build(force: bool = False, verbose: bool = False) -> pathlib.Path:
    BUILD.mkdir(exist_ok=True)
    _write_rtc_headers(force)
    sources = sorted(CSRC.glob("*.cu"))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, verbose), sources))
    newest = max(o.stat().st_mtime for o in objs)
    if force or not LIB.exists() or LIB.stat().st_mtime < newest:
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [NVCC, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", str(tmp),
               *map(str, objs), "-ldl", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))

"""Ahead-of-time build of the native libraries (sm_100a only).

Produces, inside the package directory:

* ``liboeqb200.so``       -- the C-ABI library (kernels + host runtime), from ``csrc/*.cu``;
* ``libtorch_oeqb200.so`` -- the thin libtorch registration of the operator schemas,
  linked against ``liboeqb200.so``.

The unrolled Clebsch-Gordan header is generated first (``csrc/gen_cg.py``).  Objects are
rebuilt only when a source, header or flag changed.  Nothing here needs a GPU.
"""

from __future__ import annotations

import concurrent.futures as cf
import hashlib
import json
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
BUILD = PKG / "_build"
LIB = PKG / "liboeqb200.so"
TORCH_LIB = PKG / "libtorch_oeqb200.so"

ARCH = "-gencode=arch=compute_100a,code=sm_100a"
LMAX_UNROLLED = int(os.environ.get("OEQB_LMAX_UNROLLED", "3"))
CU_SOURCES = ["capi.cu", "kern_f32_batch.cu", "kern_f64_batch.cu", "kern_f32_det.cu",
              "kern_f64_det.cu", "kern_sc.cu",
              "kern_uvw_tc.cu", "kern_uvw_sw.cu", "kern_edge_pipe.cu"]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the native build needs the CUDA toolkit")
    return cand


def _nvcc_flags():
    return ["-std=c++20", ARCH, "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-Xptxas", "-v",
            f"-I{CSRC}", f"-I{INCLUDE}"]


def _digest(paths, extra: str) -> str:
    h = hashlib.sha256(extra.encode())
    for p in paths:
        h.update(Path(p).read_bytes())
    return h.hexdigest()


def _run(cmd, log: Path):
    res = subprocess.run(cmd, capture_output=True, text=True)
    log.write_text(" ".join(cmd) + "\n" + res.stdout + res.stderr)
    if res.returncode != 0:
        tail = (res.stdout + res.stderr)[-4000:]
        raise RuntimeError(f"command failed: {' '.join(cmd)}\n{tail}")


def _includes(path: Path, seen: set) -> None:
    """Adds the repository headers `path` includes (transitively) to `seen`."""
    for line in path.read_text().splitlines():
        line = line.strip()
        if not line.startswith("#include \""):
            continue
        name = line.split('"')[1]
        for base in (CSRC, INCLUDE):
            dep = base / name
            if dep.exists() and dep not in seen:
                seen.add(dep)
                _includes(dep, seen)
                break


def _deps(src: str):
    """The source and every repository header it includes, in a stable order."""
    seen: set = set()
    _includes(CSRC / src, seen)
    return [CSRC / src] + sorted(seen)


def build_native(jobs: int | None = None, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    subprocess.run([sys.executable, str(CSRC / "gen_cg.py"), str(CSRC / "cg_unrolled.cuh"),
                    str(LMAX_UNROLLED)], check=True)
    flags = _nvcc_flags()
    stamp_file = BUILD / "stamps.json"
    stamps = json.loads(stamp_file.read_text()) if stamp_file.exists() else {}
    work = []
    for src in CU_SOURCES:
        obj = BUILD / (src + ".o")
        dig = _digest(_deps(src), " ".join(flags))
        if not obj.exists() or stamps.get(src) != dig:
            work.append((src, obj, dig))
    jobs = jobs or min(len(work) or 1, os.cpu_count() or 4)

    def compile_one(item):
        src, obj, dig = item
        _run([_nvcc(), *flags, "-c", str(CSRC / src), "-o", str(obj)], BUILD / (src + ".log"))
        return src, dig

    if work:
        if verbose:
            print(f"[oeqb] compiling {[w[0] for w in work]} with {jobs} jobs", flush=True)
        errors = []
        with cf.ThreadPoolExecutor(jobs) as ex:
            futures = [ex.submit(compile_one, w) for w in work]
            for fut in cf.as_completed(futures):
                try:
                    src, dig = fut.result()
                except RuntimeError as exc:
                    errors.append(str(exc))
                    continue
                stamps[src] = dig
                stamp_file.write_text(json.dumps(stamps, indent=1))
        if errors:
            raise RuntimeError("\n\n".join(errors))
    objs = [str(BUILD / (s + ".o")) for s in CU_SOURCES]
    link_dig = _digest(objs, "link")
    if work or not LIB.exists() or stamps.get("__link__") != link_dig:
        tmp = LIB.with_suffix(".so.tmp")
        _run([_nvcc(), ARCH, "-shared", "-o", str(tmp), *objs], BUILD / "link.log")
        os.replace(tmp, LIB)
        stamps["__link__"] = link_dig
        stamp_file.write_text(json.dumps(stamps, indent=1))
    return LIB


def build_torch_shim(verbose: bool = False) -> Path:
    import torch
    from torch.utils import cpp_extension

    src = CSRC / "torch_ops.cpp"
    incs = cpp_extension.include_paths(device_type="cuda")
    libdirs = cpp_extension.library_paths(device_type="cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-std=c++17", "-O2", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           f"-I{INCLUDE}", *[f"-I{d}" for d in incs], str(src), "-o", str(TORCH_LIB) + ".tmp",
           *[f"-L{d}" for d in libdirs], f"-L{PKG}", "-loeqb200", "-lc10", "-lc10_cuda",
           "-ltorch", "-ltorch_cpu", "-Wl,-rpath,$ORIGIN",
           *[f"-Wl,-rpath,{d}" for d in libdirs]]
    stamp_file = BUILD / "stamps.json"
    stamps = json.loads(stamp_file.read_text()) if stamp_file.exists() else {}
    dig = _digest([src, INCLUDE / "oeqb200.h"], " ".join(cmd) + torch.__version__)
    if TORCH_LIB.exists() and stamps.get("__torch__") == dig:
        return TORCH_LIB
    if verbose:
        print("[oeqb] compiling torch shim", flush=True)
    _run(cmd, BUILD / "torch_shim.log")
    os.replace(str(TORCH_LIB) + ".tmp", TORCH_LIB)
    stamps["__torch__"] = dig
    stamp_file.write_text(json.dumps(stamps, indent=1))
    return TORCH_LIB


def build(jobs: int | None = None, verbose: bool = True) -> None:
    BUILD.mkdir(exist_ok=True)
    build_native(jobs=jobs, verbose=verbose)
    build_torch_shim(verbose=verbose)


if __name__ == "__main__":
    build()

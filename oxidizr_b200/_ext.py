"""Build and load the in-tree sm_100a extension.

The extension is compiled with nvcc for ``sm_100a`` only
(``-gencode arch=compute_100a,code=sm_100a``) into ``build/`` at the repo root,
so the built ``.so`` travels with the source tree.  ``load()`` imports the
built module directly when it exists and is newer than every source file;
otherwise it (re)builds first.
"""
from __future__ import annotations

import glob
import importlib.machinery
import importlib.util
import os
import sys
import threading

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(REPO, "csrc")
BUILD_DIR = os.path.join(REPO, "build", "oxidizr_b200_C")
NAME = "oxidizr_b200_C"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr", "--expt-extended-lambda",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__", "-U__CUDA_NO_BFLOAT162_OPERATORS__",
    "-Xptxas=-v" if os.environ.get("OXI_PTXAS_VERBOSE") else "-Xptxas=-O3",
]

_lock = threading.Lock()
_mod = None

# Measurement tools (NVLink access microbenchmark) live in a separate
# extension built from csrc/tools/, so the training library carries none of them.
TOOLS_DIR = os.path.join(CSRC, "tools")
TOOLS_BUILD_DIR = os.path.join(REPO, "build", "oxidizr_b200_tools")
TOOLS_NAME = "oxidizr_b200_tools"
_tools = None


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + sorted(glob.glob(os.path.join(CSRC, "*.cpp")))


def _headers():
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh"))) + sorted(glob.glob(os.path.join(CSRC, "*.h")))


def so_path():
    return os.path.join(BUILD_DIR, NAME + ".so")


def _stale() -> bool:
    so = so_path()
    if not os.path.exists(so):
        return True
    t = os.path.getmtime(so)
    return any(os.path.getmtime(s) > t for s in sources() + _headers())


# torch's builder serialises builds of one directory through a ``lock`` file that it
# deletes when done, and waits without limit while another build holds it.  A copy of the
# tree taken while a build ran carries that file, so a build in the copy would wait
# forever.  Before building, wait for a lock file only until it is STALE_LOCK_S old (no
# build here takes that long), then treat it as left over and remove it.
STALE_LOCK_S = 10 * 60


def _clear_stale_lock(build_dir: str) -> None:
    import time
    path = os.path.join(build_dir, "lock")
    while True:
        try:
            age = time.time() - os.path.getmtime(path)
        except OSError:
            return  # no lock (or it went away): go ahead
        if age > STALE_LOCK_S:
            print(f"oxidizr_b200: removing a stale build lock ({age / 60:.0f} min old): {path}", file=sys.stderr)
            try:
                os.remove(path)
            except OSError:
                pass
            return
        time.sleep(min(5.0, STALE_LOCK_S - age + 0.1))


def build(verbose: bool = False, force: bool = False):
    """Compile every CUDA/C++ source of the extension for sm_100a (imports the built module
    without invoking the builder when it is newer than every source, unless ``force``)."""
    if not force and not _stale():
        return _import_built()
    os.makedirs(BUILD_DIR, exist_ok=True)
    _clear_stale_lock(BUILD_DIR)
    from torch.utils.cpp_extension import load
    os.environ.setdefault("MAX_JOBS", str(max(os.cpu_count() or 4, 4)))
    mod = load(
        name=NAME,
        sources=sources(),
        extra_cflags=["-O3", "-std=c++17"],
        extra_cuda_cflags=NVCC_FLAGS,
        extra_include_paths=[CSRC],
        extra_ldflags=["-lcuda"],
        build_directory=BUILD_DIR,
        with_cuda=True,
        verbose=verbose,
    )
    return mod


def _import_built():
    loader = importlib.machinery.ExtensionFileLoader(NAME, so_path())
    spec = importlib.util.spec_from_file_location(NAME, so_path(), loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    sys.modules[NAME] = mod
    return mod


def load(required: bool = True):
    """Return the extension module (building it if needed)."""
    global _mod
    if _mod is not None:
        return _mod
    with _lock:
        if _mod is not None:
            return _mod
        import torch  # noqa: F401  (the extension links against torch)
        try:
            if _stale() or os.environ.get("OXI_FORCE_BUILD"):
                _mod = build(verbose=bool(os.environ.get("OXI_BUILD_VERBOSE")), force=True)
            else:
                _mod = _import_built()
        except Exception as e:  # pragma: no cover - only hit without a toolchain
            if required:
                raise RuntimeError(f"oxidizr_b200 CUDA extension unavailable: {e}") from e
            return None
        return _mod


def tools_sources():
    return sorted(glob.glob(os.path.join(TOOLS_DIR, "*.cu"))) + sorted(glob.glob(os.path.join(TOOLS_DIR, "*.cpp")))


def build_tools(verbose: bool = False):
    """Compile the measurement-tools extension (csrc/tools/) for sm_100a."""
    os.makedirs(TOOLS_BUILD_DIR, exist_ok=True)
    _clear_stale_lock(TOOLS_BUILD_DIR)
    from torch.utils.cpp_extension import load as _load
    return _load(name=TOOLS_NAME, sources=tools_sources(), extra_cflags=["-O3", "-std=c++17"],
                 extra_cuda_cflags=NVCC_FLAGS, extra_include_paths=[CSRC, TOOLS_DIR],
                 build_directory=TOOLS_BUILD_DIR, with_cuda=True, verbose=verbose)


def load_tools():
    """The measurement-tools extension module (built on first use)."""
    global _tools
    with _lock:
        if _tools is None:
            import torch  # noqa: F401
            _tools = build_tools(verbose=bool(os.environ.get("OXI_BUILD_VERBOSE")))
        return _tools

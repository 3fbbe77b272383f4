"""Build and load the package's native extensions in-tree.

Two extensions:

* ``_sp_kernels`` — the sm_100a CUDA kernels (tcgen05 GEMM, MLA decode and
  prefill attention, norms/RoPE, MoE routing, sampling) plus their torch
  bindings. Compiled with ``-gencode arch=compute_100a,code=sm_100a`` only.
* ``_sp_core`` — the C++ serving runtime (KV arena, prefix cache, scheduler,
  work control, tokenizer, request API, wire codecs, ...), host code only.

Built objects live in ``sparkpipe_rs_b200/_ext/<name>/``. A content hash of
the sources, headers and flags is stored next to each ``.so``; ``load`` imports
the ``.so`` directly when the hash matches and rebuilds otherwise, so a source
change can never run against a stale binary.
"""
from __future__ import annotations

import hashlib
import importlib.util
import os
import sys
import threading
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
INCLUDE = PKG_DIR / "include"  # public C headers (driver ABI)
EXT_DIR = PKG_DIR / "_ext"

CUDA_ARCH_FLAGS = ["-gencode=arch=compute_100a,code=sm_100a"]
CUDA_FLAGS = CUDA_ARCH_FLAGS + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas=-warn-spills",
]
CXX_FLAGS = ["-O3", "-std=c++17"]

# SPARKPIPE_SANITIZE=address (AddressSanitizer + UndefinedBehaviorSanitizer) or thread
# (ThreadSanitizer) builds the host runtime extension `_sp_core` instrumented, into its
# own directory, and loads that build; the sanitizer runtime must be preloaded into the
# interpreter (utils/sanitize.py does both). The CUDA extension is never instrumented.
SANITIZE = os.environ.get("SPARKPIPE_SANITIZE", "")
_SAN_FLAGS = {
    "address": ["-fsanitize=address,undefined", "-fno-sanitize-recover=undefined", "-fno-omit-frame-pointer",
                "-g", "-O1"],
    "thread": ["-fsanitize=thread", "-fno-omit-frame-pointer", "-g", "-O1"],
}
if SANITIZE and SANITIZE not in _SAN_FLAGS:
    raise RuntimeError(f"SPARKPIPE_SANITIZE must be one of {sorted(_SAN_FLAGS)}")


def _sanitizer_link_flags() -> list[str]:
    """-fsanitize for the link plus the directory of the sanitizer runtime as the system
    compiler reports it (a compiler wrapper may not search that directory itself)."""
    import subprocess

    lib = "libasan.so" if SANITIZE == "address" else "libtsan.so"
    flags = [f"-fsanitize={'address,undefined' if SANITIZE == 'address' else 'thread'}"]
    for cc in ("g++", "/usr/bin/g++"):
        try:
            path = subprocess.run([cc, f"-print-file-name={lib}"], capture_output=True, text=True).stdout.strip()
        except OSError:
            continue
        if os.path.isabs(path) and os.path.exists(path):
            flags.append(f"-L{os.path.dirname(path)}")
            break
    return flags


def _kernel_sources() -> list[Path]:
    d = CSRC / "kernels"
    return sorted(d.glob("*.cu")) + [d / "ops.cpp"]


def _core_sources() -> list[Path]:
    return sorted((CSRC / "core").glob("*.cpp"))


SPECS = {
    "_sp_kernels": {
        "sources": _kernel_sources,
        "headers": lambda: sorted((CSRC / "kernels").glob("*.h")) + sorted((CSRC / "kernels").glob("*.cuh")),
        "cuda": True,
    },
    "_sp_core": {
        "sources": _core_sources,
        "headers": lambda: sorted((CSRC / "core").glob("*.h")) + sorted(INCLUDE.rglob("*.h")),
        "cuda": False,
    },
}

_lock = threading.Lock()
_loaded: dict[str, object] = {}


def _sanitized(name: str) -> bool:
    return bool(SANITIZE) and not SPECS[name]["cuda"]


def _cxx_flags(name: str) -> list[str]:
    if _sanitized(name):
        return ["-std=c++17"] + _SAN_FLAGS[SANITIZE]
    return CXX_FLAGS


def _build_dir(name: str) -> Path:
    return EXT_DIR / (f"{name}_{SANITIZE}" if _sanitized(name) else name)


def _digest(name: str) -> str:
    spec = SPECS[name]
    h = hashlib.sha256()
    for p in list(spec["sources"]()) + list(spec["headers"]()):
        h.update(p.name.encode())
        h.update(p.read_bytes())
    h.update(repr(CUDA_FLAGS if spec["cuda"] else []).encode())
    h.update(repr(_cxx_flags(name)).encode())
    import torch

    h.update(torch.__version__.encode())
    return h.hexdigest()


def _so_path(name: str) -> Path:
    return _build_dir(name) / f"{name}.so"


def _import_so(name: str, path: Path):
    spec = importlib.util.spec_from_file_location(name, str(path))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    sys.modules[name] = mod
    return mod


def build(name: str, verbose: bool = False):
    """Compile extension ``name`` in-tree and import it."""
    import torch  # noqa: F401  (torch must be imported before its extension helpers)
    from torch.utils import cpp_extension

    spec = SPECS[name]
    out = _build_dir(name)
    out.mkdir(parents=True, exist_ok=True)
    os.environ.setdefault("MAX_JOBS", str(max(1, os.cpu_count() or 1)))
    srcs = [str(p) for p in spec["sources"]()]
    if not srcs:
        raise RuntimeError(f"no sources for extension {name}")
    # the stamp names the sources this build compiled, not ones edited while it ran
    digest = _digest(name)
    kw = dict(
        name=name,
        sources=srcs,
        extra_cflags=_cxx_flags(name),
        build_directory=str(out),
        verbose=verbose,
        with_cuda=spec["cuda"],
    )
    if spec["cuda"]:
        kw["extra_cuda_cflags"] = CUDA_FLAGS
        kw["extra_include_paths"] = [str(CSRC / "kernels")]
    else:
        kw["extra_include_paths"] = [str(CSRC / "core"), str(INCLUDE)]
        kw["extra_ldflags"] = ["-ldl"] + (_sanitizer_link_flags() if _sanitized(name) else [])
    mod = cpp_extension.load(**kw)
    (out / f"{name}.srchash").write_text(digest)
    _loaded[name] = mod
    return mod


def load(name: str):
    """Import extension ``name``, rebuilding it first if its sources changed."""
    with _lock:
        if name in _loaded:
            return _loaded[name]
        so = _so_path(name)
        stamp = _build_dir(name) / f"{name}.srchash"
        if so.exists() and stamp.exists() and stamp.read_text().strip() == _digest(name):
            mod = _import_so(name, so)
        else:
            mod = build(name)
        _loaded[name] = mod
        return mod


def build_all(verbose: bool = False) -> None:
    for name in SPECS:
        if not SPECS[name]["sources"]():
            continue
        so = _so_path(name)
        stamp = _build_dir(name) / f"{name}.srchash"
        if so.exists() and stamp.exists() and stamp.read_text().strip() == _digest(name):
            continue
        build(name, verbose=verbose)


def kernels():
    """The sm_100a kernel extension (raises if it cannot be built or loaded)."""
    return load("_sp_kernels")


def core():
    """The C++ serving-runtime extension."""
    return load("_sp_core")

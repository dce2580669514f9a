"""Build and load the in-tree sm_100a CUDA extension (``wb_C``).

The extension is compiled with ``torch.utils.cpp_extension`` into
``wavelet_b200/_build/`` inside the source tree, so the built ``.so`` travels
with the repository snapshot and is the module that every op imports.  A
content hash of the sources is stored next to the library; on import the hash
is compared and the extension is rebuilt when a source changed.

On a machine with a GPU the extension is mandatory: ops raise instead of
falling back to eager PyTorch when it cannot be loaded.
"""

from __future__ import annotations

import hashlib
import importlib.machinery
import importlib.util
import os
import sys
import threading
from pathlib import Path
from types import ModuleType

_PKG = Path(__file__).resolve().parent.parent
CSRC = _PKG / "csrc"
BUILD_DIR = _PKG / "_build"
NAME = "wb_C"

SOURCES = ["bindings.cpp", "runtime.cu", "gemm.cu", "kernels.cu", "attention.cu", "attention_noalloc.cu", "decode.cu", "comm.cu", "moe.cu", "policy.cu"]

CUDA_FLAGS = [
    "-gencode=arch=compute_100a,code=sm_100a",
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xptxas=-v" if os.environ.get("WB_PTXAS_VERBOSE") else "-Xptxas=-O3",
    "-DNDEBUG",
]
CXX_FLAGS = ["-O3", "-std=c++17"]

_lock = threading.Lock()
_module: ModuleType | None = None


def _sources() -> list[Path]:
    return [CSRC / s for s in SOURCES if (CSRC / s).exists()]


def source_hash() -> str:
    h = hashlib.sha256()
    for p in sorted(CSRC.glob("*")):
        if p.suffix in {".cu", ".cuh", ".h", ".cpp"}:
            h.update(p.name.encode())
            h.update(p.read_bytes())
    h.update(" ".join(CUDA_FLAGS).encode())
    return h.hexdigest()[:16]


def _so_path() -> Path | None:
    for suffix in importlib.machinery.EXTENSION_SUFFIXES + [".so"]:
        p = BUILD_DIR / f"{NAME}{suffix}"
        if p.exists():
            return p
    return None


def _stamp_path() -> Path:
    return BUILD_DIR / f"{NAME}.hash"


def is_built() -> bool:
    """True when the in-tree library exists and matches the current sources."""
    st = _stamp_path()
    return _so_path() is not None and st.exists() and st.read_text().strip() == source_hash()


def build(verbose: bool = False) -> ModuleType:
    """Compile the extension for sm_100a (works without a GPU) and load it."""
    from torch.utils import cpp_extension

    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    os.environ.setdefault("MAX_JOBS", str(max(4, (os.cpu_count() or 8))))
    mod = cpp_extension.load(
        name=NAME,
        sources=[str(s) for s in _sources()],
        extra_cflags=CXX_FLAGS,
        extra_cuda_cflags=CUDA_FLAGS,
        build_directory=str(BUILD_DIR),
        verbose=verbose,
        with_cuda=True,
    )
    _stamp_path().write_text(source_hash())
    return mod


def _import_prebuilt(path: Path) -> ModuleType:
    import torch  # noqa: F401  (libtorch symbols must be loaded first)

    spec = importlib.util.spec_from_file_location(NAME, str(path))
    assert spec is not None and spec.loader is not None
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    sys.modules[NAME] = mod
    return mod


def load(rebuild_if_stale: bool = True) -> ModuleType:
    """Return the loaded extension module, building it when needed."""
    global _module
    if _module is not None:
        return _module
    with _lock:
        if _module is not None:
            return _module
        so = _so_path()
        stamp = _stamp_path()
        fresh = so is not None and stamp.exists() and stamp.read_text().strip() == source_hash()
        if so is not None and (fresh or not rebuild_if_stale):
            _module = _import_prebuilt(so)
        else:
            _module = build()
        return _module


def available() -> bool:
    try:
        load()
        return True
    except Exception:  # pragma: no cover - depends on the toolchain
        return False


# --------------------------------------------------------------------------
# Launch accounting: the library counts every kernel it launches (a counter
# bumped at each launch site); ``count_launches()`` reports the kernels this
# repository launched inside the block.  A graph replay adds the number of
# library kernels recorded when the graph was captured (``note_launches``).
class count_launches:
    """Context manager: ``count`` = kernels this library launched in the block."""

    def __enter__(self):
        self._m = load()
        self._start = int(self._m.launch_count())
        self._end = None
        return self

    @property
    def count(self) -> int:
        end = self._end if self._end is not None else int(self._m.launch_count())
        return end - self._start

    def __exit__(self, *exc):
        self._end = int(self._m.launch_count())
        return False

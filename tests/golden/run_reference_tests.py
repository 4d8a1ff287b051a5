"""RUN THE REFERENCE'S OWN TESTS AGAINST THIS PACKAGE -- a compatibility
check for a container that has an Afterimage checkout; never run on a GPU
box (the checkout is not there) and never part of the product.

It writes a small import shim into a temp directory. The shim's package
`afterimage.runtime` resolves each module name to
`afterimage_b200.runtime.<module>`. Names this package does not define fall
back to the reference's own module: its CPU test oracles (this package has
no CPU decoder) and its tracing types. The script then runs the reference's
test files in place, read-only: no bytecode, no pytest cache, and the
checkout's conftest and pytest config switched off. It prints pytest's
summary and the names that fell back.

Usage:

    python tests/golden/run_reference_tests.py <path to the checkout> [test file names...]

With no file names it runs the files of this path: huffman,
huffman_chunked, compressed_store, sliced_decompress, binstore,
vram_planner, decode_table_reuse, gpu_decode, gpu_decode_v2,
compress_pipeline, config and verify.
"""
from __future__ import annotations

import os
import pathlib
import subprocess
import sys
import tempfile

REPO = pathlib.Path(__file__).resolve().parents[2]
FILES = ["test_huffman.py", "test_huffman_chunked.py", "test_compressed_store.py", "test_sliced_decompress.py",
         "test_binstore.py", "test_vram_planner.py", "test_decode_table_reuse.py", "test_gpu_decode.py",
         "test_gpu_decode_v2.py", "test_compress_pipeline.py", "test_config.py", "test_verify.py"]
MODULES = ["huffman", "huffman_chunked", "gpu_decode", "gpu_decode_v2", "compressed_store", "binstore",
           "vram_planner", "streaming_engine", "verify", "config", "critical_path", "cpu_decode", "directio"]

SHIM = '''import importlib, importlib.util, sys, types, pathlib, atexit
REF = pathlib.Path(%(ref)r)
FALLBACKS = set()


def _ref_module(name):
    key = "afterimage_refcopy." + name
    if key not in sys.modules:
        spec = importlib.util.spec_from_file_location(key, REF / (name + ".py"))
        mod = importlib.util.module_from_spec(spec)
        mod.__package__ = "afterimage.runtime"
        sys.modules[key] = mod
        spec.loader.exec_module(mod)
    return sys.modules[key]


class _Proxy(types.ModuleType):
    def __init__(self, name, ours):
        super().__init__("afterimage.runtime." + name)
        self._name, self._ours = name, ours

    def __getattr__(self, attr):
        if attr.startswith("__"):
            raise AttributeError(attr)
        if self._ours is not None and hasattr(self._ours, attr):
            return getattr(self._ours, attr)
        FALLBACKS.add(self._name + "." + attr)
        return getattr(_ref_module(self._name), attr)


for _n in %(modules)r:
    try:
        _ours = importlib.import_module("afterimage_b200.runtime." + _n)
    except ImportError:
        _ours = None
    sys.modules["afterimage.runtime." + _n] = _Proxy(_n, _ours)

atexit.register(lambda: print("names taken from the reference:", sorted(FALLBACKS)))
'''


def main() -> int:
    if len(sys.argv) < 2:
        print(__doc__)
        return 2
    checkout = pathlib.Path(sys.argv[1]).resolve()
    files = sys.argv[2:] or FILES
    with tempfile.TemporaryDirectory(prefix="reference_tests_") as tmp:
        shim = pathlib.Path(tmp) / "shim" / "afterimage" / "runtime"
        shim.mkdir(parents=True)
        (shim.parent / "__init__.py").write_text("")
        (shim / "__init__.py").write_text(SHIM % {"ref": str(checkout / "afterimage" / "runtime"),
                                                   "modules": MODULES})
        env = dict(os.environ, PYTHONDONTWRITEBYTECODE="1", NUMBA_CACHE_DIR=str(pathlib.Path(tmp) / "numba"),
                   PYTHONPATH=os.pathsep.join([str(shim.parent.parent), str(REPO)]))
        cmd = [sys.executable, "-m", "pytest", "-p", "no:cacheprovider", "--noconftest", "-c", os.devnull,
               "--rootdir", tmp, "-q", "-m", "not archive", "-rf"] + [str(checkout / "tests" / f) for f in files]
        return subprocess.run(cmd, cwd=tmp, env=env).returncode


if __name__ == "__main__":
    sys.exit(main())

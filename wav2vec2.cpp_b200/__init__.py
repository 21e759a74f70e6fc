"""wav2vec2-b200: B200-native wav2vec2 CTC inference engine (Python side).

The engine itself is C++/CUDA behind a C ABI (include/wav2vec2.h,
include/wav2vec2_b200.h) built into libwav2vec2_b200.so in this directory.
This package holds only the Python pieces that tests, the benchmark and users
scripting the library need: a ctypes binding (`binding`) and the seeded
synthetic model/audio generator (`synth`).

The directory name contains a dot, so it is imported by path:

    import importlib.util, sys
    spec = importlib.util.spec_from_file_location(
        "w2v_b200", "<repo>/wav2vec2.cpp_b200/__init__.py",
        submodule_search_locations=["<repo>/wav2vec2.cpp_b200"])
    w2v = importlib.util.module_from_spec(spec); sys.modules["w2v_b200"] = w2v
    spec.loader.exec_module(w2v)
"""
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = PKG_DIR / "libwav2vec2_b200.so"


def import_package(repo_root=None):
    """Import this package (under the module name 'w2v_b200') and return it."""
    import importlib.util
    import sys
    if "w2v_b200" in sys.modules:
        return sys.modules["w2v_b200"]
    root = Path(repo_root) if repo_root else PKG_DIR.parent
    pkg = root / "wav2vec2.cpp_b200"
    spec = importlib.util.spec_from_file_location(
        "w2v_b200", pkg / "__init__.py", submodule_search_locations=[str(pkg)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["w2v_b200"] = mod
    spec.loader.exec_module(mod)
    return mod

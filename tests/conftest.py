import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = Path(__file__).resolve().parent / "golden"
MODEL_CACHE = Path(os.environ.get("W2V_MODEL_CACHE", "/tmp/w2v_models"))

sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "oracle"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: takes more than ~20 s on the CPU")


def _pkg():
    from importlib import util
    if "w2v_b200" in sys.modules:
        return sys.modules["w2v_b200"]
    spec = util.spec_from_file_location("w2v_b200", ROOT / "wav2vec2.cpp_b200" / "__init__.py",
                                        submodule_search_locations=[str(ROOT / "wav2vec2.cpp_b200")])
    mod = util.module_from_spec(spec)
    sys.modules["w2v_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="session")
def pkg():
    return _pkg()


@pytest.fixture(scope="session")
def synth(pkg):
    import w2v_b200.synth as s
    return s


@pytest.fixture(scope="session")
def model_path(synth):
    """model_path(arch, dtype, **kw) -> cached seeded GGUF path."""
    def get(arch, dtype, **kw):
        return synth.cached_model(MODEL_CACHE, arch, dtype, **kw)
    return get


def load_golden(case):
    z = np.load(GOLDEN / f"ref_{case}.npz")
    return {k: (z[k].item() if z[k].shape == () else z[k]) for k in z.files}


@pytest.fixture(scope="session")
def golden():
    return load_golden

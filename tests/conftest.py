import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import __graft_entry__ as graft  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


@pytest.fixture(scope="session")
def pkg():
    return graft.load_package()


@pytest.fixture(scope="session")
def model_dir(tmp_path_factory):
    return tmp_path_factory.mktemp("models")


@pytest.fixture(scope="session")
def tiny_model(pkg, model_dir):
    """Seeded random-init GGUF at small dimensions (nc 8, 2 layers everywhere)."""
    return pkg.synth_model(str(model_dir / "tiny.gguf"), preset="tiny", seed=3)


@pytest.fixture(scope="session")
def tiny_oracle(tiny_model):
    import breeze_oracle as bo
    return bo.Model(tiny_model)


@pytest.fixture(scope="session")
def reference_bindings():
    """The reference's own Python bindings module (python/bz_ggml/bindings.py), loaded from the
    reference checkout that oracle/Makefile points at; skips where there is none."""
    import importlib.util
    import subprocess
    r = subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "print-ref"], capture_output=True, text=True)
    path = os.path.join(r.stdout.strip(), "python", "bz_ggml", "bindings.py")
    if r.returncode != 0 or not os.path.exists(path):
        pytest.skip("no reference checkout here")
    spec = importlib.util.spec_from_file_location("reference_bindings", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod

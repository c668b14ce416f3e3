import os
import pathlib
import sys

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); runs the sm_100a kernels")


@pytest.fixture(scope="session", autouse=True)
def built_libraries():
    """Builds the product, the synthetic-model writer and the checker in-tree."""
    from nuthatch_b200 import build

    build.build_synth()
    build.build_product()
    build.build_checker()
    return True


def gpu_available() -> bool:
    from nuthatch_b200._lib import lib

    return lib().nh_device_sm_count(0) > 0


@pytest.fixture(scope="session")
def gpu():
    if not gpu_available():
        pytest.skip("no CUDA device")
    return True


@pytest.fixture(scope="session")
def tmp_models(tmp_path_factory):
    return tmp_path_factory.mktemp("models")


@pytest.fixture(scope="session")
def synth_dir():
    d = pathlib.Path(os.environ.get("NUTHATCH_SYNTH_DIR", "/tmp/nuthatch_synth"))
    d.mkdir(parents=True, exist_ok=True)
    return d

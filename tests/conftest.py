import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (B200); run with -m gpu")
    config.addinivalue_line("markers", "slow: full-size configurations")


@pytest.fixture(scope="session", autouse=True)
def _cache_dir(tmp_path_factory):
    # synthetic models and the expf table are cached per machine; tests share them
    if not os.environ.get("EMBER_CACHE_DIR"):
        os.environ["EMBER_CACHE_DIR"] = os.path.join(
            os.path.expanduser("~"), ".cache", "ember_b200")
    yield

"""Test configuration: the `gpu` marker, import paths and shared fixtures.

CPU tests (-m "not gpu") cover the oracle against the reference and the golden vectors,
the GGUF / quantisation tooling, the host logic and the C-ABI's exported symbols.  GPU tests
(-m gpu) are the parity tests proper: they call the CUDA path through the C-ABI and compare
with the oracle and the committed golden fixtures.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(ROOT, "agent-serve_b200"), os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")
    config.addinivalue_line("markers", "slow: full-size configuration (minutes)")


@pytest.fixture(scope="session")
def model_cache(tmp_path_factory):
    d = os.environ.get("TFB200_CACHE") or str(tmp_path_factory.mktemp("models"))
    os.environ["TFB200_CACHE"] = d
    return d

from __future__ import annotations

import os
import sys

import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)
# The reference engine itself (`pip install --no-deps --target baseline/_ref`, done by
# __graft_entry__.build() where the reference source is present): the engine tests run its own
# ModelRunner and graph runners with the int8 modules swapped in.
REF_SITE = os.path.join(REPO, "baseline", "_ref")
if os.path.isdir(os.path.join(REF_SITE, "llm_serving_engine")) and REF_SITE not in sys.path:
    sys.path.append(REF_SITE)


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100a) device; run with -m gpu")
    config.addinivalue_line("markers", "multigpu: needs >= 2 CUDA devices")


def pytest_runtest_setup(item: pytest.Item) -> None:
    """A GPU test fails without CUDA (as the reference's `cuda` marker does,
    tests/conftest.py:11-14 there), so a run can only pass by running it."""
    if item.get_closest_marker("gpu") and not torch.cuda.is_available():
        pytest.fail("needs CUDA; on a CPU-only machine run pytest -m 'not gpu'", pytrace=False)


@pytest.fixture(scope="session")
def golden_dir() -> str:
    return os.path.join(REPO, "tests", "golden")

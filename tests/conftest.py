import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def pkg():
    import __graft_entry__
    return __graft_entry__.load_package()


@pytest.fixture(scope="session")
def nanovllm_ref():
    """Directory of the unmodified reference nano-vLLM (baseline/_ref), put on sys.path.

    Installed from the checkout when one is present; a GPU box gets the installed
    copy with the repository.  The drop-in tests are the evidence that this package
    replaces the reference's attention path inside its own modules, so a missing
    reference fails them instead of skipping them."""
    import __graft_entry__
    where = __graft_entry__.install_reference()
    if where is None:
        pytest.fail("the reference nano-vLLM is not installed in baseline/_ref and no checkout is available "
                    "to install it from: run __graft_entry__.build() where the checkout exists")
    if where not in sys.path:
        sys.path.insert(0, where)
    return where

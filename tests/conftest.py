import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (REPO, os.path.join(REPO, "tests"), os.path.join(REPO, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle():
    import oracle as _oracle
    _oracle.build()
    return _oracle


def load_mri():
    """The product package (directory name is not an identifier)."""
    import importlib
    return importlib.import_module("mini-rust-inference_b200")


@pytest.fixture(scope="session")
def mri():
    return load_mri()


@pytest.fixture(scope="session")
def gpu_ctx(mri):
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a machine without CUDA")
    return mri.default_context(0)


@pytest.fixture
def ctx_option(gpu_ctx):
    """set(option, value): a kernel-variant option of the default context for
    the duration of one test (restored afterwards)."""
    saved = []

    def set_(option, value):
        saved.append((option, gpu_ctx.get_option(option)))
        gpu_ctx.set_option(option, value)

    yield set_
    for option, value in reversed(saved):
        gpu_ctx.set_option(option, value)

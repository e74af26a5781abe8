import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from oracle import cpu as _cpu  # noqa: E402

# The reference checkout (SC_REFERENCE_DIR, else where the build found it); it
# exists only where the library was built, never on GPU boxes.
REFERENCE = _cpu.reference_dir()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); parity tests of the CUDA path")


@pytest.fixture(scope="session", autouse=True)
def _built():
    """Builds libsc_b200.so and the oracle if they are missing or stale (no-op
    when up to date; on a GPU box the prebuilt files travel with the tree)."""
    from sparse_computation_b200 import build as b
    if not os.path.exists(b.LIB) or os.environ.get("SC_REBUILD"):
        b.build()
    from oracle import cpu
    if not os.path.exists(cpu.LIBORACLE):
        cpu.build()
    yield


def has_reference() -> bool:
    return bool(REFERENCE) and os.path.isdir(os.path.join(REFERENCE, "code_gen"))


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("CUDA GPU required for -m gpu tests")
    return torch.device("cuda:0")

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")
    config.addinivalue_line("markers", "slow: full-size parity case")


def _has_gpu() -> bool:
    try:
        import nutllm_b200 as nb
        return nb.device_count() > 0
    except Exception:
        return False


@pytest.fixture(scope="session")
def gpu():
    if not _has_gpu():
        pytest.fail("GPU test run without a usable CUDA device "
                    "(nutllm_b200 has no CPU fallback)")
    return 0


@pytest.fixture(scope="session")
def orc():
    import oracle
    return oracle.Oracle()


@pytest.fixture(scope="session")
def ref():
    import oracle
    if not oracle.reference_available():
        pytest.skip("reference build (oracle/_ref) not present")
    return oracle.Reference()


GOLDEN = os.path.join(ROOT, "tests", "golden")


def golden_path(name: str) -> str:
    return os.path.join(GOLDEN, name)

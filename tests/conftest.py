"""Shared test setup: import paths for the product package and the CPU oracle, the `gpu` marker."""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT / "codon-infer_b200", ROOT / "oracle", ROOT / "tests" / "golden"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

# The bundled real ESM-2 8M weights of the reference checkout (present only where it is mounted).
REF_WEIGHTS_8M = Path("/root/reference/esm2_8m_weights.bin")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU; run with -m gpu")


@pytest.fixture(scope="session")
def esm():
    import esm_b200
    esm_b200.lib()
    return esm_b200


@pytest.fixture(scope="session")
def orc():
    import oracle
    oracle.lib()
    return oracle

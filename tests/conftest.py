"""Shared test setup: import paths for the product package and the CPU oracle, the `gpu` marker,
the location of the reference's bundled real 8M weights, and the parity record."""
import json
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT / "codon-infer_b200", ROOT / "oracle", ROOT / "tests" / "golden"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

# The codon-infer checkout: CODON_INFER_REF, else a sibling directory of this repository.
REF_ROOT = Path(os.environ.get("CODON_INFER_REF", str(ROOT.parent / "reference")))
# Its bundled real ESM-2 8M weights (30 MB, never committed). __graft_entry__.build() stages a copy
# under tests/golden/_ref/ (git-ignored) so that machines without the checkout have it too.
_STAGED_8M = ROOT / "tests" / "golden" / "_ref" / "esm2_8m_weights.bin"
REF_WEIGHTS_8M = _STAGED_8M if _STAGED_8M.exists() else REF_ROOT / "esm2_8m_weights.bin"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU; run with -m gpu")


def parity_record(case: str, **numbers) -> None:
    """Appends one JSON line of measured parity figures (max-abs errors, top-1 rates) to the file
    named by ESM_PARITY_LOG, when set, so a run's figures can be reported next to its pass/fail."""
    path = os.environ.get("ESM_PARITY_LOG")
    if not path:
        return
    rec = {"case": case}
    rec.update({k: (float(v) if hasattr(v, "__float__") and not isinstance(v, (int, bool)) else v)
                for k, v in numbers.items()})
    with open(path, "a") as f:
        f.write(json.dumps(rec) + "\n")


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

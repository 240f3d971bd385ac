import json
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")

# Measured parity figures of this session (test name -> {quantity: value}).  Written as JSON to the
# path in $UTTT_PARITY_REPORT at the end of the session, so a GPU run keeps the numbers behind
# every bound, not only pass / fail.
PARITY = {}


def record(name, **values):
    """Keep the measured values of one parity check for the session's report."""
    PARITY.setdefault(name, {}).update({k: (float(v) if isinstance(v, (int, float)) else v)
                                        for k, v in values.items()})


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


def pytest_sessionfinish(session, exitstatus):
    path = os.environ.get("UTTT_PARITY_REPORT")
    if path and PARITY:
        os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
        with open(path, "w") as fh:
            json.dump(PARITY, fh, indent=1, sort_keys=True)


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN

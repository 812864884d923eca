import json
import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"
WEIGHTS = ROOT / "hikoboshi_b200" / "weights" / "Hikoboshi-ProteinMPNN-v48-020.safetensors"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (run with -m gpu)")
    config.addinivalue_line("markers", "slow: long-running CPU oracle comparison")


@pytest.fixture(scope="session")
def weights_path():
    if not WEIGHTS.exists():
        from hikoboshi_b200._build import stage_weights
        stage_weights()
    return WEIGHTS


@pytest.fixture(scope="session")
def oracle(weights_path):
    from oracle.oracle import Oracle
    return Oracle(weights_path)


@pytest.fixture(scope="session")
def upstream():
    return json.loads((GOLDEN / "upstream_fixtures.json").read_text())


@pytest.fixture(scope="session")
def refsyn():
    return dict(np.load(GOLDEN / "ref_synthetic.npz", allow_pickle=False))


def fixture_arrays(rec):
    L = rec["residue_count"]
    c = np.asarray(rec["coords"], np.float32).reshape(L, 5, 3)
    s = np.asarray(rec["sources"], np.uint8).reshape(L, 5)
    return c, s


@pytest.fixture(scope="session")
def engine_fp32(weights_path):
    from hikoboshi_b200 import DesignEngine
    eng = DesignEngine(weights_path, device=0, precision="fp32")
    yield eng
    eng.close()


@pytest.fixture(scope="session")
def engine_f16(weights_path):
    from hikoboshi_b200 import DesignEngine
    eng = DesignEngine(weights_path, device=0, precision="f16")
    yield eng
    eng.close()


@pytest.fixture(scope="session")
def engine_bf16(weights_path):
    from hikoboshi_b200 import DesignEngine
    eng = DesignEngine(weights_path, device=0, precision="bf16")
    yield eng
    eng.close()

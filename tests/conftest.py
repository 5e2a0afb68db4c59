import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "enginesmith-qwen35-08b-long-decode-m5max-round005_b200")
for p in (PKG, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)

SYNTH_DIR = os.environ.get("Q35_SYNTH_DIR", "/tmp/q35_synth_3")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def synth_model_dir():
    import q35
    if not os.path.exists(os.path.join(SYNTH_DIR, "model.safetensors")):
        q35.write_synthetic_model(SYNTH_DIR, 3)
    return SYNTH_DIR


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def oracle_threads():
    import q35_oracle
    q35_oracle.set_threads(min(32, os.cpu_count() or 1))
    return q35_oracle

import json
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden" / "golden.json"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "slow: long-running CPU test")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden():
    return json.loads(GOLDEN.read_text())


@pytest.fixture(scope="session")
def fixture_dir(tmp_path_factory, golden):
    """The seed-0 fixture checkpoint, regenerated and checked against the golden hashes."""
    from safetensors.torch import load_file
    from hexgen2_b200.fixture import create
    import hashlib

    folder = create(tmp_path_factory.mktemp("fixture") / "model", seed=golden["fixture_seed"])
    raw = {}
    for shard in sorted(folder.glob("*.safetensors")):
        raw.update(load_file(str(shard)))
    for k, v in raw.items():
        digest = hashlib.sha256(v.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()
        assert digest == golden["fixture_tensor_sha256"][k], f"fixture tensor {k} differs"
    return folder


def from_bits(values, dtype):
    if dtype == torch.float32:
        return torch.tensor(values, dtype=torch.float32)
    return torch.tensor(values, dtype=torch.int16).view(dtype)

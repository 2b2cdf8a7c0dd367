import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")
    config.addinivalue_line("markers", "slow: long CPU-oracle comparisons")


@pytest.fixture(scope="session")
def bundle_root(tmp_path_factory):
    return tmp_path_factory.mktemp("bundles")


@pytest.fixture(scope="session")
def tiny_bundle(bundle_root):
    from soc_b200.bundle import tiny_config, write_synthetic_bundle
    return write_synthetic_bundle(bundle_root / "tiny", tiny_config(), seed=0)


@pytest.fixture(scope="session")
def make_bundle(bundle_root):
    """Factory: (name, cfg, seed, dtype, quant) -> manifest path, cached per session."""
    from soc_b200.bundle import write_synthetic_bundle
    cache = {}

    def _make(name, cfg, seed=0, dtype="float16", quant=None):
        key = name
        if key not in cache:
            cache[key] = write_synthetic_bundle(bundle_root / name, cfg, seed=seed, dtype=dtype, quant=quant)
        return cache[key]

    return _make


@pytest.fixture(scope="session")
def gpu_ctx():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("gpu test selected but no CUDA device is visible")
    from soc_b200.runtime import Context
    ctx = Context(0)
    yield ctx
    ctx.close()

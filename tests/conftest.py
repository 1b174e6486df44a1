"""Shared fixtures.  `gpu`-marked tests need a B200; the rest run on CPU."""
from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def native():
    """The product library; built in-tree when missing (never a fallback)."""
    from omnivoice_b200 import _native
    if not _native.LIB_PATH.exists():
        from omnivoice_b200 import build
        build.build()
    return _native.lib()


@pytest.fixture(scope="session")
def oracle_lib():
    from oracle import binding
    binding.oracle()
    return binding


@pytest.fixture(scope="session")
def decoding_golden():
    return json.loads((GOLDEN / "decoding_golden.json").read_text())


@pytest.fixture(scope="session")
def cuda_device():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, minor = torch.cuda.get_device_capability(0)
    if (major, minor) != (10, 0):
        pytest.skip(f"needs sm_100 (B200), found sm_{major}{minor}")
    return torch.device("cuda:0")


def small_config(**kw):
    """A reduced-size model with the real kernel shapes (head_dim 128)."""
    from omnivoice_b200 import model_config
    base = dict(vocab_size=4096, hidden_size=256, intermediate_size=512, layers=2, heads=2,
                kv_heads=1)
    base.update(kw)
    return model_config(**base)


def oracle_config_from(cfg):
    from oracle import binding
    names = [f[0] for f in binding.OracleConfig._fields_]
    return binding.OracleConfig(**{n: getattr(cfg, n) for n in names})


os.environ.setdefault("OMNIVOICE_B200_TESTS", "1")

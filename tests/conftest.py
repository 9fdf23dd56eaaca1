import importlib.util
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built CUDA library")
    config.addinivalue_line("markers", "slow: long-running CPU oracle test")


def load_llmrs():
    """The CUDA package (directory llm.rs_b200, loaded by path)."""
    if "llmrs_b200" in sys.modules:
        return sys.modules["llmrs_b200"]
    pkg = os.path.join(ROOT, "llm.rs_b200")
    spec = importlib.util.spec_from_file_location("llmrs_b200", os.path.join(pkg, "__init__.py"),
                                                  submodule_search_locations=[pkg])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["llmrs_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="session")
def llmrs():
    return load_llmrs()


@pytest.fixture(scope="session")
def orc():
    from oracle import oracle as O
    O.lib()
    return O


@pytest.fixture(scope="session")
def ctx(llmrs):
    # GPU tests must run on the CUDA path: no silent skip when the GPU or the
    # library is missing.
    c = llmrs.Context(0)
    yield c
    c.close()


@pytest.fixture(scope="session")
def be(llmrs, ctx):
    return llmrs.CudaBackend(ctx)


@pytest.fixture
def rng():
    return np.random.default_rng(1234)


# model shapes of the batch-1 token-loop configs
CFG_1B = dict(n_layers=16, hidden=2048, n_heads=32, n_kv_heads=8, head_dim=64, ffn=8192, vocab=128256,
              max_seq=256, rms_eps=1e-5, rope_theta=500000.0, weight_format=0, tied_embeddings=1)
CFG_8B = dict(n_layers=32, hidden=4096, n_heads=32, n_kv_heads=8, head_dim=128, ffn=14336, vocab=128256,
              max_seq=4352, rms_eps=1e-5, rope_theta=500000.0, weight_format=0, tied_embeddings=0)
CFG_70B = dict(n_layers=80, hidden=8192, n_heads=64, n_kv_heads=8, head_dim=128, ffn=28672, vocab=128256,
               max_seq=2176, rms_eps=1e-5, rope_theta=500000.0, weight_format=0, tied_embeddings=0)
CFG_TINY = dict(n_layers=2, hidden=256, n_heads=8, n_kv_heads=2, head_dim=32, ffn=512, vocab=1000,
                max_seq=64, rms_eps=1e-5, rope_theta=500000.0, weight_format=0, tied_embeddings=1)


def with_(cfg, **kw):
    c = dict(cfg)
    c.update(kw)
    return c

"""Shared test setup.

Markers: ``gpu`` -- needs a B200 (the driver runs ``-m gpu`` on one and ``-m "not gpu"`` here).
Fixtures build the native libraries in-tree and write the small synthetic GGUF models
(tpt_spark_b200.synth.TINY) once per session.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100a)")


@pytest.fixture(scope="session", autouse=True)
def built_libs():
    from tpt_spark_b200 import _build
    from oracle import oracle

    _build.build()
    oracle.build()


@pytest.fixture(scope="session")
def tiny_models(tmp_path_factory):
    from tpt_spark_b200 import synth

    d = tmp_path_factory.mktemp("models")
    paths = {}
    for name, cfg in synth.TINY.items():
        p = str(d / f"{name}.gguf")
        synth.write_gguf(p, cfg, seed=7)
        paths[name] = p
    return paths


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")

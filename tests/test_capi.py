"""The C ABI library: loads without a GPU, exports every symbol include/tptc.h declares, and
host-only entry points behave as the reference's.  CPU only."""
import ctypes
import os
import re

import numpy as np
import pytest

from tpt_spark_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "tptc.h")).read()
    return sorted(set(re.findall(r"TPTC_API\s+[\w\s\*]+?\b(tptc_\w+)\s*\(", src)))


def test_header_parse_sanity():
    syms = declared_symbols()
    assert "tptc_create" in syms and "tptc_gemv" in syms and len(syms) >= 25


def test_library_exports_every_declared_symbol():
    L = ctypes.CDLL(os.path.join(ROOT, "tpt_spark_b200", "lib", "libtptc.so"))
    missing = [s for s in declared_symbols() if not hasattr(L, s)]
    assert not missing, missing


def test_python_binding_covers_header():
    assert set(declared_symbols()) == set(_lib.SIGNATURES)


def test_version_and_device_count_without_gpu():
    L = _lib.lib()
    assert L.tptc_version().startswith(b"tptc")
    assert L.tptc_device_count() >= 0


def test_create_fails_loudly_without_device():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from tpt_spark_b200.engine import CudaEngine, EngineError

    with pytest.raises(EngineError):
        CudaEngine(0)


def prefix(cached, new):
    a = np.ascontiguousarray(np.asarray(cached, np.uint32))
    b = np.ascontiguousarray(np.asarray(new, np.uint32))
    return _lib.lib().tptc_common_prefix_len(a.ctypes.data if a.size else None, a.size,
                                             b.ctypes.data if b.size else None, b.size)


# The six KvCache tests of the reference (src-tauri/src/engine/wgpu_kvcache.rs:81-133); the
# reset test runs on a device in test_gpu_forward.py.
def test_empty_cache_returns_zero():
    assert prefix([], [1, 2, 3]) == 0


def test_full_prefix_match():
    assert prefix([1, 2, 3], [1, 2, 3, 4, 5]) == 3


def test_diverges_at_second_token():
    assert prefix([1, 99, 3], [1, 2, 3]) == 1


def test_no_match_at_all():
    assert prefix([5, 6, 7], [1, 2, 3]) == 0


def test_new_tokens_shorter_than_cached():
    assert prefix([1, 2, 3, 4, 5], [1, 2, 3]) == 3


def test_prefix_rejects_bad_args():
    L = _lib.lib()
    assert L.tptc_common_prefix_len(None, 3, None, 0) == -1


def test_kernel_entries_reject_bad_arguments_before_any_device_work():
    """Argument checks of the sampling, fused-GEMM and setting entries run on the host: a bad
    call fails with TPTC_ERR_ARG (-1) even without a GPU."""
    L = _lib.lib()
    assert L.tptc_sample(None, 10, None, 1.0, 0.7, 0.9, 1, None, None, None, None, None) == -1
    assert L.tptc_sample(None, 0, None, 1.0, 0.7, 0.9, 1, None, None, None, None, None) == -1
    assert b"sample" in L.tptc_last_error(None)
    assert L.tptc_gemm_q(None, None, None, 4, None) == -1
    assert b"gemm_q" in L.tptc_last_error(None)
    assert L.tptc_set_prefill_fused(None, 1) == -1
    assert L.tptc_set_prefill_gemm_min(None, 16) == -1


def test_profile_cases_usage_without_arguments(capsys):
    from tpt_spark_b200 import profile_cases

    assert profile_cases.main([]) == 2
    assert "gemm_q" in capsys.readouterr().out

"""The pybind11 module dee_b200._pydee: pydee.Engine's routed-expert methods
(dee.cpp/pydee/pydee.cpp:430-509) over the C ABI.  On the host: it builds,
imports, reports a failed init through last_error_message, and applies the
reference binding's argument checks (expert_ids shape, topk equal to
EngineConfig.topk) before any CUDA call."""
import numpy as np
import pytest


@pytest.fixture(scope="module")
def pydee():
    from dee_b200 import build
    build.build()
    build.build_pydee()
    import dee_b200._pydee as m
    return m


def test_module_exposes_the_reference_methods(pydee):
    e = pydee.Engine()
    for name in ("init", "last_error_message", "attach_bank", "moe_forward_batch_device",
                 "moe_forward_combined_device", "sync_status", "close"):
        assert hasattr(e, name), name
    from dee_b200 import _native
    import ctypes
    assert pydee.abi_config_size() == ctypes.sizeof(_native.DeeConfig)


def test_argument_checks_come_before_any_cuda_call(pydee):
    e = pydee.Engine()
    cfg = pydee.EngineConfig(hidden=512, inter=512, num_experts=16, topk=6)
    e.init(cfg)  # fails without a GPU; the checks below do not depend on it
    with pytest.raises(RuntimeError, match=r"shape \[tokens, topk\]"):
        e.moe_forward_batch_device(0, 0, 3, np.zeros((2, 6), np.int32), 6, 0)
    with pytest.raises(RuntimeError, match="does not match EngineConfig.topk"):
        e.moe_forward_batch_device(0, 0, 2, np.zeros((2, 4), np.int32), 4, 0)
    with pytest.raises(RuntimeError, match="does not match EngineConfig.topk"):
        e.moe_forward_combined_device(0, 0, 2, 0, 4, 0, 0, 0, 0)


def test_failed_init_is_reported(pydee):
    import torch
    if torch.cuda.is_available():
        pytest.skip("init succeeds on a GPU host")
    e = pydee.Engine()
    assert e.init(pydee.EngineConfig(hidden=512, inter=512, num_experts=16)) is False
    assert "dee_engine_create failed" in e.last_error_message()
    assert e.moe_forward_batch_device(0, 0, 1, np.zeros((1, 6), np.int32), 6, 0) is False

"""CPU checks of the C-ABI library: it loads, exports every symbol the public
header declares, and fails closed (no compute) when no GPU is visible."""
import ctypes
import os
import re

import pytest

import firewing_b200 as fw

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "fwmoe.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_]*\s*\**\s*([a-z_][a-z0-9_]*)\s*\(",
                       text, flags=re.M)
    return sorted(set(names))


def test_header_declares_the_entry_points():
    names = declared_functions()
    for required in ("fw_moe_create", "fw_moe_forward", "fw_moe_forward_async", "fw_linear_bf16",
                     "fw_route_bf16", "fw_swiglu_bf16", "firewing_cuda_topk_bf16", "fw_last_error"):
        assert required in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(fw.library_path())
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"missing exports: {missing}"


def test_static_library_is_built():
    assert os.path.exists(os.path.join(ROOT, "firewing_b200", "libfwmoe.a"))


def test_invalid_config_is_rejected_before_any_device_call():
    bad = fw.MoeConfig(hidden=100)
    with pytest.raises(fw.FwError) as e:
        fw.MoeBlock(bad)
    assert e.value.code == fw.FW_EINVAL
    with pytest.raises(fw.FwError):
        fw.MoeBlock(fw.MoeConfig(top_k=0))
    with pytest.raises(fw.FwError):
        fw.MoeBlock(fw.MoeConfig(max_tokens=257))


def test_topk_dropin_rejects_shim_invalid_arguments():
    import numpy as np
    v = np.zeros(64, dtype=np.uint16)
    # native/topk_shim.cpp:22-24: k == 0 and k > count fail without work.
    assert fw.topk_bf16(v, 0) is None
    assert fw.topk_bf16(v[:4], 5) is None

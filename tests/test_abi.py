"""CPU checks of the C-ABI library: it loads, exports every entry point that
include/gtmoe.h declares, and fails loudly (no CPU fallback) without a GPU."""
import ctypes
import os
import re

import pytest

from gotransformers_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    text = open(os.path.join(ROOT, "include", "gtmoe.h")).read()
    return sorted(set(re.findall(r"GTMOE_API\s+[\w\s\*]*?\b(gtmoe_\w+)\s*\(", text)))


def test_header_and_binding_agree():
    assert header_functions() == sorted(_lib.EXPORTS)


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    for name in header_functions():
        assert hasattr(L, name), name
    assert L.gtmoe_version() == 100


def test_config_struct_layout():
    # int32 x 8 then a double: 40 bytes, double at offset 32
    assert ctypes.sizeof(_lib.Config) == 40
    assert _lib.Config.clamp_limit.offset == 32


def test_no_cpu_fallback_without_gpu():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from gotransformers_b200 import moe as G

    with pytest.raises(_lib.GtmoeError) as e:
        G.MixtureOfExperts(8, 8, 0, 2, 1)
    assert e.value.code == -2  # GTMOE_ENODEVICE
    assert _lib.lib().gtmoe_bounded_wait_selftest(0) == -2


def test_invalid_config_is_rejected_before_touching_a_device():
    from gotransformers_b200 import moe as G

    with pytest.raises(_lib.GtmoeError) as e:
        G.MixtureOfExperts(8, 8, 0, 2, 3)  # more experts per token than experts
    assert e.value.code == -1 and "experts per token" in str(e.value)
    with pytest.raises(_lib.GtmoeError):
        G.MixtureOfExperts(8, 8, 1, 0, 1)  # no routed experts
    with pytest.raises(_lib.GtmoeError):
        G.MixtureOfExperts(8, 8, -1, 2, 1)  # negative shared

"""The C-ABI library: it loads, exports every entry point include/adai_b200.h declares, and
refuses to run without an sm_100 device instead of falling back to the CPU."""
import ctypes
import os
import re

import pytest

import adai_b200
from adai_b200.api import ModelDesc, load
from adai_b200.config import LARGE, MID, TINY
from adai_b200.synth import tensor_specs
from tests.conftest import ROOT


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "adai_b200.h")).read()
    return sorted(set(re.findall(r"ADAI_B200_API\s+[\w\s\*]*?\b(adai_b200_\w+)\s*\(", text)))


def test_header_declares_the_python_export_list():
    assert declared_symbols() == sorted(adai_b200.EXPORTS)


def test_library_exports_every_declared_symbol():
    lib = load()
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing


@pytest.mark.parametrize("cfg", [TINY, MID, LARGE])
def test_tensor_count_matches_upload_order(cfg):
    lib = load()
    assert lib.adai_b200_model_tensor_count(ctypes.byref(ModelDesc.of(cfg))) == len(tensor_specs(cfg))


def test_null_desc_is_rejected():
    assert load().adai_b200_model_tensor_count(None) == -1


def test_no_cpu_fallback_without_device():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(adai_b200.api.NoDevice):
        adai_b200.Context(0)
    assert "CUDA device" in load().adai_b200_last_error().decode()

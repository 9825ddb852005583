"""The C ABI libraries load and export every entry point their headers
declare, and argument errors come back as the reference's exception
classes without touching a GPU."""
import ctypes
import os
import re

import pytest

import nutllm_b200 as nb

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared(header):
    text = open(os.path.join(ROOT, "include", header)).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(nut_[a-z0-9_]+)\s*\(", text)))


@pytest.mark.parametrize("header,loader", [("nutllm_cuda.h", nb.cuda_lib),
                                           ("nutllm_host.h", nb.host_lib)])
def test_every_declared_symbol_is_exported(header, loader):
    lib = loader()
    names = declared(header)
    assert len(names) >= 4
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, f"{header}: not exported: {missing}"


def test_null_arguments_are_invalid_argument():
    lib = nb.cuda_lib()
    out = ctypes.c_void_p()
    assert lib.nut_model_create(None, 0, ctypes.byref(out)) == nb.NUT_INVALID_ARGUMENT
    assert b"null" in lib.nut_last_error()
    assert lib.nut_qmatrix_create(None, 0, ctypes.byref(out)) == nb.NUT_INVALID_ARGUMENT
    assert lib.nut_kv_create(None, ctypes.byref(out)) == nb.NUT_INVALID_ARGUMENT
    assert lib.nut_decode_token(None, None, 0, None) == nb.NUT_INVALID_ARGUMENT
    assert lib.nut_generate_greedy(None, None, None, 0, 1, 0, None, None, None,
                                   None) == nb.NUT_INVALID_ARGUMENT


def test_invalid_config_rejected_before_device_work():
    """ModelConfig::validate (src/attention.cpp:15-27): heads * head_dim must
    equal dim; the check runs before any allocation."""
    lib = nb.cuda_lib()
    view = nb.ModelView()
    view.config = nb.Config(2, 3, 10, 4, 8, 16, 8, 1, 3)  # 3 * 4 != 10
    view.quant_type = nb.INT8
    view.n_layers = 2
    out = ctypes.c_void_p()
    status = lib.nut_model_create(ctypes.byref(view), 0, ctypes.byref(out))
    assert status == nb.NUT_INVALID_ARGUMENT
    assert lib.nut_last_error() == b"model config: invalid dimensions"


def test_status_codes_map_to_reference_exception_classes():
    for code, exc in [(nb.NUT_INVALID_ARGUMENT, ValueError), (nb.NUT_OUT_OF_RANGE, IndexError),
                      (nb.NUT_LENGTH_ERROR, nb.LengthError), (nb.NUT_RANGE_ERROR, nb.RangeError),
                      (nb.NUT_RUNTIME_ERROR, RuntimeError), (nb.NUT_DEVICE_TIMEOUT, nb.DeviceTimeout)]:
        with pytest.raises(exc):
            nb._check(code)

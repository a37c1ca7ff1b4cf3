"""The C ABI library loads, exports every declared entry point, and rejects bad
arguments on the host before any launch (CPU only: no compute calls)."""

import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _declared():
    text = (ROOT / "include" / "ksd8.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*)\s+(ksd8_\w+)\(", text, re.M)))


def test_library_exports_every_declared_symbol():
    from ksdraft_b200 import _lib
    lib = _lib.load()
    names = _declared()
    assert len(names) >= 15
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) <= set(_lib.SIGNATURES), set(names) - set(_lib.SIGNATURES)


def test_status_strings_and_version():
    from ksdraft_b200 import _lib
    assert _lib.load().ksd8_version() == 1
    assert _lib.status_string(0) == "ok"
    assert "shape" in _lib.status_string(_lib.ERR_SHAPE)


def test_host_side_validation_without_launch():
    from ksdraft_b200 import _lib
    lib = _lib.load()
    # group != 128 -> unsupported, checked before anything touches the device
    assert lib.ksd8_quantize_rows(None, 0, 1, 128, 128, 32, 0, 0.0, 0, 0, None, 128, None, None,
                                  None) == _lib.ERR_UNSUPPORTED
    assert lib.ksd8_quantize_rows(None, 9, 1, 128, 128, 128, 0, 0.0, 0, 0, None, 128, None,
                                  None, None) == _lib.ERR_DTYPE
    assert lib.ksd8_w8a8_gemm(None, None, None, None, 4, 4, 100, 128, None, 0, 4, None, 0, None,
                              None) == _lib.ERR_SHAPE
    assert lib.ksd8_w8a8_gemm(None, None, None, None, 4, 4, 128, 64, None, 0, 4, None, 0, None,
                              None) == _lib.ERR_UNSUPPORTED
    assert lib.ksd8_rosa_match(None, None, None, 1, 1, 10, 70, None, None, 0, 0, 0, 0, None,
                               None, None, None) == _lib.ERR_ARG
    assert lib.ksd8_ks3_vjp(None, None, 4, 100, None, None, None, None, None, None, None, None,
                            None, None, None, None, None) == _lib.ERR_SHAPE
    # Rosa credits: cap beyond the 64-bit window, T beyond the kernel's limit,
    # missing buffers -- all rejected before any device call
    assert lib.ksd8_rosa_credits(None, None, None, 1, 4, 65, None, None, None, None, None,
                                 None) == _lib.ERR_ARG
    assert lib.ksd8_rosa_credits(None, None, None, 1, 20000, 62, None, None, None, None, None,
                                 None) == _lib.ERR_UNSUPPORTED
    assert lib.ksd8_rosa_credits(None, None, None, 1, 8, 7, None, None, None, None, None,
                                 None) == _lib.ERR_ARG
    assert lib.ksd8_rosa_set_algorithm(5) == _lib.ERR_ARG


def test_status_mapping_to_reference_exceptions():
    from ksdraft_b200 import _lib
    with pytest.raises(ValueError):
        _lib.check(_lib.ERR_SHAPE, "x")
    with pytest.raises(TypeError):
        _lib.check(_lib.ERR_DTYPE, "x")
    with pytest.raises(RuntimeError):
        _lib.check(_lib.ERR_TIMEOUT, "x")


def test_cpu_tensors_are_rejected_not_computed():
    import torch
    from ksdraft_b200.kernels.quant import quantize_last_dim
    from ksdraft_b200.model.rosa import _match_payload_sign
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        quantize_last_dim(torch.randn(2, 128))
    b = torch.zeros(1, 8, dtype=torch.int8)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        _match_payload_sign(b, b, b)
    with pytest.raises(TypeError):
        quantize_last_dim(torch.ones(2, 4, dtype=torch.int32))


def test_sm_reserve_setting_is_host_only_and_bounded():
    from ksdraft_b200 import _lib
    lib = _lib.load()
    assert lib.ksd8_get_sm_reserve() == 0
    try:
        assert lib.ksd8_set_sm_reserve(16) == 0
        assert lib.ksd8_get_sm_reserve() == 16
        assert lib.ksd8_set_sm_reserve(-1) == _lib.ERR_ARG
        assert lib.ksd8_set_sm_reserve(100000) == _lib.ERR_ARG
        assert lib.ksd8_get_sm_reserve() == 16      # a rejected value changes nothing
    finally:
        assert lib.ksd8_set_sm_reserve(0) == 0

"""The C ABI library: loads without a GPU, exports every declared symbol,
validates arguments on the host and honours host-side fault injection
(no kernel is launched by any call in this file)."""

import ctypes

import pytest

from comfyui_vc_attention_b200.vc_attention import _native as N


def test_library_loads_and_exports_every_declared_symbol():
    lib = N.lib()
    declared = N.declared_symbols()
    assert len(declared) >= 13
    for name in declared:
        assert hasattr(lib, name), name
    assert set(declared) == set(N._SIGNATURES)


def test_abi_version():
    assert N.lib().vcattn_abi_version() == 1


def test_workspace_sizes_are_sane():
    lib = N.lib()
    assert lib.vcattn_kmeans_workspace_bytes(2, 1024, 128, 16, 16) > 2 * 1024 * 4
    assert lib.vcattn_kmeans_workspace_bytes(0, 1024, 128, 16, 16) == 0
    big = lib.vcattn_prepare_workspace_bytes(56, 65536, 128)
    assert 56 * 128 * 8 < big < 64 << 20


def test_argument_validation_returns_status_without_launching():
    lib = N.lib()
    rc = lib.vcattn_attn_fp8(None, None, None, None, None, None, None, 1, 2, 1024, 1024, 128, 64,
                             0.1, 0, -0.35, None, 0, 0, 0, 0, None)
    assert rc == N.ERR_ARG
    assert b"null pointer" in lib.vcattn_last_error()
    v = N.BHND(None, 0, 0, 0)
    rc = lib.vcattn_kmeans(ctypes.byref(v), 0, 1, 2, 1024, 96, 16, 3, None, None, 0, None, None,
                           None, None, 0, None)
    assert rc == N.ERR_ARG and b"D must be 64 or 128" in lib.vcattn_last_error()
    rc = lib.vcattn_expcast_codes(None, None, 4, 4, -0.35, 7, None, None)
    assert rc == N.ERR_ARG


def test_fault_injection_is_host_side():
    lib = N.lib()
    N.inject_fault("vcattn_attn_fp8")
    try:
        rc = lib.vcattn_attn_fp8(None, None, None, None, None, None, None, 1, 2, 1024, 1024, 128,
                                 64, 0.1, 0, -0.35, None, 0, 0, 0, 0, None)
        assert rc == N.ERR_INJECTED
        with pytest.raises(N.VCAttnError) as ei:
            N.check("vcattn_attn_fp8", rc)
        assert ei.value.code == N.ERR_INJECTED
    finally:
        N.inject_fault(None)
    rc = lib.vcattn_attn_fp8(None, None, None, None, None, None, None, 1, 2, 1024, 1024, 128, 64,
                             0.1, 0, -0.35, None, 0, 0, 0, 0, None)
    assert rc == N.ERR_ARG

"""vcattn_prepare_fp8_noalloc: prepare without a caller-provided workspace.

Some callers cannot allocate device memory (a host that owns every device
byte through its own pool, or an FFI binding with no device allocator).  For
them the library keeps its prepare scratch in a fixed 16 MiB array of its
own.  This file checks, through the C ABI, that two calls in a row give
exactly the bytes of the workspace entry point, and that a shape whose
scratch does not fit is refused before anything is launched.

It sits in a file of its own, named so that pytest collects it last, and runs
the same in a fresh process or after the other tests.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle.inputs import make_qkv

pytestmark = pytest.mark.gpu


def _run_prepare(lib, N, q, k, v, perm, br, noalloc):
    b, h, n, d = q.shape
    g = b * h
    n_pad = -(-n // br) * br
    nb = n_pad // br
    dev = q.device
    out = {
        "q8": torch.empty((g, n_pad, d), dtype=torch.uint8, device=dev),
        "qs": torch.empty((g, n_pad), dtype=torch.float32, device=dev),
        "k8": torch.empty((g, n_pad, d), dtype=torch.uint8, device=dev),
        "ks": torch.empty((g, n_pad), dtype=torch.float32, device=dev),
        "v8": torch.empty((g, n_pad, d), dtype=torch.uint8, device=dev),
        "vs": torch.empty((g, nb, d), dtype=torch.float32, device=dev),
        "mu": torch.empty((g, nb, d), dtype=torch.float32, device=dev),
        "v8t": torch.empty((g, nb, d, br), dtype=torch.uint8, device=dev),
    }
    for t in out.values():   # poison, so stale memory cannot pass for a result
        t.fill_(0x5A if t.dtype == torch.uint8 else float("nan"))
    views = [N.BHND(t.data_ptr(), t.stride(0), t.stride(1), t.stride(2)) for t in (q, k, v)]
    flags = N.HADAMARD | N.SMOOTH_K
    stream = torch.cuda.current_stream(dev).cuda_stream
    common = (ctypes.byref(views[0]), ctypes.byref(views[1]), ctypes.byref(views[2]), N.DTYPE_BF16,
              b, h, n, d, perm.data_ptr(), g, br, flags,
              out["q8"].data_ptr(), out["qs"].data_ptr(), out["k8"].data_ptr(), out["ks"].data_ptr(),
              out["v8"].data_ptr(), out["vs"].data_ptr(), out["mu"].data_ptr(), out["v8t"].data_ptr(),
              None)
    if noalloc:
        rc = lib.vcattn_prepare_fp8_noalloc(*common, stream)
        N.check("vcattn_prepare_fp8_noalloc", rc)
    else:
        ws_bytes = lib.vcattn_prepare_workspace_bytes(g, n, d)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        rc = lib.vcattn_prepare_fp8(*common, ws.data_ptr(), ws_bytes, stream)
        N.check("vcattn_prepare_fp8", rc)
    torch.cuda.synchronize(dev)
    return {key: t.cpu().numpy() for key, t in out.items()}


@pytest.fixture(scope="module")
def native():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from comfyui_vc_attention_b200.vc_attention import _native
    _native.lib()
    return _native


def test_noalloc_prepare_matches_workspace_entry_point(native):
    lib = native.lib()
    dev = torch.device("cuda:0")
    b, h, n, d, br = 1, 3, 1000, 128, 128
    q, k, v = (torch.from_numpy(a).to(dev).to(torch.bfloat16) for a in make_qkv(b, h, n, d, seed=17))
    perm = torch.stack([torch.randperm(n, generator=torch.Generator().manual_seed(i)) for i in range(h)])
    perm = perm.to(torch.int32).to(dev)
    ref = _run_prepare(lib, native, q, k, v, perm, br, noalloc=False)
    for _ in range(2):   # two calls in a row share (and reuse) the static scratch
        got = _run_prepare(lib, native, q, k, v, perm, br, noalloc=True)
        for key in ref:
            if got[key].dtype == np.float32:
                assert not np.isnan(got[key]).any(), key
            np.testing.assert_array_equal(got[key], ref[key], err_msg=key)
    # a second, differently shaped call right after still matches
    q2, k2, v2 = (torch.from_numpy(a).to(dev).to(torch.bfloat16) for a in make_qkv(1, 2, 640, d, seed=18))
    perm2 = torch.arange(640, dtype=torch.int32, device=dev).flip(0).repeat(2, 1).contiguous()
    ref2 = _run_prepare(lib, native, q2, k2, v2, perm2, 64, noalloc=False)
    got2 = _run_prepare(lib, native, q2, k2, v2, perm2, 64, noalloc=True)
    for key in ref2:
        np.testing.assert_array_equal(got2[key], ref2[key], err_msg=key)


def test_noalloc_prepare_refuses_shapes_beyond_its_scratch(native):
    lib = native.lib()
    # 512 heads x 65536 tokens needs 512 * 256 * 128 * 8 bytes of partial sums,
    # far above 16 MiB: refused on the host, before pointers are even looked at.
    # The code and scale pointers are stand-ins that are never dereferenced.
    dummy = native.BHND(None, 0, 0, 0)
    fake = ctypes.c_void_p(4096)
    rc = lib.vcattn_prepare_fp8_noalloc(ctypes.byref(dummy), ctypes.byref(dummy), ctypes.byref(dummy),
                                        native.DTYPE_BF16, 1, 512, 65536, 128, None, 0, 128,
                                        native.HADAMARD | native.SMOOTH_K, fake, fake, fake, fake,
                                        fake, fake, fake, None, None, None)
    assert rc == native.ERR_ARG
    msg = lib.vcattn_last_error().decode()
    assert "limit" in msg and "vcattn_prepare_fp8" in msg


def test_noalloc_prepare_honours_host_fault_injection(native):
    """The router's fallback test hook reaches this entry point too: while the
    fault is set it returns the injected-fault status and launches nothing."""
    lib = native.lib()
    dummy = native.BHND(None, 0, 0, 0)
    lib.vcattn_inject_fault(b"vcattn_prepare_fp8_noalloc")
    try:
        rc = lib.vcattn_prepare_fp8_noalloc(ctypes.byref(dummy), ctypes.byref(dummy), ctypes.byref(dummy),
                                            native.DTYPE_BF16, 1, 1, 128, 128, None, 0, 128,
                                            native.HADAMARD | native.SMOOTH_K, None, None, None, None,
                                            None, None, None, None, None, None)
    finally:
        lib.vcattn_inject_fault(None)
    assert rc == native.ERR_INJECTED
    assert "injected" in lib.vcattn_last_error().decode()

"""Bounded waits of the tcgen05 kernels, made to run out on purpose.

Every mbarrier wait in the kernels gives up after a limit, sets the CTA's
abort word and the device status word, and the CTA drains its copies and
MMAs, frees its tensor memory and returns.  Here the dense kernel's producer
is told (vcattn_inject_stall) to issue no copies from KV tile 2 on: the
waits on tile 2 find nothing to wait for and give up after their limit
(about 2 s; every CTA of the small grid waits at once).  No fault, trap or
unbounded wait is involved; the launch returns, the status names the wait,
and the context stays usable for a normal call afterwards.
"""

import numpy as np
import pytest
import torch

from oracle import vc_oracle as O
from oracle.inputs import make_qkv

pytestmark = pytest.mark.gpu

# the waits on KV tile 2: MMA issuer (3), softmax (7), correction (11, 12),
# per-tile factors (13)
WAITS_ON_A_TILE = {3, 7, 11, 12, 13}


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from comfyui_vc_attention_b200.vc_attention import _native as N
    N.lib()
    return torch.device("cuda:0")


def _run(dev, q, k, v, perm):
    from comfyui_vc_attention_b200.vc_attention.kernels.cuda_attn import TritonConfig, attention_prepared, prepare
    b, h, n, d = q.shape
    p = prepare(*(torch.from_numpy(a).to(dev).to(torch.bfloat16) for a in (q, k, v)),
                torch.from_numpy(perm).to(dev), block_rows=128, want_v=True)
    out = torch.zeros((b, h, n, d), dtype=torch.float32, device=dev)
    attention_prepared(p, n, out, d ** -0.5, TritonConfig(block_n=128, enable_expcast=True), kernel="tc")
    torch.cuda.synchronize()
    return out.cpu().numpy().reshape(b * h, n, d)


def test_wait_that_runs_out_reports_and_the_context_stays_usable(dev):
    from comfyui_vc_attention_b200.vc_attention import _native as N
    from comfyui_vc_attention_b200.vc_attention.kernels.cuda_attn import attention_status
    h, n, d = 1, 1024, 128
    q, k, v = make_qkv(1, h, n, d, seed=51)
    perm = np.random.default_rng(5).permutation(n).astype(np.int32)[None]
    assert attention_status(reset=True) == (0, 0, 0)
    N.inject_stall(2)
    try:
        _run(dev, q, k, v, perm)             # returns: every wait is bounded
        code, where, block = attention_status(reset=True)
    finally:
        N.inject_stall(-1)
    assert code == 1, "a wait on the missing tile must have given up"
    assert where in WAITS_ON_A_TILE, where
    assert 0 <= block < n // 128
    # the same call without the stall, in the same context
    got = _run(dev, q, k, v, perm)
    assert attention_status() == (0, 0, 0)
    prep = O.prepare(q.reshape(h, n, d), k.reshape(h, n, d), v.reshape(h, n, d), perm, block_rows=128)
    ref = O.attention_codes(prep, n, 128, 128, d ** -0.5, expcast=True)
    assert O.rel_l2(got, ref) <= 1e-3

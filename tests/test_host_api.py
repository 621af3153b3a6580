"""Host-side interface (no GPU): schedule, cache, router gating, hooks, step
counter and the ComfyUI nodes.  Mirrors the reference's tests/test_install.py."""

import torch

from comfyui_vc_attention_b200.vc_attention.h3 import H3, estimate_tokens, recommended_config
from comfyui_vc_attention_b200.vc_attention.patch import (VCAttentionConfig, VCAttentionRuntime, _try_vc,
                                                          get_runtime, install,
                                                          install_attention_override, is_installed,
                                                          kernel_status, uninstall)
from comfyui_vc_attention_b200.vc_attention.schedule import GroupSchedule, PermutationCache, StepTracker


def test_h3_schedule():
    h3 = recommended_config(total_steps=8)
    assert h3["group_steps"] == 2 and h3["block_rows"] == 128
    rt = VCAttentionRuntime(VCAttentionConfig(total_steps_hint=8))
    s = rt.schedule
    assert s.should_group(0, 8) and s.should_group(1, 8) and not s.should_group(2, 8)
    assert s.should_recompute(0) and not s.should_recompute(1) and s.should_recompute(4)
    assert GroupSchedule(group_fraction=0.0).group_steps(8) == 1
    assert GroupSchedule(group_fraction=0.5).group_steps(20) == 10
    assert H3.qkv_dim == 7168 and H3.rope_dims == 96
    est = estimate_tokens(243, 768, 1344, audio_seconds=10.1)
    assert est["latent_grid"] == (61, 24, 42) and est["audio"] == 404


def test_step_tracker_and_cache():
    t = StepTracker()
    assert t.current == 0
    t.begin_step(); t.begin_step()
    assert t.current == 1
    t.observe_total(20)
    assert t.total_steps == 20
    t.reset()
    assert t.index == -1 and t.total_steps is None
    c = PermutationCache(max_entries=2)
    assert c.get(0, 10, 2) is None and c.misses == 1
    c.put(0, 10, 2, "p0", "c0")
    c.put(1, 10, 2, "p1", "c1")
    c.put(2, 10, 2, "p2", "c2")      # FIFO: evicts bucket 0
    assert c.get(0, 10, 2) is None and c.get(2, 10, 2) == ("p2", "c2") and c.hits == 1
    assert len(c) == 2
    c.clear()
    assert len(c) == 0 and c.hits == 0


def test_runtime_gating_on_cpu():
    rt = VCAttentionRuntime(VCAttentionConfig(min_tokens=256))
    q = torch.randn(1, 2, 512, 128)
    assert rt.attention(q, q, q) is None                      # CPU tensors defer
    assert rt.attention(q, q, q, is_causal=True) is None
    assert rt.attention(q, q, q, attn_mask=torch.ones(1)) is None
    assert rt.attention(q[..., :96], q[..., :96], q[..., :96]) is None
    assert rt.attention(q[:, :, :100], q[:, :, :100], q[:, :, :100]) is None
    assert rt.stats["calls"] == 5 and rt.stats["skipped"] == 5 and rt.stats["used"] == 0


def test_sdpa_hook_falls_through_and_uninstalls():
    orig = torch.nn.functional.scaled_dot_product_attention
    install(VCAttentionConfig(enabled=True, min_tokens=256), model=None)
    try:
        assert is_installed()
        q, k, v = (torch.randn(1, 4, 512, 128) for _ in range(3))
        got = torch.nn.functional.scaled_dot_product_attention(q, k, v)
        assert torch.allclose(got, orig(q, k, v))
        assert get_runtime().stats["calls"] > 0
    finally:
        uninstall()
    assert torch.nn.functional.scaled_dot_product_attention is orig
    assert not is_installed()


class _FakeDenoiser:
    def __init__(self):
        self.calls = 0

    def forward(self, *a, **kw):
        self.calls += 1


class _FakeModel:
    def __init__(self):
        self.diffusion_model = _FakeDenoiser()
        self.model_options = {"transformer_options": {}}


def test_step_counter_and_override_chain():
    model = _FakeModel()
    rt = install(VCAttentionConfig(), model=model)
    try:
        for _ in range(3):
            model.diffusion_model.forward(transformer_options={"sample_sigmas": list(range(21))})
        assert rt.tracker.index == 2 and rt.tracker.total_steps == 20
        ov = model.model_options["transformer_options"]["optimized_attention_override"]
        calls = []

        def func(q, k, v, heads, **kw):
            calls.append(heads)
            return "original"

        q = torch.randn(1, 64, 256)           # 3-D ComfyUI layout, CPU -> defers
        assert ov(func, q, q, q, 2) == "original" and calls == [2]
    finally:
        uninstall()
    assert "optimized_attention_override" not in model.model_options["transformer_options"]


def test_override_priority_defer_and_front():
    model = _FakeModel()
    prev_calls = []

    def prev(func, *a, **kw):
        prev_calls.append(1)
        return "prev"

    model.model_options["transformer_options"]["optimized_attention_override"] = prev
    rt = VCAttentionRuntime(VCAttentionConfig(override_priority="defer"))
    assert install_attention_override(rt, model) is False
    assert model.model_options["transformer_options"]["optimized_attention_override"] is prev
    assert install_attention_override(rt, model, priority="front") is True
    ov = model.model_options["transformer_options"]["optimized_attention_override"]
    assert ov is not prev and ov._vc_prev is prev
    q = torch.randn(1, 64, 256)
    assert ov(lambda *a, **k: "func", q, q, q, 2) == "prev" and prev_calls == [1]
    uninstall()
    assert model.model_options["transformer_options"]["optimized_attention_override"] is prev


def test_try_vc_reshapes_3d_and_4d(monkeypatch):
    seen = {}

    class RT:
        config = VCAttentionConfig()

        def attention(self, q, k, v, attn_mask=None):
            seen["shape"] = tuple(q.shape)
            seen["stride"] = q.stride()
            seen["mask"] = attn_mask
            return None if attn_mask is not None else q * 2

    q3 = torch.randn(2, 10, 4 * 8)
    out = _try_vc(RT(), q3, q3, q3, 4)
    assert seen["shape"] == (2, 4, 10, 8) and seen["stride"] == (320, 8, 32, 1)   # a view, no copy
    assert torch.allclose(out, q3 * 2)
    q4 = torch.randn(2, 4, 10, 8)
    assert torch.allclose(_try_vc(RT(), q4, q4, q4, 4, skip_output_reshape=True), q4 * 2)
    m = torch.ones(1)
    assert _try_vc(RT(), q3, q3, q3, 4, mask=m) is None and seen["mask"] is m   # handed to the runtime
    assert _try_vc(RT(), q3, q3, q3, 5) is None


def test_nodes_execute():
    import comfyui_vc_attention_b200 as pkg

    class DummyModel:
        pass

    Node = pkg.VCAttentionMiniMaxH3
    assert "model" in Node.INPUT_TYPES()["required"]
    assert pkg.NODE_DISPLAY_NAME_MAPPINGS["VCAttentionMiniMaxH3"] == "VC Attention (MiniMax-H3)"
    try:
        out = Node().apply(model=DummyModel())
        assert isinstance(out, tuple) and out[0] is not None
        for kw in ({"backend": "reference"}, {"backend": "fp8", "enable_expcast": True},
                   {"backend": "nvfp4", "total_steps": 20, "block_rows": 64, "min_tokens": 512},
                   {"enable_vsmooth": False, "modality_aware": True, "kmeans_iters": 1, "reuse_every": 1}):
            Node().apply(model=DummyModel(), **kw)
        assert isinstance(pkg.VCAttentionDisable().apply(model=DummyModel()), tuple)
    finally:
        uninstall()
    assert "inactive" in kernel_status()


def test_mma_key_slot_is_an_involution_within_32_row_chunks():
    """VCATTN_V_MMA_ORDER: the V-row order of the tcgen05 kernel transposes
    (row/8 % 4, row/2 % 4) inside each 32-row chunk and is its own inverse."""
    import torch
    from comfyui_vc_attention_b200.vc_attention.kernels.cuda_attn import mma_key_slot
    r = torch.arange(256)
    s = mma_key_slot(r)
    assert torch.equal(mma_key_slot(s), r)
    assert torch.equal(torch.sort(s).values, r)
    assert torch.equal(s // 32, r // 32)
    # thread q of the 16x256b fragment holds keys 8r + 2q + e; their P bytes
    # sit at A-operand positions 8q + 2r + e, where V row 8r + 2q + e must be
    for q in range(4):
        for rr in range(4):
            for e in range(2):
                assert int(mma_key_slot(torch.tensor(8 * rr + 2 * q + e))) == 8 * q + 2 * rr + e


def test_host_chunk_bounds_cover_every_unit_once():
    """vc_attention_host's unit ranges: contiguous, non-empty, covering [0, G),
    at most c units each, the last c units in shrinking pieces."""
    from comfyui_vc_attention_b200.vc_attention.kernels.cuda_attn import _chunk_bounds
    for g in range(1, 130):
        for c in (1, 2, 3, 4, 7, 8, 16):
            b = _chunk_bounds(g, c)
            assert b[0][0] == 0 and b[-1][1] == g
            assert all(x[1] == y[0] for x, y in zip(b, b[1:]))
            assert all(0 < hi - lo <= c for lo, hi in b)
            if g > 1:
                assert b[-1][1] - b[-1][0] == 1
    assert [hi - lo for lo, hi in _chunk_bounds(56, 4)] == [4] * 13 + [2, 1, 1]


def test_key_padding_mask_forms():
    """Which attention masks the router accepts: key padding only (the same
    for every head and query), as bool (True = attend) or additive 0/-inf."""
    from comfyui_vc_attention_b200.vc_attention.patch import key_padding_mask
    b, n = 2, 8
    keep = torch.ones(b, n, dtype=torch.bool)
    keep[0, 6:] = False
    keep[1, 3] = False
    got = key_padding_mask(keep[:, None, None, :], b, n)
    assert torch.equal(got, keep)
    add = torch.zeros(b, 1, n)
    add[:, 0][~keep] = float("-inf")
    assert torch.equal(key_padding_mask(add, b, n), keep)              # (B, 1, S) -> (B, 1, 1, S)
    assert torch.equal(key_padding_mask(keep[0], b, n), keep[0].expand(b, n))   # (S,) broadcast
    assert key_padding_mask(torch.zeros(b, 1, n) + 0.5, b, n) is None      # a real bias
    assert key_padding_mask(torch.ones(b, 1, 4, n, dtype=torch.bool), b, n) is None   # varies by query
    assert key_padding_mask(torch.ones(b, 3, 1, n, dtype=torch.bool), b, n) is None   # varies by head
    assert key_padding_mask(torch.ones(b, 1, 1, n + 1, dtype=torch.bool), b, n) is None
    assert key_padding_mask(torch.ones(b, n, dtype=torch.int32), b, n) is None


def test_tau_schedule_across_steps():
    """Dense for the first steps, then tau moving linearly to its end value;
    the runtime hands each step's (sparse, tau) to the kernel config."""
    from comfyui_vc_attention_b200.vc_attention.schedule import TauSchedule
    ts = TauSchedule(tau_start=1.0, tau_end=2.0, dense_steps=2)
    assert ts.tau(0, 8) is None and ts.tau(1, 8) is None
    assert ts.tau(2, 8) == 1.0 and ts.tau(7, 8) == 2.0
    assert abs(ts.tau(5, 8) - 1.6) < 1e-12
    assert ts.tau(9, 8) == 2.0                      # past the announced total: stays at the end
    rt = VCAttentionRuntime(VCAttentionConfig(tau_schedule=(1.0, 2.0, 2), total_steps_hint=8))
    got = []
    for _ in range(8):
        rt.begin_step()
        got.append(rt.sparsity(16384))
    assert got[0] == (False, 1.3) and got[1] == (False, 1.3)
    assert got[2] == (True, 1.0) and got[7] == (True, 2.0)
    assert rt.sparsity(1024)[0] is False            # below sparsity_min_tokens: always dense
    plain = VCAttentionRuntime(VCAttentionConfig())
    assert plain.sparsity(16384) == (True, 1.3)

"""The token mixer end to end: rotary q/k, selection, attention, o_proj, decode cache.

Compared with the reference's own PyramidSparseAttention (xmixers, from the
offline install under baseline/_ref) run with its torch backend on the same
GPU and the same weights; skipped when that install is absent.  The rotary
kernel is compared with the reference's fp32 formula (rotary_torch.py:5-9).
"""

import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


def _config(**kw):
    base = dict(hidden_size=256, num_attention_heads=8, num_key_value_heads=2, head_dim=64, attention_method="pisa",
                block_size=16, topk=8, prefill_routing="auto", leaf_tile=4, force_first=True, force_recent=1,
                rope_theta=10000.0, rope_fraction=0.5, rope_position_mode="document", bias=False, backend="auto")
    base.update(kw)
    return SimpleNamespace(**base)


def _rotary_reference(x, theta, positions):
    angles = positions.to(device=x.device, dtype=torch.float32)[..., None, None] * theta.flatten().float()
    first, second = x.float().chunk(2, -1)
    c, s = angles.cos(), angles.sin()
    return torch.cat((first * c - second * s, first * s + second * c), -1).to(x.dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_rotary_matches_reference_formula(cuda_device, dtype):
    from nlogn_pisa_b200.mixer import RotaryEmbedding, token_positions

    g = torch.Generator(device=cuda_device).manual_seed(1)
    x = torch.randn(2, 300, 4, 64, generator=g, device=cuda_device).to(dtype)
    rope = RotaryEmbedding(64, 10000.0, 0.5).to(cuda_device)
    cu = torch.tensor([0, 100, 300], device=cuda_device)
    for positions in (token_positions(300, cuda_device), token_positions(300, cuda_device, cu, 0) + 7):
        got = rope(x, positions)
        want = _rotary_reference(x, rope.theta, positions)
        tol = 1e-5 if dtype == torch.float32 else 1e-2
        torch.testing.assert_close(got.float(), want.float(), atol=tol, rtol=tol)
    # gradient: the transpose rotation
    xr = x.float().requires_grad_(True)
    rope(xr, positions).square().sum().backward()
    xt = x.float().requires_grad_(True)
    _rotary_reference(xt, rope.theta, positions).square().sum().backward()
    torch.testing.assert_close(xr.grad, xt.grad, atol=1e-4, rtol=1e-4)


def _reference_mixer_class(monkeypatch):
    ref = ROOT / "baseline" / "_ref"
    if not (ref / "xmixers").exists():
        pytest.skip("the reference package is not installed under baseline/_ref")
    if str(ref) not in sys.path:
        sys.path.append(str(ref))
    try:
        import xmixers.modules.pes.lrpe as lrpe
        from xmixers.modules.token_mixers.vanilla_attention.pyramid_sparse_attention import PyramidSparseAttention
    except Exception as exc:
        pytest.skip(f"reference mixer not importable: {type(exc).__name__}")
    # the reference's eager rotary formula instead of its Triton kernel
    monkeypatch.setattr(lrpe, "rotary_fn", lambda x, f, p, use_triton=True: _rotary_reference(x, f, p))
    return PyramidSparseAttention


@pytest.mark.parametrize("method", ["pisa", "pisa2"])
def test_mixer_matches_reference_prefill_and_decode(cuda_device, monkeypatch, method):
    from nlogn_pisa_b200.mixer import PyramidSparseAttention

    RefMixer = _reference_mixer_class(monkeypatch)
    cfg = _config(attention_method=method)
    torch.manual_seed(3)
    ref = RefMixer(cfg).to(cuda_device)
    ours = PyramidSparseAttention(cfg).to(cuda_device)
    ours.load_state_dict(ref.state_dict())
    torch.testing.assert_close(ours.rope.theta, ref.rope.theta.to(cuda_device))
    g = torch.Generator(device=cuda_device).manual_seed(4)
    x = torch.randn(2, 200, cfg.hidden_size, generator=g, device=cuda_device)
    steps = torch.randn(2, 3, cfg.hidden_size, generator=g, device=cuda_device)
    with torch.no_grad():
        want, ref_cache = ref(x, use_cache=True, backend="torch")
        got, cache = ours(x, use_cache=True)
        torch.testing.assert_close(got, want, atol=2e-3, rtol=2e-3)
        assert set(cache) == set(ref_cache)
        for i in range(3):
            want, ref_cache = ref(steps[:, i:i + 1], cache=ref_cache, use_cache=True, backend="torch")
            got, cache = ours(steps[:, i:i + 1], cache=cache, use_cache=True)
            torch.testing.assert_close(got, want, atol=2e-3, rtol=2e-3)
            assert cache["k"].shape == ref_cache["k"].shape
            np.testing.assert_array_equal(cache["pyramid"].level_sizes, ref_cache["pyramid"].level_sizes)


def test_mixer_packed_documents_and_backward(cuda_device):
    """cu_seqlens prefill (document-relative positions) with gradients to the weights."""
    from nlogn_pisa_b200.mixer import PyramidSparseAttention

    cfg = _config(attention_method="pisa2")
    torch.manual_seed(5)
    mixer = PyramidSparseAttention(cfg).to(cuda_device).to(torch.bfloat16)
    g = torch.Generator(device=cuda_device).manual_seed(6)
    x = torch.randn(1, 300, cfg.hidden_size, generator=g, device=cuda_device).to(torch.bfloat16)
    cu = torch.tensor([0, 120, 300], device=cuda_device)
    out, _ = mixer(x, cu_seqlens=cu)
    out.float().square().mean().backward()
    for name, p in mixer.named_parameters():
        assert p.grad is not None and torch.isfinite(p.grad.float()).all(), name
    # each document alone gives the same rows
    with torch.no_grad():
        a, _ = mixer(x[:, :120])
        b, _ = mixer(x[:, 120:])
        torch.testing.assert_close(out.detach(), torch.cat([a, b], 1), atol=0, rtol=0)

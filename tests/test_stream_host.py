"""Host parts of the CPU-master streaming trainer (megaslide_b200/stream.py) and the DiT model around
the attention (megaslide_b200/dit.py), on CPU: the flat-buffer AdamW against torch.optim.AdamW, and
the model's parameter names / shapes against the reference's MegaSlideDiT."""

import sys
from pathlib import Path

import pytest
import torch

from megaslide_b200.dit import MegaSlideDiT, VideoDiTConfig
from megaslide_b200.stream import _HostAdamW

import os

# checkout of the reference repository (jasonliu0704/megaslide); the tests that import its model skip
# when it is absent
REF = Path(os.environ.get("MEGASLIDE_REFERENCE", str(Path(__file__).resolve().parents[2] / "reference")))


def test_host_adamw_matches_torch_adamw():
    """msl_host_adamw (native, one pass) against torch.optim.AdamW, with clipping scale and the bf16
    staging copy written in the same pass."""
    torch.manual_seed(0)
    n = 100_003
    p0 = torch.randn(n)
    p_ref = torch.nn.Parameter(p0.clone())
    opt = torch.optim.AdamW([p_ref], lr=1e-3, betas=(0.9, 0.99), eps=1e-8, weight_decay=0.05)
    p = p0.clone()
    stage = torch.empty(n, dtype=torch.bfloat16)
    host = _HostAdamW(n, 1e-3, (0.9, 0.99), 1e-8, 0.05)
    for step in range(5):
        g = torch.randn(n)
        scale = 0.5 if step == 2 else 1.0
        p_ref.grad = g * scale
        opt.step()
        host.update(p, g.clone(), scale, stage=stage)
        assert torch.allclose(p, p_ref.detach(), rtol=1e-5, atol=1e-7), step
        assert torch.equal(stage, p.to(torch.bfloat16)), step


def test_host_accumulate_and_sum_of_squares():
    from megaslide_b200.stream import _accumulate

    torch.manual_seed(1)
    a = torch.randn(50_001).to(torch.bfloat16)
    b = torch.randn(50_001)
    dst = torch.full((50_001,), 7.0)
    sq = _accumulate(dst, a, overwrite=True)
    assert torch.equal(dst, a.float())
    assert abs(sq - float(a.double().square().sum())) <= 1e-9 * sq
    sq = _accumulate(dst, b, overwrite=False)
    assert torch.allclose(dst, a.float() + b)
    assert abs(sq - float(dst.double().square().sum())) <= 1e-9 * sq


def test_config_validation():
    with pytest.raises(ValueError):
        VideoDiTConfig(hidden_size=100, num_heads=3)
    with pytest.raises(ValueError):
        VideoDiTConfig(height=30, width=32, patch_size=4, hidden_size=64, num_heads=2)
    c = VideoDiTConfig(frames=4, height=16, width=16, patch_size=2, hidden_size=64, num_heads=2, num_layers=2)
    assert c.num_patches == 4 * 8 * 8 and c.mlp_hidden_size == 256 and c.head_dim == 32


@pytest.mark.skipif(not (REF / "infinity").exists(), reason="reference sources not mounted")
def test_dit_parameters_match_the_reference_model():
    sys.path.insert(0, str(REF))
    try:
        from infinity.video.config import MegaSlideConfig
        from infinity.video.model import MegaSlideDiT as RefDiT
    finally:
        sys.path.remove(str(REF))
    kw = dict(frames=4, height=16, width=16, patch_size=2, hidden_size=64, num_heads=2, num_layers=3,
              dsa_kernel_size=(3, 3, 3))
    for text in (False, True):
        ref = RefDiT(MegaSlideConfig(**kw, use_text_conditioning=text))
        ours = MegaSlideDiT(VideoDiTConfig(**kw, use_text_conditioning=text))
        a = {k: tuple(v.shape) for k, v in ref.state_dict().items()}
        b = {k: tuple(v.shape) for k, v in ours.state_dict().items()}
        assert a == b
        ours.load_state_dict(ref.state_dict())  # state dicts move between the two

"""MegaSlide-DiT model around the B200 attention: the caller that CPUMasterVideoDiT streams.

Same module tree, parameter names / shapes and initialisation as the reference's MegaSlideDiT
(infinity/video/model.py:21-264: MLP, DiTBlock with pre-norm 3D-DSA + optional text cross-attention +
MLP, spatial patchify, additive sinusoidal timestep embedding, unpatchify), so state dicts move
between the two.  The attention is megaslide_b200.DeformableSlideAttention3D; the other layers are
torch modules (cuBLAS GEMMs, torch LayerNorm / GELU).  `VideoDiTConfig` carries the fields of the
reference's MegaSlideConfig (infinity/video/config.py) that the model and the trainer read, with the
same names and defaults.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional, Tuple, Union

import torch
import torch.nn as nn
from torch import Tensor

from .attention import DeformableSlideAttention3D


@dataclass
class VideoDiTConfig:
    frames: int = 256
    in_channels: int = 4
    height: int = 1080
    width: int = 1920
    patch_size: int = 16
    hidden_size: int = 8192
    num_layers: int = 48
    num_heads: int = 64
    mlp_ratio: float = 4.0
    dsa_kernel_size: Tuple[int, int, int] = (3, 7, 7)
    offset_scale: float = 1.0
    dropout: float = 0.0
    use_text_conditioning: bool = False
    # trainer (CPU-master streaming)
    learning_rate: float = 1e-5
    weight_decay: float = 0.01
    max_grad_norm: float = 1.0
    checkpoint_interval: int = 4
    num_grad_slabs: int = 12
    beta1: float = 0.9
    beta2: float = 0.999
    eps: float = 1e-8
    dtype: str = "bfloat16"
    device: Union[int, str] = 0
    force_cpu: bool = False
    log_interval: int = 10
    resident_blocks: Optional[bool] = None  # CPU-master trainer: None = decide from device memory

    @property
    def num_patches(self) -> int:
        return self.frames * (self.height // self.patch_size) * (self.width // self.patch_size)

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_heads

    @property
    def mlp_hidden_size(self) -> int:
        return int(self.hidden_size * self.mlp_ratio)

    def __post_init__(self):
        if self.hidden_size % self.num_heads:
            raise ValueError(f"hidden_size ({self.hidden_size}) must be divisible by num_heads ({self.num_heads})")
        if self.height % self.patch_size or self.width % self.patch_size:
            raise ValueError("height and width must be divisible by patch_size")
        if len(self.dsa_kernel_size) != 3:
            raise ValueError("dsa_kernel_size must be a 3-tuple (k_t, k_h, k_w)")
        if self.checkpoint_interval <= 0:
            raise ValueError("checkpoint_interval must be positive")
        if self.num_grad_slabs < 2:
            raise ValueError("num_grad_slabs must be at least 2")


class MLP(nn.Module):
    def __init__(self, hidden_size: int, intermediate_size: int, dropout: float = 0.0):
        super().__init__()
        self.fc1 = nn.Linear(hidden_size, intermediate_size)
        self.act = nn.GELU()
        self.fc2 = nn.Linear(intermediate_size, hidden_size)
        self.dropout = nn.Dropout(dropout)

    def forward(self, x: Tensor) -> Tensor:
        return self.dropout(self.fc2(self.dropout(self.act(self.fc1(x)))))


class DiTBlock(nn.Module):
    """x + attn(norm1(x)) [+ cross_attn(norm_cross(x), text)] + mlp(norm2(.))  (model.py:40-117)."""

    def __init__(self, config: VideoDiTConfig):
        super().__init__()
        self.norm1 = nn.LayerNorm(config.hidden_size, eps=1e-6)
        self.attn = DeformableSlideAttention3D(config.hidden_size, config.num_heads, tuple(config.dsa_kernel_size),
                                               offset_scale=config.offset_scale, dropout=config.dropout)
        self.norm2 = nn.LayerNorm(config.hidden_size, eps=1e-6)
        self.mlp = MLP(config.hidden_size, config.mlp_hidden_size, config.dropout)
        if config.use_text_conditioning:
            self.norm_cross = nn.LayerNorm(config.hidden_size, eps=1e-6)
            self.cross_attn = nn.MultiheadAttention(config.hidden_size, config.num_heads, dropout=config.dropout,
                                                    batch_first=True)

    def forward(self, x: Tensor, video_shape: Tuple[int, int, int], text_embeds: Optional[Tensor] = None,
                text_mask: Optional[Tensor] = None) -> Tensor:
        x = x + self.attn(self.norm1(x), video_shape)
        if text_embeds is not None and hasattr(self, "cross_attn"):
            xn = self.norm_cross(x)
            out, _ = self.cross_attn(xn, text_embeds, text_embeds,
                                     key_padding_mask=~text_mask if text_mask is not None else None)
            x = x + out
        return x + self.mlp(self.norm2(x))


class MegaSlideDiT(nn.Module):
    """Video diffusion transformer predicting noise [B, C, T, H, W] (model.py:120-264)."""

    def __init__(self, config: VideoDiTConfig):
        super().__init__()
        self.config = config
        p = config.patch_size
        self.patch_embed = nn.Conv3d(config.in_channels, config.hidden_size, kernel_size=(1, p, p), stride=(1, p, p),
                                     padding=0, bias=True)
        self.pos_embed = nn.Parameter(torch.randn(1, config.num_patches, config.hidden_size) * 0.02)
        self.time_embed = nn.Sequential(nn.Linear(config.hidden_size, config.hidden_size * 4), nn.GELU(),
                                        nn.Linear(config.hidden_size * 4, config.hidden_size))
        self.blocks = nn.ModuleList([DiTBlock(config) for _ in range(config.num_layers)])
        self.norm_out = nn.LayerNorm(config.hidden_size, eps=1e-6)
        self.out_proj = nn.Linear(config.hidden_size, config.in_channels * p * p, bias=True)
        for m in self.modules():  # the reference's _init_weights (model.py:163-178)
            if isinstance(m, (nn.Linear, nn.Conv3d)):
                nn.init.xavier_uniform_(m.weight)
                if m.bias is not None:
                    nn.init.zeros_(m.bias)
        nn.init.normal_(self.pos_embed, std=0.02)

    def embed(self, latents: Tensor, timesteps: Tensor) -> Tuple[Tensor, Tuple[int, int, int]]:
        """patchify + positional + timestep embedding: [B, C, T, H, W] -> tokens [B, N, D]."""
        x = self.patch_embed(latents)
        _, D, T, Hp, Wp = x.shape
        x = x.flatten(2).transpose(1, 2) + self.pos_embed
        t = self.time_embed(self._get_timestep_embedding(timesteps.to(latents.device), D, latents.device).to(x.dtype))
        return x + t.unsqueeze(1), (T, Hp, Wp)

    def head(self, x: Tensor, shape: Tuple[int, ...]) -> Tensor:
        """norm_out + out_proj + unpatchify: tokens -> [B, C, T, H, W] (shape = latents.shape)."""
        B, C, T, H, W = shape
        p = self.config.patch_size
        x = self.out_proj(self.norm_out(x))
        x = x.view(B, T, H // p, W // p, C, p, p).permute(0, 4, 1, 2, 5, 3, 6).contiguous()
        return x.view(B, C, T, H, W)

    def forward(self, latents: Tensor, timesteps: Tensor, text_embeds: Optional[Tensor] = None,
                text_mask: Optional[Tensor] = None) -> Tensor:
        x, vshape = self.embed(latents, timesteps)
        for block in self.blocks:
            x = block(x, vshape, text_embeds, text_mask)
        return self.head(x, tuple(latents.shape))

    @staticmethod
    def _get_timestep_embedding(timesteps: Tensor, dim: int, device, max_period: int = 10000) -> Tensor:
        """Sinusoidal embedding [B, dim]: cos then sin of t * exp(-ln(max_period) k / half)."""
        half = dim // 2
        freqs = torch.exp(-math.log(max_period) * torch.arange(half, device=device, dtype=torch.float32) / half)
        args = timesteps[:, None].float() * freqs[None]
        emb = torch.cat([torch.cos(args), torch.sin(args)], dim=-1)
        if dim % 2 == 1:
            emb = torch.cat([emb, torch.zeros_like(emb[:, :1])], dim=-1)
        return emb

"""Drop-in ``DeformableSlideAttention3D`` running on the sm_100a kernels of libmegaslide_b200.so.

Same constructor arguments, forward signature, submodules, parameter names / shapes and default
initialisation order as the reference module ``infinity/video/attention.py:19-80`` of
jasonliu0704/megaslide, so ``MegaSlideDiT`` (model.py:55-61) and ``CPUMasterVideoDiT``
(trainer.py:158-174, 308, 397, 424-438) can use it unchanged and state dicts round-trip.

The forward is one ``torch.autograd.Function`` (so it works under ``no_grad``, ``autograd.grad`` and
per-parameter ``requires_grad`` toggling, as the trainer uses it):

  qkv  = x @ [Wq;Wk;Wv]^T + b                     cuBLAS GEMM (plain library GEMM)
  h    = GELU(dwconv3^3(x) + b1)                  msl_dwconv3d_fwd (epilogue GELU)
  off  = h @ W2^T + b2   (float32 out)            cuBLAS GEMM, bf16 in / fp32 out
  D    = dwconv_k(x) + bd + bo                    msl_dwconv3d_fwd (out_proj bias fused)
  a    = deformable gather attention(q, k, v, off, extra)   msl_dsa_attn_fwd
  y    = a @ Wo^T + D                             cuBLAS GEMM accumulating into D

and the backward mirrors it with msl_dsa_attn_bwd, msl_dwconv3d_bwd_data / _bwd_weight and the
GELU'-epilogue conv.  Activations compute in the input's dtype (float32 or bfloat16; under CUDA
autocast to bfloat16 the input is cast), every gather / softmax / stencil accumulates in float32.
There is no CPU path: CPU tensors raise.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.nn as nn
from torch import Tensor

from . import ops
from ._lib import MSL_EPI_GELU, MSL_EPI_GELU_GRAD, MSL_EPI_NONE, MSL_ERR_UNSUPPORTED, MslError


def _mm_f32(a: Tensor, b: Tensor) -> Tensor:
    """a @ b with a float32 result (bf16 operands accumulate in fp32 on the tensor cores)."""
    if a.dtype == torch.float32:
        return torch.mm(a, b)
    return torch.mm(a, b, out_dtype=torch.float32)


class _Cfg:
    __slots__ = ("shape", "conv_k", "conv_3", "dtype", "param_dtypes", "G", "kernel", "capture")

    def __init__(self, shape, conv_k, conv_3, dtype, param_dtypes, G, kernel, capture=None):
        self.shape = shape
        self.conv_k = conv_k
        self.conv_3 = conv_3
        self.dtype = dtype
        self.param_dtypes = param_dtypes
        self.G = G
        self.kernel = kernel
        self.capture = capture  # dict that receives the call's intermediates (parity checks), or None


class DSA3DFunction(torch.autograd.Function):
    """Forward/backward of DeformableSlideAttention3D (attention.py:82-192) on the B200 kernels."""

    @staticmethod
    def forward(ctx, cfg: _Cfg, x, extra_kv, off_in, wq, bq, wk, bk, wv, bv, wo, bo, wd, bd, w1, b1, w2, b2):
        sh: ops.DsaShape = cfg.shape
        dt = cfg.dtype
        B, N, C = x.shape
        G = cfg.G
        x2 = x.reshape(B * N, C).to(dt).contiguous()
        wqkv = torch.cat([wq, wk, wv], 0).to(dt)
        bqkv = torch.cat([bq, bk, bv], 0).to(dt)
        qkv = torch.addmm(bqkv, x2, wqkv.t())  # [BN, 3C]
        q, k, v = qkv[:, :C], qkv[:, C:2 * C], qkv[:, 2 * C:]
        O = w2.shape[0]
        w2m = w2.reshape(O, C)
        w1_kc = ops.conv_weight_kc(w1)
        b1f = b1.detach().float().contiguous()
        if off_in is None:
            # offset predictor: GELU(dw3^3(x) + b1) fused, then the 1x1 conv as a GEMM with fp32 output
            hact = ops.dwconv_fwd(cfg.conv_3, x2, w1_kc, b1f, epilogue=MSL_EPI_GELU)
            off = _mm_f32(hact, w2m.to(dt).t())  # its bias b2 is added by the attention kernels as they read it
            b2f = b2.detach().float().contiguous()
        else:
            # raw offsets given by the caller in place of the offset predictor's output (its bias included)
            hact = None
            off = off_in.reshape(B * N, O)
            b2f = None
        # depthwise conv term with both biases (dw_conv and out_proj) fused
        wd_kc = ops.conv_weight_kc(wd)
        D = ops.dwconv_fwd(cfg.conv_k, x2, wd_kc, bd.detach().float().contiguous(), bo.detach().float().contiguous(),
                           epilogue=MSL_EPI_NONE)
        ek = ev = e2 = None
        if G:
            e2 = extra_kv.reshape(B * G, C).to(dt).contiguous()
            ekv = torch.addmm(torch.cat([bk, bv], 0).to(dt), e2, torch.cat([wk, wv], 0).to(dt).t())
            ek, ev = ekv[:, :C], ekv[:, C:]
        train = any(ctx.needs_input_grad)
        sw = ops.status_word(x2.device)
        sw.poll()  # raises if an earlier call produced invalid results
        probs = saved = None
        if train and ops.wants_probs(sh, dt):
            # the tensor-core backward reads the forward's per-sample softmax weights and records
            probs, saved = ops.saved_buffers(sh, dt, x2.device)
            try:
                attn, lse = ops.attn_fwd(sh, q, k, v, off, ek, ev, probs=probs, saved=saved, offset_bias=b2f,
                                         status=sw.word)
            except MslError as e:
                if e.code != MSL_ERR_UNSUPPORTED:
                    raise
                probs = saved = None
        if probs is None:
            attn, lse = ops.attn_fwd(sh, q, k, v, off, ek, ev, offset_bias=b2f, status=sw.word)
        sw.post()
        y = D.addmm_(attn, wo.to(dt).t())  # in place: D is not used again
        if cfg.capture is not None:
            cfg.capture.update(x2=x2, qkv=qkv, hact=hact, off=off, offset_bias=b2f, attn=attn, lse=lse, y=y)
        if train:
            ctx.save_for_backward(x2, qkv, hact, off, b2f, attn, lse, e2, ek, ev, wqkv, wo, w2m, w1_kc, b1f, wd_kc, probs,
                                  saved)
            ctx.cfg = cfg
            ctx.in_dtype = x.dtype
            ctx.off_dtype = off_in.dtype if off_in is not None else None
            ctx.extra_dtype = extra_kv.dtype if extra_kv is not None else None
        return y.view(B, N, C)

    @staticmethod
    def backward(ctx, dy):
        (x2, qkv, hact, off, b2f, attn, lse, e2, ek, ev, wqkv, wo, w2m, w1_kc, b1f, wd_kc, probs,
         saved) = ctx.saved_tensors
        cfg: _Cfg = ctx.cfg
        sh: ops.DsaShape = cfg.shape
        dt = cfg.dtype
        BN, C = x2.shape
        B = sh.batch
        G = cfg.G
        with torch.autocast("cuda", enabled=False):
            dy2 = dy.reshape(BN, C).to(dt).contiguous()
            # out_proj
            dattn = torch.mm(dy2, wo.to(dt))
            g_wo = _mm_f32(dy2.t(), attn)
            g_bo = dy2.sum(0, dtype=torch.float32)
            g_wd = torch.zeros_like(wd_kc)
            g_bd = torch.zeros(C, device=dy2.device, dtype=torch.float32)
            ops.dwconv_bwd_weight(cfg.conv_k, dy2, x2, g_wd, g_bd)
            # deformable attention core -> dq, dk, dv written straight into one [BN, 3C] buffer
            dqkv = torch.empty_like(qkv)
            q, k, v = qkv[:, :C], qkv[:, C:2 * C], qkv[:, 2 * C:]
            sw = ops.status_word(dy2.device)
            _, _, _, doff, dek, dev = ops.attn_bwd(
                sh, q, k, v, off, attn, lse, dattn, ek=ek, ev=ev,
                dq=dqkv[:, :C], dk=dqkv[:, C:2 * C], dv=dqkv[:, 2 * C:], probs=probs, saved=saved, doff_dtype=dt,
                offset_bias=b2f, status=sw.word)
            sw.post()
            # q/k/v projections; dx accumulates in float32 across the three branches (the depthwise
            # convs add their transposed convolutions into it)
            dx = _mm_f32(dqkv, wqkv)
            ops.dwconv_bwd_data(cfg.conv_k, dy2, wd_kc, out=dx, accumulate=True)
            g_wqkv = _mm_f32(dqkv.t(), x2)
            g_bqkv = dqkv.sum(0, dtype=torch.float32)
            g_wq, g_wk, g_wv = g_wqkv[:C], g_wqkv[C:2 * C], g_wqkv[2 * C:]
            g_bq, g_bk, g_bv = g_bqkv[:C], g_bqkv[C:2 * C], g_bqkv[2 * C:]
            d_extra = None
            if G:
                dekv = torch.cat([dek, dev], 1)  # [BG, 2C] fp32
                wkv = wqkv[C:].float()
                d_extra = torch.mm(dekv, wkv).view(B, G, C)
                g_ekv = torch.mm(dekv.t(), e2.float())
                g_wk = g_wk + g_ekv[:C]
                g_wv = g_wv + g_ekv[C:]
                sums = dekv.sum(0)
                g_bk = g_bk + sums[:C]
                g_bv = g_bv + sums[C:]
            if cfg.capture is not None:
                cfg.capture.update(dy2=dy2, dattn=dattn, dqkv=dqkv, doff=doff, dx=dx)
            d_off_in = None
            if hact is not None:
                # offset predictor (the kernel wrote doff in the compute dtype, the GEMMs' operand type); dh
                # and du stay float32 (bf16 operands, fp32 results)
                dh = _mm_f32(doff, w2m.to(dt))
                g_w2 = _mm_f32(doff.t(), hact)
                g_b2 = doff.sum(0, dtype=torch.float32)
                du = ops.dwconv_fwd(cfg.conv_3, x2, w1_kc, b1f, epilogue=MSL_EPI_GELU_GRAD, aux=dh,
                                    out_dtype=torch.float32)
                ops.dwconv_bwd_data(cfg.conv_3, du, w1_kc, out=dx, accumulate=True)
                g_w1 = torch.zeros_like(w1_kc)
                g_b1 = torch.zeros(C, device=dy2.device, dtype=torch.float32)
                ops.dwconv_bwd_weight(cfg.conv_3, du, x2, g_w1, g_b1)
            elif ctx.needs_input_grad[3]:
                d_off_in = doff.view(B, BN // B, -1).to(ctx.off_dtype)

        pd = cfg.param_dtypes
        kt, kh, kw = cfg.kernel

        def conv_w(gkc, k3):
            return gkc.t().reshape(C, 1, *k3)

        grads = (
            g_wq.to(pd[0]), g_bq.to(pd[1]), g_wk.to(pd[2]), g_bk.to(pd[3]), g_wv.to(pd[4]), g_bv.to(pd[5]),
            g_wo.to(pd[6]), g_bo.to(pd[7]), conv_w(g_wd, (kt, kh, kw)).to(pd[8]), g_bd.to(pd[9]),
        )
        if hact is not None:
            grads += (conv_w(g_w1, (3, 3, 3)).to(pd[10]), g_b1.to(pd[11]),
                      g_w2.reshape(w2m.shape[0], C, 1, 1, 1).to(pd[12]), g_b2.to(pd[13]))
        else:  # the offset predictor did not run: no gradient for its parameters
            grads += (None, None, None, None)
        dx_out = dx.view(B, BN // B, C).to(ctx.in_dtype)
        de = d_extra.to(ctx.extra_dtype) if d_extra is not None else None
        return (None, dx_out, de, d_off_in) + grads


class DeformableSlideAttention3D(nn.Module):
    """3D Deformable Slide Attention (3D-DSA) on B200 kernels.

    Args (as the reference, attention.py:26-41):
        hidden_size: hidden dimension D.
        num_heads: number of attention heads.
        kernel_size: (k_t, k_h, k_w) local neighbourhood; odd sizes (padding k//2 keeps the
            volume only for odd k — the reference's dw term fails to reshape otherwise).
        offset_scale: scale of the learned offsets.
        dropout: dropout on the softmax weights (counter-based in-kernel mask in training mode).

    ``capture`` (not a parameter; None by default): a dict set here receives references to the
    intermediates of the next forward / backward (q/k/v, offsets, attention output, lse and their
    gradients), which a checker compares with an independent implementation at sampled rows.
    """

    def __init__(self, hidden_size: int, num_heads: int, kernel_size: Tuple[int, int, int] = (3, 7, 7),
                 offset_scale: float = 1.0, dropout: float = 0.0):
        super().__init__()
        assert hidden_size % num_heads == 0, "hidden_size must be divisible by num_heads"
        self.hidden_size = hidden_size
        self.num_heads = num_heads
        self.head_dim = hidden_size // num_heads
        self.k_t, self.k_h, self.k_w = kernel_size
        self.offset_scale = offset_scale
        # same modules, names and construction order as the reference (attention.py:52-80), so a
        # given torch seed initialises both identically
        self.q_proj = nn.Linear(hidden_size, hidden_size, bias=True)
        self.k_proj = nn.Linear(hidden_size, hidden_size, bias=True)
        self.v_proj = nn.Linear(hidden_size, hidden_size, bias=True)
        self.out_proj = nn.Linear(hidden_size, hidden_size, bias=True)
        self.dw_conv = nn.Conv3d(hidden_size, hidden_size, kernel_size=kernel_size,
                                 padding=(self.k_t // 2, self.k_h // 2, self.k_w // 2), groups=hidden_size, bias=True)
        num_offsets = num_heads * self.k_t * self.k_h * self.k_w * 3
        self.offset_net = nn.Sequential(
            nn.Conv3d(hidden_size, hidden_size, 3, padding=1, groups=hidden_size),
            nn.GELU(),
            nn.Conv3d(hidden_size, num_offsets, 1, bias=True),
        )
        nn.init.zeros_(self.offset_net[-1].weight)
        nn.init.zeros_(self.offset_net[-1].bias)
        self.dropout = nn.Dropout(dropout)
        self.capture: Optional[dict] = None

    def _params(self):
        return (self.q_proj.weight, self.q_proj.bias, self.k_proj.weight, self.k_proj.bias,
                self.v_proj.weight, self.v_proj.bias, self.out_proj.weight, self.out_proj.bias,
                self.dw_conv.weight, self.dw_conv.bias, self.offset_net[0].weight, self.offset_net[0].bias,
                self.offset_net[2].weight, self.offset_net[2].bias)

    def forward(self, x: Tensor, video_shape: Tuple[int, int, int], extra_kv: Optional[Tensor] = None) -> Tensor:
        """x: [B, N, D] tokens (N = T*H*W); video_shape: (T, H, W); extra_kv: optional [B, G, D]
        appended to every neighbourhood.  Returns [B, N, D]."""
        return self._run(x, video_shape, extra_kv, None)

    def forward_with_offsets(self, x: Tensor, video_shape: Tuple[int, int, int], offsets: Tensor,
                             extra_kv: Optional[Tensor] = None) -> Tensor:
        """The forward with the offset predictor replaced by given raw offsets (float32 [B, N, nh*K*3]
        in the 1x1 conv's channel order, i.e. what offset_net(x) computes at attention.py:105-106,
        bias included; offset_scale still applies).  Used to drive the op with synthetic offsets of a
        chosen distribution; gradients flow to x, the projection / dw_conv parameters and `offsets`
        (the offset_net parameters get none)."""
        if offsets.dtype != torch.float32:
            raise TypeError("offsets must be float32")
        B, N = x.shape[:2]
        want = (B, N, self.num_heads * self.k_t * self.k_h * self.k_w * 3)
        if tuple(offsets.shape) != want:
            raise ValueError(f"offsets must have shape {want}, got {tuple(offsets.shape)}")
        if not offsets.is_cuda or offsets.device != x.device:
            raise RuntimeError("offsets must be on x's CUDA device")
        return self._run(x, video_shape, extra_kv, offsets.contiguous())

    def _run(self, x: Tensor, video_shape: Tuple[int, int, int], extra_kv: Optional[Tensor],
             offsets: Optional[Tensor]) -> Tensor:
        B, N, D = x.shape
        T, H, W = video_shape
        assert N == T * H * W, f"Expected N={T * H * W} but got {N}"
        assert D == self.hidden_size
        if not x.is_cuda:
            raise RuntimeError("megaslide_b200.DeformableSlideAttention3D runs on CUDA tensors only "
                               "(the B200 kernels have no CPU fallback)")
        if self.k_t % 2 == 0 or self.k_h % 2 == 0 or self.k_w % 2 == 0:
            raise RuntimeError(f"kernel_size {(self.k_t, self.k_h, self.k_w)} must be odd")
        dt = x.dtype
        if torch.is_autocast_enabled("cuda"):
            ad = torch.get_autocast_dtype("cuda")
            if ad == torch.bfloat16:
                dt = torch.bfloat16
        if dt not in (torch.float32, torch.bfloat16):
            raise TypeError(f"megaslide_b200 supports float32 and bfloat16, got {dt}")
        G = 0
        if extra_kv is not None:
            if extra_kv.shape[0] != B or extra_kv.shape[2] != D:
                raise ValueError(f"extra_kv must be [B, G, D] = [{B}, G, {D}], got {tuple(extra_kv.shape)}")
            G = extra_kv.shape[1]
            if not extra_kv.is_cuda or extra_kv.device != x.device:
                raise RuntimeError("extra_kv must be on the same CUDA device as x")
        p = self.dropout.p if self.training else 0.0
        seed = int(torch.randint(0, 2 ** 62, (1,)).item()) if p > 0 else 0
        shape = ops.DsaShape(B, T, H, W, self.num_heads, self.head_dim, (self.k_t, self.k_h, self.k_w), extra=G,
                             offset_scale=float(self.offset_scale), dropout_p=float(p), dropout_seed=seed)
        cfg = _Cfg(shape,
                   ops.ConvShape(B, T, H, W, D, (self.k_t, self.k_h, self.k_w)),
                   ops.ConvShape(B, T, H, W, D, (3, 3, 3)),
                   dt, tuple(t.dtype for t in self._params()), G, (self.k_t, self.k_h, self.k_w),
                   capture=self.capture)
        with torch.autocast("cuda", enabled=False):
            return DSA3DFunction.apply(cfg, x, extra_kv, offsets, *self._params())

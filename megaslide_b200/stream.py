"""CPU-master training of MegaSlide-DiT with the transformer blocks streamed through two GPU slots.

Same interface as the reference's CPUMasterVideoDiT (infinity/video/trainer.py:23-650:
`forward_and_backward(latents, timesteps, target_noise, text_embeds=None, text_mask=None) ->
(loss, timings)`, `optimizer_step() -> grad norm`, `zero_grad()`, `get_parameters()`, `cleanup()`,
`save_checkpoint(path)`, `load_checkpoint(path)`), same schedule (no-grad forward through the blocks
with an activation checkpoint every `checkpoint_interval` blocks; per checkpoint segment in reverse,
recompute then `autograd.grad` block by block; head and embeddings resident on the GPU), re-built
around the copies:

* every block's fp32 master weights live in ONE flat pinned host buffer (the CPU block's parameters
  are views into it), next to a pinned compute-dtype (bf16) staging copy; a block moves to the GPU
  with a single cudaMemcpyAsync from pinned memory (the reference copies parameter by parameter from
  pageable memory, fp32);
* the two GPU slots are flat device buffers; the slot's block module has its parameters viewing the
  buffer.  Block l+1 is copied on a side stream while block l computes; before overwriting a slot
  the copy waits for the event the compute stream records when it is done with the slot (the
  reference records such events but never waits on them);
* a slot keeps the block it holds: the recompute / backward of a segment reuses a block still
  resident instead of copying it again;
* a block's parameter gradients are packed into one flat device buffer and returned with one D2H
  copy into a pinned slab; a host thread accumulates them into the block's flat fp32 gradient
  buffer while the GPU works on the next blocks;
* optimizer_step() computes the global gradient norm (clipping as the reference), then a host
  thread runs AdamW on each block's flat fp32 buffers and refreshes its bf16 staging copy, block 0
  first; the next forward copies block i as soon as block i is updated, so the host AdamW overlaps
  the next step's GPU work.  Head / embedding parameters (GPU-resident) use torch's AdamW on the GPU.

Resident mode (chosen when every block's bf16 weights and autograd activations fit in 60% of the
free HBM -- config 3 on a 180 GB B200 -- or forced with config.resident_blocks): each block keeps its
own device weight buffer, refreshed by one H2D copy after its host update, and the step is one
forward with autograd plus one backward (no recompute).  The streaming mode above is the one for
models whose weights do not fit.

The optimizer state is per block (flat buffers), so optimizer checkpoints are not interchangeable
with the reference's torch.optim state dict; model state dicts are.
"""

from __future__ import annotations

import copy
import ctypes
import math
import queue
import threading
import time
from typing import Dict, List, Optional, Tuple

import torch
import torch.nn as nn
from torch import Tensor

from . import _lib


def _flat_params(module: nn.Module) -> List[nn.Parameter]:
    return [p for _, p in module.named_parameters()]


class _HostAdamW:
    """AdamW state of one flat float32 buffer; the update is msl_host_adamw (one multi-threaded pass
    over parameters, moments and gradient that also writes the compute-dtype staging copy)."""

    def __init__(self, numel: int, lr: float, betas: Tuple[float, float], eps: float, weight_decay: float):
        self.m = torch.zeros(numel, dtype=torch.float32)
        self.v = torch.zeros(numel, dtype=torch.float32)
        self.step = 0
        self.lr, self.betas, self.eps, self.wd = lr, betas, eps, weight_decay

    def update(self, p: Tensor, g: Tensor, scale: float, stage: Optional[Tensor] = None) -> None:
        for t in (p, g, self.m, self.v):
            if t.dtype != torch.float32 or not t.is_contiguous() or t.device.type != "cpu":
                raise TypeError("host AdamW buffers must be contiguous float32 host tensors")
        sdt = 0
        if stage is not None:
            sdt = {torch.float32: _lib.MSL_DTYPE_F32, torch.bfloat16: _lib.MSL_DTYPE_BF16}[stage.dtype]
        self.step += 1
        _lib.check("msl_host_adamw", _lib.load().msl_host_adamw(
            p.data_ptr(), self.m.data_ptr(), self.v.data_ptr(), g.data_ptr(), p.numel(), self.lr, self.betas[0],
            self.betas[1], self.eps, self.wd, self.step, scale, stage.data_ptr() if stage is not None else None, sdt))

    def state_dict(self):
        return {"m": self.m, "v": self.v, "step": self.step}

    def load_state_dict(self, d):
        self.m.copy_(d["m"])
        self.v.copy_(d["v"])
        self.step = int(d["step"])


def _accumulate(dst: Tensor, src: Tensor, overwrite: bool) -> float:
    """dst (float32) = [dst +] src (float32 or bf16) on the host; returns sum(dst^2)."""
    sq = ctypes.c_double(0.0)
    code = {torch.float32: _lib.MSL_DTYPE_F32, torch.bfloat16: _lib.MSL_DTYPE_BF16}[src.dtype]
    _lib.check("msl_host_accumulate", _lib.load().msl_host_accumulate(
        dst.data_ptr(), src.data_ptr(), code, dst.numel(), 1 if overwrite else 0, ctypes.byref(sq)))
    return float(sq.value)


class CPUMasterVideoDiT:
    """CPU-master trainer for a MegaSlideDiT (megaslide_b200.dit or the reference's model built with
    megaslide_b200.DeformableSlideAttention3D): fp32 master weights and AdamW on the host, blocks
    streamed through two GPU slots."""

    def __init__(self, model: nn.Module, config, force_cpu: bool = False):
        self.model = model
        self.config = config
        self.force_cpu = force_cpu
        self.use_cuda = torch.cuda.is_available() and not force_cpu and not getattr(config, "force_cpu", False)
        if not self.use_cuda:
            raise RuntimeError("megaslide_b200.CPUMasterVideoDiT streams to a CUDA device (no CPU mode); "
                               "the reference's CPU-only mode stays the reference's")
        dev = config.device
        self.device = torch.device(f"cuda:{dev}" if isinstance(dev, int) or str(dev).isdigit() else dev)
        self.cdtype = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}[config.dtype]
        self.step_count = 0
        self.h2d_bytes = 0  # block weights copied to the GPU (counters for measurement)
        self.d2h_bytes = 0  # block gradients copied back
        self.model.to("cpu").float()
        self.blocks = self.model.blocks
        self.num_blocks = len(self.blocks)
        self._setup_host_buffers()
        self._setup_gpu()
        self.resident: Optional[bool] = None  # decided at the first step (needs the token count)
        # a list set here receives (kind, block, stream, start event, end event) for every weight copy
        # ("h2d"), block forward / recompute / backward ("fwd", "recompute", "bwd") and gradient copy
        # ("d2h") of the next steps: the streaming timeline (timeline_summary)
        self.timeline: Optional[list] = None
        self._worker_q: "queue.Queue" = queue.Queue()
        self._worker_err: List[BaseException] = []
        self._worker = threading.Thread(target=self._work_loop, daemon=True)
        self._worker.start()

    # ------------------------------------------------------------------ set-up
    def _setup_host_buffers(self):
        cfg = self.config
        self.block_numel = [sum(p.numel() for p in _flat_params(b)) for b in self.blocks]
        self.master: List[Tensor] = []
        self.stage: List[Tensor] = []
        self.hgrad: List[Tensor] = []
        self.opt: List[_HostAdamW] = []
        self.stage_ready = [threading.Event() for _ in range(self.num_blocks)]
        for i, b in enumerate(self.blocks):
            n = self.block_numel[i]
            flat = torch.empty(n, dtype=torch.float32, pin_memory=True)
            off = 0
            for p in _flat_params(b):
                k = p.numel()
                flat[off:off + k].copy_(p.data.reshape(-1))
                p.data = flat[off:off + k].view(p.shape)  # the CPU block now views the master buffer
                off += k
            self.master.append(flat)
            st = torch.empty(n, dtype=self.cdtype, pin_memory=True)
            st.copy_(flat)
            self.stage.append(st)
            self.hgrad.append(torch.zeros(n, dtype=torch.float32))
            self.opt.append(_HostAdamW(n, cfg.learning_rate, (cfg.beta1, cfg.beta2), cfg.eps, cfg.weight_decay))
            self.stage_ready[i].set()
        self.has_grad = [False] * self.num_blocks
        self.sumsq = [0.0] * self.num_blocks  # sum of squares of each block's gradient

    def _setup_gpu(self):
        cfg = self.config
        dev = self.device
        self.compute_stream = torch.cuda.current_stream(dev)
        self.weight_stream = torch.cuda.Stream(device=dev)
        self.grad_stream = torch.cuda.Stream(device=dev)
        nmax = max(self.block_numel)
        self.slot_buf = [torch.empty(nmax, dtype=self.cdtype, device=dev) for _ in range(2)]
        self.slot_block = [-1, -1]  # block held by each slot
        self._last_slot = 1
        self.slot_ready = [torch.cuda.Event() for _ in range(2)]
        self.slot_free = [torch.cuda.Event() for _ in range(2)]
        for e in self.slot_free:
            e.record(self.compute_stream)
        self.gpu_blocks = []
        for s in range(2):
            gb = copy.deepcopy(self.blocks[0]).to(dev, self.cdtype)
            off = 0
            for p in _flat_params(gb):
                k = p.numel()
                p.data = self.slot_buf[s][off:off + k].view(p.shape)
                p.requires_grad_(False)
                off += k
            self.gpu_blocks.append(gb)
        self.gflat = torch.empty(nmax, dtype=self.cdtype, device=dev)
        self.slabs = [torch.empty(nmax, dtype=self.cdtype, pin_memory=True) for _ in range(max(2, cfg.num_grad_slabs))]
        self.slab_free: "queue.Queue" = queue.Queue()
        for i in range(len(self.slabs)):
            self.slab_free.put(i)
        self.slab_done = [torch.cuda.Event() for _ in self.slabs]
        self.gflat_free = torch.cuda.Event()
        self.gflat_free.record(self.compute_stream)
        # resident head / tail (fp32 master on the GPU, torch AdamW there)
        m = self.model
        self.resident = [m.patch_embed, m.time_embed, m.norm_out, m.out_proj]
        for mod in self.resident:
            mod.to(dev)
        m.pos_embed.data = m.pos_embed.data.to(dev)
        self.res_params = [p for mod in self.resident for p in mod.parameters()] + [m.pos_embed]
        self.gpu_opt = torch.optim.AdamW(self.res_params, lr=cfg.learning_rate, betas=(cfg.beta1, cfg.beta2),
                                         eps=cfg.eps, weight_decay=cfg.weight_decay)

    # ------------------------------------------------------------------ resident mode
    def _decide_resident(self, tokens: int) -> bool:
        """Resident mode when every block's compute-dtype weights and autograd activations fit in 60%
        of the free device memory (B200: 180 GB); the estimate per block and token is the hidden state
        in ~24 copies (projections, norms, MLP) plus the attention's float32 offsets and softmax weights.
        config.resident_blocks (True / False) overrides."""
        forced = getattr(self.config, "resident_blocks", None)
        if forced is not None:
            return bool(forced)
        cfg = self.config
        es = torch.tensor([], dtype=self.cdtype).element_size()
        K = cfg.dsa_kernel_size[0] * cfg.dsa_kernel_size[1] * cfg.dsa_kernel_size[2]
        weights = sum(self.block_numel) * es
        acts = tokens * (cfg.hidden_size * es * 24 + cfg.num_heads * K * 16) * self.num_blocks
        free, _ = torch.cuda.mem_get_info(self.device)
        return weights + acts <= 0.6 * free

    def _setup_resident(self):
        dev = self.device
        self.res_buf = [torch.empty(n, dtype=self.cdtype, device=dev) for n in self.block_numel]
        self.res_blocks = []
        for i, b in enumerate(self.blocks):
            gb = copy.deepcopy(b).to(dev, self.cdtype)
            off = 0
            for p in _flat_params(gb):
                k = p.numel()
                p.data = self.res_buf[i][off:off + k].view(p.shape)
                p.requires_grad_(False)
                off += k
            self.res_blocks.append(gb)
        self.res_dirty = [True] * self.num_blocks
        self.res_ready = [torch.cuda.Event() for _ in range(self.num_blocks)]

    def _upload(self, i: int) -> None:
        """Copies block i's updated staging weights to its resident buffer (side stream)."""
        if not self.res_dirty[i]:
            return
        if not self.stage_ready[i].wait(timeout=600.0):
            raise RuntimeError(f"block {i}: host optimizer update did not finish")
        with torch.cuda.stream(self.weight_stream):
            ev = self._mark(self.weight_stream)
            self.res_buf[i].copy_(self.stage[i], non_blocking=True)
            self.res_ready[i].record(self.weight_stream)
            self._mark_end("h2d", i, "weight", self.weight_stream, ev)
        self.res_dirty[i] = False
        self.h2d_bytes += self.block_numel[i] * self.stage[i].element_size()

    def _blocks_resident(self, x: Tensor, vshape, te, tm, head_fn) -> Tuple[Tensor, Tensor, Tensor]:
        """One forward with autograd through all blocks (graphs kept), the head, then one backward
        block by block; returns (loss, gradient w.r.t. the block input, the fwd-end event)."""
        saved = []
        for i in range(self.num_blocks):
            self._upload(i)
            if i + 1 < self.num_blocks:
                self._upload(i + 1)
            self.compute_stream.wait_event(self.res_ready[i])
            blk = self.res_blocks[i]
            for p in _flat_params(blk):
                p.requires_grad_(True)
            inp = x.detach().requires_grad_(True)
            ev = self._mark(self.compute_stream)
            out = blk(inp, vshape, te, tm)
            self._mark_end("fwd", i, "compute", self.compute_stream, ev)
            saved.append((inp, out))
            x = out.detach()
        loss, grad_hidden, fwd_end = head_fn(x)
        for i in range(self.num_blocks - 1, -1, -1):
            inp, out = saved[i]
            params = _flat_params(self.res_blocks[i])
            ev = self._mark(self.compute_stream)
            grads = torch.autograd.grad(out, (inp, *params), grad_outputs=grad_hidden, allow_unused=True)
            self._mark_end("bwd", i, "compute", self.compute_stream, ev)
            for p in params:
                p.requires_grad_(False)
            grad_hidden = grads[0].detach()
            self._return_grads(i, params, grads[1:])
            saved[i] = None
            del inp, out
        return loss, grad_hidden, fwd_end

    # ------------------------------------------------------------------ host worker
    def _work_loop(self):
        while True:
            task = self._worker_q.get()
            if task is None:
                return
            try:
                task()
            except BaseException as e:  # surfaced by the next synchronising call
                self._worker_err.append(e)

    def _worker_flush(self):
        done = threading.Event()
        self._worker_q.put(done.set)
        done.wait()
        if self._worker_err:
            raise RuntimeError("host worker failed") from self._worker_err[0]

    # ------------------------------------------------------------------ streaming
    def _load(self, i: int) -> int:
        """Slot holding block i, copying it in (side stream) if no slot has it; returns the slot."""
        for s in range(2):
            if self.slot_block[s] == i:
                return s
        s = 0 if self.slot_block[0] == -1 else (1 if self.slot_block[1] == -1 else None)
        if s is None:  # the slot not used by the block computed last
            s = 1 if self._last_slot == 0 else 0
        if not self.stage_ready[i].wait(timeout=600.0):
            raise RuntimeError(f"block {i}: host optimizer update did not finish")
        n = self.block_numel[i]
        with torch.cuda.stream(self.weight_stream):
            self.weight_stream.wait_event(self.slot_free[s])
            ev = self._mark(self.weight_stream)
            self.slot_buf[s][:n].copy_(self.stage[i], non_blocking=True)
            self.slot_ready[s].record(self.weight_stream)
            self._mark_end("h2d", i, "weight", self.weight_stream, ev)
        self.slot_block[s] = i
        self.h2d_bytes += n * self.stage[i].element_size()
        return s

    def _mark(self, stream) -> Optional[torch.cuda.Event]:
        if self.timeline is None:
            return None
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(stream)
        return ev

    def _mark_end(self, kind: str, block: int, sname: str, stream, start: Optional[torch.cuda.Event]) -> None:
        if self.timeline is not None and start is not None:
            end = torch.cuda.Event(enable_timing=True)
            end.record(stream)
            self.timeline.append((kind, block, sname, start, end))

    def _run(self, i: int, x: Tensor, vshape, text_embeds, text_mask, prefetch: Optional[int] = None,
             kind: str = "fwd"):
        s = self._load(i)
        self._last_slot = s
        if prefetch is not None and 0 <= prefetch < self.num_blocks:
            self._load(prefetch)
        self.compute_stream.wait_event(self.slot_ready[s])
        ev = self._mark(self.compute_stream)
        y = self.gpu_blocks[s](x, vshape, text_embeds, text_mask)
        self._mark_end(kind, i, "compute", self.compute_stream, ev)
        self.slot_free[s].record(self.compute_stream)
        return y

    def _return_grads(self, i: int, params, grads) -> None:
        """Packs block i's parameter gradients into one buffer and queues one D2H copy and the host
        accumulation."""
        n = self.block_numel[i]
        slab_i = self.slab_free.get(timeout=600.0)
        self.compute_stream.wait_event(self.gflat_free)
        off = 0
        for p, g in zip(params, grads):
            k = p.numel()
            if g is None:
                self.gflat[off:off + k].zero_()
            else:
                self.gflat[off:off + k].copy_(g.reshape(-1))
            off += k
        packed = torch.cuda.Event()
        packed.record(self.compute_stream)
        self.d2h_bytes += n * self.gflat.element_size()
        with torch.cuda.stream(self.grad_stream):
            self.grad_stream.wait_event(packed)
            ev = self._mark(self.grad_stream)
            self.slabs[slab_i][:n].copy_(self.gflat[:n], non_blocking=True)
            self.slab_done[slab_i].record(self.grad_stream)
            self.gflat_free.record(self.grad_stream)
            self._mark_end("d2h", i, "grad", self.grad_stream, ev)

        def accumulate(i=i, slab_i=slab_i, n=n):
            self.slab_done[slab_i].synchronize()
            self.sumsq[i] = _accumulate(self.hgrad[i], self.slabs[slab_i][:n], overwrite=not self.has_grad[i])
            self.has_grad[i] = True
            self.slab_free.put(slab_i)

        self._worker_q.put(accumulate)

    # ------------------------------------------------------------------ training step
    def forward_and_backward(self, latents: Tensor, timesteps: Tensor, target_noise: Tensor,
                             text_embeds: Optional[Tensor] = None,
                             text_mask: Optional[Tensor] = None) -> Tuple[float, Dict[str, float]]:
        cfg = self.config
        dev = self.device
        m = self.model
        start, fwd_end, bwd_end = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        start.record(self.compute_stream)
        lat = latents.to(dev, non_blocking=True)
        tgt = target_noise.to(dev, non_blocking=True)
        ts = timesteps.to(dev, non_blocking=True)
        te = text_embeds.to(dev, self.cdtype) if text_embeds is not None else None
        tm = text_mask.to(dev) if text_mask is not None else None
        self._last_slot = 1
        # forward: embeddings (resident, recorded for their backward), blocks without autograd
        with torch.autocast("cuda", dtype=self.cdtype, enabled=self.cdtype != torch.float32):
            x0, vshape = m.embed(lat, ts)
        x0 = x0.to(self.cdtype)
        if self.resident is None:
            self.resident = self._decide_resident(x0.shape[0] * x0.shape[1])
            if self.resident:
                self._setup_resident()
        if self.resident:

            def head_fn(xb):
                hidden = xb.detach().requires_grad_(True)
                with torch.autocast("cuda", dtype=self.cdtype, enabled=self.cdtype != torch.float32):
                    pred = m.head(hidden, tuple(lat.shape))
                loss_ = nn.functional.mse_loss(pred.float(), tgt.float())
                fwd_end.record(self.compute_stream)
                loss_.backward()
                return loss_, hidden.grad.detach().to(self.cdtype), fwd_end

            loss, grad_hidden, _ = self._blocks_resident(x0.detach(), vshape, te, tm, head_fn)
            x0.backward(grad_hidden.to(x0.dtype))
            bwd_end.record(self.compute_stream)
            bwd_end.synchronize()
            self._worker_flush()
            return float(loss.item()), {"forward": start.elapsed_time(fwd_end) / 1e3,
                                        "backward": fwd_end.elapsed_time(bwd_end) / 1e3,
                                        "total": start.elapsed_time(bwd_end) / 1e3}
        ckpt: Dict[int, Tensor] = {}
        x = x0.detach()
        with torch.no_grad():
            for i in range(self.num_blocks):
                if i % cfg.checkpoint_interval == 0:
                    ckpt[i] = x
                x = self._run(i, x, vshape, te, tm, prefetch=i + 1)
        # head and loss (resident parameters, autograd)
        hidden = x.detach().requires_grad_(True)
        with torch.autocast("cuda", dtype=self.cdtype, enabled=self.cdtype != torch.float32):
            pred = m.head(hidden, tuple(lat.shape))
        loss = nn.functional.mse_loss(pred.float(), tgt.float())
        fwd_end.record(self.compute_stream)
        loss.backward()
        grad_hidden = hidden.grad.detach().to(self.cdtype)
        # backward through the blocks, one checkpoint segment at a time (last first)
        nseg = (self.num_blocks + cfg.checkpoint_interval - 1) // cfg.checkpoint_interval
        for seg in range(nseg - 1, -1, -1):
            b0 = seg * cfg.checkpoint_interval
            b1 = min(b0 + cfg.checkpoint_interval, self.num_blocks)
            inputs = {b0: ckpt[b0]}
            with torch.no_grad():
                h = ckpt[b0]
                for j in range(b0, b1 - 1):
                    h = self._run(j, h, vshape, te, tm, prefetch=j + 1, kind="recompute")
                    inputs[j + 1] = h
            for i in range(b1 - 1, b0 - 1, -1):
                s = self._load(i)
                self._last_slot = s
                # prefetch the block needed next: the previous one of this segment, or the first
                # block of the previous segment (its recompute comes next)
                nxt = i - 1 if i > b0 else (b0 - cfg.checkpoint_interval if seg > 0 else None)
                if nxt is not None:
                    self._load(nxt)
                self.compute_stream.wait_event(self.slot_ready[s])
                gb = self.gpu_blocks[s]
                params = _flat_params(gb)
                for p in params:
                    p.requires_grad_(True)
                inp = inputs[i].detach().requires_grad_(True)
                ev = self._mark(self.compute_stream)
                out = gb(inp, vshape, te, tm)
                grads = torch.autograd.grad(out, (inp, *params), grad_outputs=grad_hidden, allow_unused=True)
                self._mark_end("bwd", i, "compute", self.compute_stream, ev)
                for p in params:
                    p.requires_grad_(False)
                grad_hidden = grads[0].detach()
                self._return_grads(i, params, grads[1:])
                self.slot_free[s].record(self.compute_stream)
                del out, inp
        # embeddings
        x0.backward(grad_hidden.to(x0.dtype))
        bwd_end.record(self.compute_stream)
        bwd_end.synchronize()
        self._worker_flush()
        loss_val = float(loss.item())
        return loss_val, {"forward": start.elapsed_time(fwd_end) / 1e3,
                          "backward": fwd_end.elapsed_time(bwd_end) / 1e3,
                          "total": start.elapsed_time(bwd_end) / 1e3}

    def optimizer_step(self) -> float:
        """Clips by the global gradient norm (as the reference) and applies AdamW: resident
        parameters on the GPU now, block masters on the host in the background (block 0 first; the
        next forward copies a block as soon as it is updated).  Returns the norm before clipping."""
        self._worker_flush()
        cfg = self.config
        sq = sum(self.sumsq[i] for i in range(self.num_blocks) if self.has_grad[i])
        res_grads = [p.grad for p in self.res_params if p.grad is not None]
        if res_grads:
            sq += float(torch.stack([g.float().square().sum() for g in res_grads]).sum())
        norm = math.sqrt(sq)
        scale = 1.0
        if cfg.max_grad_norm > 0 and norm > cfg.max_grad_norm:
            scale = cfg.max_grad_norm / (norm + 1e-6)
        if res_grads:
            if scale != 1.0:
                for g in res_grads:
                    g.mul_(scale)
            self.gpu_opt.step()
        for i in range(self.num_blocks):
            if not self.has_grad[i]:
                continue
            self.stage_ready[i].clear()

            def upd(i=i):
                try:
                    self.opt[i].update(self.master[i], self.hgrad[i], scale, stage=self.stage[i])
                finally:
                    self.stage_ready[i].set()

            self._worker_q.put(upd)
        # the slots / resident buffers hold pre-update weights: force fresh copies
        self.slot_block = [-1, -1]
        if self.resident:
            self.res_dirty = [True] * self.num_blocks
        self.step_count += 1
        if cfg.log_interval and self.step_count % cfg.log_interval == 0:
            print(f"  [Step {self.step_count}] Gradient norm: {norm:.4f}")
        return norm

    def zero_grad(self):
        self._worker_flush()
        for i in range(self.num_blocks):
            self.has_grad[i] = False
        self.gpu_opt.zero_grad(set_to_none=True)

    def get_parameters(self):
        self._worker_flush()
        return list(self.model.parameters())

    def cleanup(self):
        if self._worker.is_alive():
            self._worker_q.put(None)
            self._worker.join(timeout=30.0)

    def save_checkpoint(self, path: str):
        self._worker_flush()
        torch.save({"model": self.model.state_dict(), "optimizer": {"blocks": [o.state_dict() for o in self.opt],
                                                                    "resident": self.gpu_opt.state_dict()},
                    "step": self.step_count, "config": self.config}, path)

    def load_checkpoint(self, path: str):
        ck = torch.load(path, map_location="cpu", weights_only=False)
        missing = [k for k in ("model", "optimizer", "step", "config") if k not in ck]
        if missing:
            raise ValueError(f"Invalid checkpoint: missing keys {missing}")
        for name in ("hidden_size", "num_layers", "num_heads", "in_channels"):
            if getattr(ck["config"], name) != getattr(self.config, name):
                raise ValueError(f"Checkpoint config mismatch: {name}")
        self._worker_flush()
        self.model.load_state_dict(ck["model"])  # copies into the master views / resident params
        for i in range(self.num_blocks):
            self.stage[i].copy_(self.master[i])
            self.opt[i].load_state_dict(ck["optimizer"]["blocks"][i])
        self.gpu_opt.load_state_dict(ck["optimizer"]["resident"])
        self.slot_block = [-1, -1]
        if self.resident:
            self.res_dirty = [True] * self.num_blocks
        self.step_count = int(ck["step"])


def timeline_summary(timeline: list, origin: torch.cuda.Event) -> dict:
    """Per-kind totals and the overlap of the side-stream copies with block compute for a recorded
    CPUMasterVideoDiT.timeline (events must be complete): intervals in ms from `origin`; overlap = the
    share of copy time during which a block computes on the compute stream."""
    iv = [(k, b, sname, origin.elapsed_time(s), origin.elapsed_time(e)) for k, b, sname, s, e in timeline]
    comp = sorted((a, z) for k, _, sname, a, z in iv if sname == "compute")

    def overlap(a: float, z: float) -> float:
        return sum(max(0.0, min(z, cz) - max(a, ca)) for ca, cz in comp)

    out: dict = {"intervals": len(iv)}
    for kind in ("h2d", "d2h", "fwd", "recompute", "bwd"):
        sel = [(a, z) for k, _, _, a, z in iv if k == kind]
        tot = sum(z - a for a, z in sel)
        out[kind] = {"count": len(sel), "ms": tot}
        if kind in ("h2d", "d2h") and tot > 0:
            out[kind]["overlapped_with_compute_frac"] = sum(overlap(a, z) for a, z in sel) / tot
    out["first_blocks"] = [[k, b, round(a, 3), round(z, 3)] for k, b, _, a, z in sorted(iv, key=lambda r: r[3])[:24]]
    return out

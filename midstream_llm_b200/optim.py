"""Fused AdamW, GradScaler and gradient clipping over the model's flat buffers.

Drop-in for the objects the reference trainer builds
(Midstream-LLM src/jishui/pretrain_torch.py:119-121, 218-233):

* `AdamW(model.parameters(), lr, betas, eps, weight_decay, fused=True)` — one
  `jx_adamw_step` launch updates every parameter, its moments and the fp16
  weight copy. `state_dict()` / `load_state_dict()` use torch.optim.AdamW's
  format (per-parameter `step`, `exp_avg`, `exp_avg_sq`; the same group keys),
  so `training.pt` bundles move between this trainer and the reference.
* `GradScaler(init_scale=...)` — torch.amp.GradScaler's API and state dict;
  the loss scale and growth tracker live on the device.
* `clip_grad_norm_(parameters, max_norm)` — total L2 norm and clip
  coefficient, as torch.nn.utils.clip_grad_norm_ computes them.

`scaler.unscale_()` unscales the flat gradient buffer in place in the same
pass that checks it for non-finite values and sums its squares, so `.grad`
holds unscaled gradients afterwards, as with torch.amp.GradScaler: the
reference loop body (pretrain_torch.py:218-219) runs unchanged with
`torch.nn.utils.clip_grad_norm_`, which rescales `.grad` itself. This
module's `clip_grad_norm_` instead finishes the norm from the statistics the
unscale pass already left and folds the clip coefficient into the AdamW pass,
so the clipped gradients are never written.
"""
from __future__ import annotations

import math
from typing import Iterable

import torch

from . import ops


def _flat_of(params):
    from .model import owner_of
    params = list(params)
    return owner_of(params).flat()


def _shard_reducer(flat):
    """The model's GradReducer when it runs the sharded (ZeRO-1-style) update, else None."""
    from .model import owner_of
    red = owner_of(flat.params[:1]).grad_reducer
    return red if red is not None and red.sharded() else None


def _stats_pass(flat, inv: torch.Tensor, found_inf: torch.Tensor, write_back: bool) -> None:
    """Sum of squares of g * inv (per-block partials in flat.stats_partial) and the inf flag, optionally
    writing g * inv back. Sharded: over this rank's shard, with the 1/world_size of the mean folded into
    inv, then the partials and the flag are summed across ranks."""
    red = _shard_reducer(flat)
    lo, hi = (0, flat.numel) if red is None else red.shard_range(flat)
    if red is not None:
        inv = inv / red.world_size()
    g = flat.g32[lo:hi]
    flat.stats_count = ops.grad_stats(g, inv, flat.stats_partial, found_inf, unscaled_out=g if write_back else None)
    if red is not None:
        red.reduce_stats(flat.stats_partial[:flat.stats_count], found_inf)


class AdamW(torch.optim.Optimizer):
    """torch.optim.AdamW(fused=True) semantics over the flat parameter buffer."""

    def __init__(self, params, lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8, weight_decay: float = 1e-2,
                 amsgrad: bool = False, *, maximize: bool = False, foreach=None, capturable: bool = False,
                 differentiable: bool = False, fused: bool | None = True):
        if amsgrad or maximize or differentiable:
            raise ValueError("amsgrad, maximize and differentiable are not supported by the fused B200 AdamW")
        if not 0.0 <= lr or not 0.0 <= eps or not 0.0 <= betas[0] < 1.0 or not 0.0 <= betas[1] < 1.0:
            raise ValueError("invalid AdamW hyper-parameters")
        defaults = dict(lr=lr, betas=tuple(betas), eps=eps, weight_decay=weight_decay, amsgrad=False,
                        maximize=False, foreach=foreach, capturable=capturable, differentiable=False, fused=True)
        super().__init__(params, defaults)
        if len(self.param_groups) != 1:
            raise ValueError("the fused B200 AdamW takes a single parameter group")
        self._m = self._v = None
        self._step_state = None
        self._flat = None

    # -- flat state --------------------------------------------------------
    def _ensure_state(self):
        params = self.param_groups[0]["params"]
        flat = _flat_of(params)
        if flat is not self._flat:
            if len(params) != len(flat.params) or any(a is not b for a, b in zip(params, flat.params)):
                raise ValueError("the fused B200 AdamW must be given all of the model's parameters, in order")
            old_m, old_v, old_flat = self._m, self._v, self._flat
            self._m = torch.zeros_like(flat.p32)
            self._v = torch.zeros_like(flat.p32)
            if self._step_state is None:
                self._step_state = torch.zeros(4, dtype=torch.float32, device=flat.device)
            if old_flat is not None:  # the model was re-flattened (e.g. moved); carry the moments over
                with torch.no_grad():
                    for n, p in zip(flat.names, flat.params):
                        o, k = old_flat.offsets[n], p.numel()
                        self._m_view(flat, n, p).copy_(old_m[o:o + k].view(p.shape))
                        self._v_view(flat, n, p).copy_(old_v[o:o + k].view(p.shape))
            self._flat = flat
        return flat

    def _m_view(self, flat, name, p):
        o = flat.offsets[name]
        return self._m[o:o + p.numel()].view(p.shape)

    def _v_view(self, flat, name, p):
        o = flat.offsets[name]
        return self._v[o:o + p.numel()].view(p.shape)

    # -- step ----------------------------------------------------------------
    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        flat = self._ensure_state()
        group = self.param_groups[0]
        if any(p.grad is None for p in group["params"]):
            if all(p.grad is None for p in group["params"]):
                return loss
            flat.prepare_grads()  # zero-fill parameters that received no gradient
        beta1, beta2 = group["betas"]
        red = _shard_reducer(flat)
        lo, hi = (0, flat.numel) if red is None else red.shard_range(flat)
        ops.adamw_step(flat.p32[lo:hi], flat.g32[lo:hi], self._m[lo:hi], self._v[lo:hi], flat.p16[lo:hi],
                       flat.inv_scale, flat.clip, flat.found_inf, self._step_state, group["lr"], beta1, beta2,
                       group["eps"], group["weight_decay"])
        if red is not None:  # every rank's updated fp16 shard, and the fp32 norm parameters, to every rank
            red.gather_f16(flat)
            red.sync_f32_params(flat)
        flat.mark_f16_current()
        flat.inv_scale = flat.clip = flat.found_inf = None
        flat.stats_ready = False
        return loss

    # -- checkpoint format -------------------------------------------------
    def state_dict(self):
        group = self.param_groups[0]
        params = group["params"]
        if self._m is None:
            state = {}
        else:
            flat = self._flat
            step = float(self._step_state[0].item())
            state = {}
            if step > 0:
                for i, (n, p) in enumerate(zip(flat.names, params)):
                    state[i] = {"step": torch.tensor(step, dtype=torch.float32, device=p.device),
                                "exp_avg": self._m_view(flat, n, p).clone(),
                                "exp_avg_sq": self._v_view(flat, n, p).clone()}
        packed = {k: v for k, v in group.items() if k != "params"}
        packed["params"] = list(range(len(params)))
        return {"state": state, "param_groups": [packed]}

    def load_state_dict(self, state_dict):
        groups = state_dict["param_groups"]
        if len(groups) != 1 or len(groups[0]["params"]) != len(self.param_groups[0]["params"]):
            raise ValueError("loaded state dict has a different parameter layout")
        for k, v in groups[0].items():
            if k != "params":
                self.param_groups[0][k] = tuple(v) if k == "betas" else v
        flat = self._ensure_state()
        params = self.param_groups[0]["params"]
        saved = state_dict["state"]
        steps = set()
        with torch.no_grad():
            self._m.zero_()
            self._v.zero_()
            for idx, (n, p) in enumerate(zip(flat.names, params)):
                entry = saved.get(idx, saved.get(str(idx)))
                if entry is None:
                    continue
                self._m_view(flat, n, p).copy_(entry["exp_avg"])
                self._v_view(flat, n, p).copy_(entry["exp_avg_sq"])
                steps.add(float(entry["step"]))
        if len(steps) > 1:
            raise ValueError("the fused B200 AdamW keeps one step count; the loaded state has several")
        self._step_state.zero_()
        if steps:
            self._step_state[0] = steps.pop()

    @property
    def state_step(self) -> float:
        return 0.0 if self._step_state is None else float(self._step_state[0].item())


class GradScaler:
    """torch.amp.GradScaler("cuda") semantics; scale and growth tracker on the device."""

    def __init__(self, device: str = "cuda", init_scale: float = 2.0 ** 16, growth_factor: float = 2.0,
                 backoff_factor: float = 0.5, growth_interval: int = 2000, enabled: bool = True):
        if not enabled:
            raise ValueError("the B200 training step always runs fp16 AMP; a disabled GradScaler is not supported")
        self._device = torch.device(device if device != "cuda" else "cuda")
        self._init_scale = float(init_scale)
        self._growth_factor = float(growth_factor)
        self._backoff_factor = float(backoff_factor)
        self._growth_interval = int(growth_interval)
        self._scale = None
        self._growth_tracker = None
        self._found_inf = None
        self._unscaled = set()

    def _lazy(self, device):
        if self._scale is None:
            self._scale = torch.full((), self._init_scale, dtype=torch.float32, device=device)
            self._growth_tracker = torch.zeros(1, dtype=torch.int32, device=device)
            self._found_inf = torch.zeros(1, dtype=torch.float32, device=device)

    def is_enabled(self) -> bool:
        return True

    def scale(self, outputs: torch.Tensor) -> torch.Tensor:
        self._lazy(outputs.device)
        return outputs * self._scale

    def unscale_(self, optimizer: AdamW) -> None:
        if id(optimizer) in self._unscaled:
            raise RuntimeError("unscale_() has already been called on this optimizer since the last update().")
        flat = optimizer._ensure_state()
        self._lazy(flat.device)
        inv = self._scale.double().reciprocal().float().reshape(1)
        self._found_inf.zero_()
        _stats_pass(flat, inv, self._found_inf, write_back=True)
        # The buffer now holds unscaled gradients: the update applies no further factor.
        flat.inv_scale, flat.found_inf, flat.clip = None, self._found_inf, None
        flat.stats_ready = True
        self._unscaled.add(id(optimizer))

    def step(self, optimizer: AdamW, *args, **kwargs):
        if id(optimizer) not in self._unscaled:
            self.unscale_(optimizer)
        return optimizer.step(*args, **kwargs)

    def update(self, new_scale=None) -> None:
        if self._scale is None:
            return
        if new_scale is not None:
            if isinstance(new_scale, float):
                self._scale.fill_(new_scale)
            else:
                self._scale.copy_(new_scale)
        else:
            ops.scaler_update(self._scale, self._growth_tracker, self._found_inf, self._growth_factor,
                              self._backoff_factor, self._growth_interval)
        self._unscaled.clear()

    def get_scale(self) -> float:
        return self._init_scale if self._scale is None else float(self._scale.item())

    @property
    def found_inf(self) -> torch.Tensor | None:
        return self._found_inf

    def state_dict(self) -> dict:
        return {"scale": self.get_scale(), "growth_factor": self._growth_factor,
                "backoff_factor": self._backoff_factor, "growth_interval": self._growth_interval,
                "_growth_tracker": 0 if self._growth_tracker is None else int(self._growth_tracker.item())}

    def load_state_dict(self, state_dict: dict) -> None:
        self._init_scale = float(state_dict["scale"])
        self._growth_factor = float(state_dict["growth_factor"])
        self._backoff_factor = float(state_dict["backoff_factor"])
        self._growth_interval = int(state_dict["growth_interval"])
        if self._scale is not None:
            self._scale.fill_(self._init_scale)
            self._growth_tracker.fill_(int(state_dict["_growth_tracker"]))
        else:
            self._pending_tracker = int(state_dict["_growth_tracker"])
            self._lazy(torch.device("cuda", torch.cuda.current_device()))
            self._growth_tracker.fill_(self._pending_tracker)


def clip_grad_norm_(parameters: Iterable[torch.nn.Parameter], max_norm: float, norm_type: float = 2.0,
                    error_if_nonfinite: bool = False, foreach=None) -> torch.Tensor:
    """Total L2 norm of the (unscaled) gradients and the clip coefficient
    min(max_norm / (norm + 1e-6), 1), applied inside the next fused update."""
    if norm_type != 2.0:
        raise ValueError("only the L2 norm is implemented")
    params = list(parameters)
    flat = _flat_of(params)
    if not flat.stats_ready:  # no GradScaler.unscale_ this update: statistics of the gradients as they are
        one = torch.ones(1, dtype=torch.float32, device=flat.device)
        if flat.found_inf is None:
            flat.found_inf = torch.zeros(1, dtype=torch.float32, device=flat.device)
        # Sharded updates reduce gradient sums: the mean's 1/world_size is written into the shard here.
        _stats_pass(flat, one, flat.found_inf, write_back=_shard_reducer(flat) is not None)
        flat.stats_ready = True
    ops.grad_finalize(flat.stats_partial, flat.stats_count, float(max_norm), flat.norm_out)
    flat.clip = flat.norm_out[1:2]
    total = flat.norm_out[0].clone()
    if error_if_nonfinite and not bool(torch.isfinite(total)):
        raise RuntimeError("the total norm of the gradients is non-finite")
    return total

"""Action codec of the gymnasium wrapper with the mask computed on the device.

Mirrors python/carl/gymnasium/action.py:8-38 (CARLActionCodec): the same
constructor, `action_shape` and `mask(observation)`; the mask is one kernel
launch (carlb_action_mask) on the current CUDA stream instead of a chain of
torch ops.  Observations must be float32 CUDA tensors whose last dimension is
one observation row.
"""

from __future__ import annotations

import torch as th
import torch.nn as nn

from . import capi
from .carl import ACTION_LOGITS, ACTION_NVECS, OBS_PREVIOUS_CONTROLS


class CARLActionCodec(nn.Module):
    def __init__(self, previous_controls: bool = False):
        super().__init__()
        self._previous_controls = bool(previous_controls)
        self._controls_size = OBS_PREVIOUS_CONTROLS if previous_controls else 0

    @property
    def action_shape(self) -> tuple[int, ...]:
        return (len(ACTION_NVECS),)

    def mask(self, observation: th.Tensor) -> th.Tensor:
        """bool [..., ACTION_LOGITS]: powerslide needs the ego on the ground,
        boost needs boost > 0, jump needs the ground or a flip with more than one
        tick of dodge window left; every other logit is allowed."""
        if not isinstance(observation, th.Tensor) or observation.dtype != th.float32:
            raise TypeError("observation must be a float32 tensor")
        if not observation.is_cuda:
            raise ValueError("observation must be on a CUDA device")
        obs = observation.contiguous()
        obs_dim = obs.shape[-1]
        rows = obs.numel() // obs_dim if obs_dim else 0
        mask = th.empty((*obs.shape[:-1], ACTION_LOGITS), dtype=th.bool, device=obs.device)
        stream = th.cuda.current_stream(obs.device).cuda_stream
        capi.action_mask(obs, rows, obs_dim, self._previous_controls, mask, stream)
        return mask


__all__ = ["ACTION_NVECS", "CARLActionCodec"]

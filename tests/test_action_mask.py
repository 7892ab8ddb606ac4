"""Device action mask (carlb_action_mask, carl_b200.action.CARLActionCodec)
against the reference's torch formula (python/carl/gymnasium/action.py:17-37),
restated below on the same observation rows: real rows packed by an env, and
synthetic rows with the edge values (zero, negative, NaN, a dodge window of
exactly PHYS_DT) in every gating field."""

from __future__ import annotations

import numpy as np
import pytest

from carl_b200 import capi, carl, workloads

pytestmark = pytest.mark.gpu


def reference_mask(observation, previous_controls: bool):
    import torch as th

    size = carl.OBS_PREVIOUS_CONTROLS if previous_controls else 0
    on_ground = observation[..., carl.OBS_EGO_ON_GROUND_INDEX].bool()
    has_boost = observation[..., carl.OBS_EGO_BOOST_INDEX].gt(0)
    flip_available = observation[..., carl.OBS_EGO_FLIP_INDEX - size].bool()
    jump_available = on_ground | (flip_available & (observation[..., carl.OBS_EGO_DODGE_TIME_INDEX - size] > carl.PHYS_DT))
    mask = th.ones((*observation.shape[:-1], carl.ACTION_LOGITS), dtype=th.bool, device=observation.device)
    mask[..., carl.ACTION_POWERSLIDE_LOGIT] = on_ground
    mask[..., carl.ACTION_BOOST_LOGIT] = has_boost
    mask[..., carl.ACTION_JUMP_LOGIT] = jump_available
    return mask


@pytest.mark.parametrize("previous_controls", [False, True])
def test_mask_of_packed_observations(previous_controls):
    import torch as th

    from carl_b200.action import CARLActionCodec

    env = carl.Env(512, 2, 2, 3, previous_controls=previous_controls)
    workloads.mixed_state(env._env, 4)
    rng = np.random.default_rng(5)
    codec = CARLActionCodec(previous_controls)
    env_stream = th.cuda.ExternalStream(env.stream)
    for _ in range(4):
        obs = env.step(th.from_numpy(workloads.discrete_actions(rng, 512 * 4).reshape(512, 4, 7)).cuda())
        # Outputs are written on the env stream; hand them to torch's stream first
        # (as the reference's gymnasium/torch.py does).
        th.cuda.current_stream().wait_stream(env_stream)
        assert th.equal(codec.mask(obs), reference_mask(obs, previous_controls))
    assert codec.action_shape == (7,)


@pytest.mark.parametrize("previous_controls", [False, True])
def test_mask_edge_values(previous_controls):
    import torch as th

    from carl_b200.action import CARLActionCodec

    obs_dim = carl.OBS_BALL + 3 * carl.OBS_PER_CAR + 2 * 34 + 6 + 2 * 6 + 6 + 2 + 5 + (8 if previous_controls else 0)
    rng = np.random.default_rng(6)
    rows = rng.normal(0, 1, (3, 1001, obs_dim)).astype(np.float32)
    size = carl.OBS_PREVIOUS_CONTROLS if previous_controls else 0
    fields = [carl.OBS_EGO_ON_GROUND_INDEX, carl.OBS_EGO_BOOST_INDEX, obs_dim + carl.OBS_EGO_FLIP_INDEX - size,
              obs_dim + carl.OBS_EGO_DODGE_TIME_INDEX - size]
    dt = np.float32(carl.PHYS_DT)
    edge = np.array([0.0, -0.0, 1.0, -1.0, np.nan, dt, np.nextafter(dt, np.float32(1)), np.inf], np.float32)
    for f in fields:
        rows[..., f] = edge[rng.integers(0, edge.size, rows.shape[:-1])]
    obs = th.from_numpy(rows).cuda()
    codec = CARLActionCodec(previous_controls)
    assert th.equal(codec.mask(obs), reference_mask(obs, previous_controls))
    # A non-contiguous view is packed the same.
    assert th.equal(codec.mask(obs[:, ::2]), reference_mask(obs[:, ::2], previous_controls))


def test_mask_argument_errors():
    import torch as th

    from carl_b200.action import CARLActionCodec

    codec = CARLActionCodec()
    with pytest.raises(TypeError):
        codec.mask(th.zeros((2, 200), dtype=th.float64, device="cuda"))
    with pytest.raises(ValueError):
        codec.mask(th.zeros((2, 200)))
    with pytest.raises(capi.CarlbError, match="obs_dim"):
        codec.mask(th.zeros((2, 20), device="cuda"))
    assert codec.mask(th.zeros((0, 200), device="cuda")).shape == (0, 18)
    obs = th.zeros((4, 200), device="cuda")
    out = th.zeros(4 * 18 + 4, dtype=th.uint8, device="cuda")
    with pytest.raises(capi.CarlbError, match="aligned"):
        capi.action_mask(obs, 4, 200, False, out.data_ptr() + 1, th.cuda.current_stream().cuda_stream)

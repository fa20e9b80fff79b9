"""CPU checks of the conv-policy oracle: the crop encoder
agrees with the 15x15 observation on the central window and transforms
consistently under D4; the autoregressive sampler's log-prob and entropy equal a
torch restatement of the reference ActionDistribution
(autoregressive-actions-v1/scripts/tactical_models.py:8-30) and its draws only
take actions of nonzero probability."""
import numpy as np
import torch
from torch.distributions import Categorical

import oracle
from golden.schedule import random_actions
from test_spec_oracle import SPEC


def played(n=48, steps=50, seed=5):
    env = oracle.OracleSpec(n, SPEC, seed=seed)
    acts = random_actions(seed, steps, n, 12)
    for k in range(steps):
        env.step(acts[k])
    return env


def test_crop_center_window_is_the_observation(oracle_lib):
    env = played()
    crop = env.crop(0)
    obs = env.obs[:, :1800].reshape(env.batch, 15, 15, 8)
    assert np.array_equal(crop[:, 24:39, 24:39] & 7, obs.argmax(-1))
    assert (crop[:, :, 63] == 0).all()
    # pixels off the map carry neither the on-map bit nor a class
    off = (crop[:, :, :63] & 8) == 0
    assert ((crop[:, :, :63][off]) == 0).all()


def test_crop_d4_elements_permute_pixels(oracle_lib):
    env = played(seed=6)
    base = env.crop(0)
    ys, xs = np.mgrid[0:63, 0:63]
    dx, dy = xs - 31, ys - 31
    for g in range(8):
        r = g % 4
        a = [dx, dy, -dx, -dy][r]
        b = [dy, -dx, -dy, dx][r]
        if g >= 4:
            a = -a
        assert np.array_equal(env.crop(g)[:, :, :63], base[:, b + 31, a + 31]), g


def test_ar_sampler_matches_reference_distribution(oracle_lib):
    env = played(n=64, seed=7)
    rng = np.random.default_rng(0)
    vl = rng.normal(size=(64, 12)).astype(np.float32)
    tl = rng.normal(size=(64, 2, 9)).astype(np.float32)
    joint, act, lp, ent = oracle.sample_ar(vl, tl, env.legal, 3, 4, 0)
    bits = torch.from_numpy(env.legal.astype(np.int64))
    b = lambda k: ((bits >> k) & 1).bool()
    tvalid = torch.stack((torch.stack([b(t) for t in range(8)] + [torch.zeros_like(b(0))], 1),
                          torch.stack([b(t) & b(10) for t in range(8)] + [b(10)], 1)), 1)
    vmask = torch.zeros(64, 12, dtype=torch.bool)
    vmask[:, 2], vmask[:, 3], vmask[:, 4] = b(8), b(9), b(11)
    type_mask = torch.cat((tvalid.any(-1), vmask[:, 2:]), -1)
    types = Categorical(logits=torch.from_numpy(vl).masked_fill(~type_mask, -1e9))
    safe = tvalid | ~tvalid.any(-1, keepdim=True)
    dirs = Categorical(logits=torch.from_numpy(tl).masked_fill(~safe, -1e9))
    j = torch.from_numpy(joint)
    kind = torch.where(j < 18, j // 9, j - 16)
    cond = dirs.logits.gather(2, (j % 9)[:, None, None].expand(-1, 2, 1)).squeeze(-1)
    cond = cond.gather(1, kind.clamp_max(1)[:, None]).squeeze(1)
    ref_lp = types.log_prob(kind) + torch.where(kind < 2, cond, torch.zeros_like(cond))
    ref_ent = types.entropy() + (types.probs[:, :2] * dirs.entropy()).sum(-1)
    assert np.allclose(lp, ref_lp.numpy(), rtol=1e-5, atol=1e-5)
    assert np.allclose(ent, ref_ent.numpy(), rtol=1e-5, atol=1e-5)
    assert (type_mask.gather(1, kind[:, None]).squeeze(1)).all()
    legal = env.legal.astype(np.int64)
    assert ((act >= 0) & (((legal >> np.maximum(act, 0)) & 1) == 1)).all()

"""Centered-map conv policy with the autoregressive head on
the GPU:

* crops: d1_spec_crop equals the CPU oracle's crop, bit for bit, under all 8
  D4 elements, on envs that played random actions in lockstep with the oracle;
* conv stack + FC + head GEMMs: against torch Conv2d/Linear in fp32 on the same
  bf16 weights, with activations rounded to bf16 between layers as the kernels
  store them (tolerance 1e-2 of the layer's scale);
* autoregressive head: target logits against the torch direction MLP; log-prob
  and entropy against a torch restatement of the reference ActionDistribution
  (autoregressive-actions-v1/scripts/tactical_models.py:8-30) at 1e-5; sampled
  (verb, target) and env actions identical to the oracle sampler; empirical
  joint frequencies against the distribution's probabilities.
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F
from torch.distributions import Categorical

import oracle
from golden.schedule import random_actions

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def mods():
    from d1 import conv_policy, spec_env
    oracle.build()
    return conv_policy, spec_env


@pytest.fixture(scope='module')
def played(mods):
    """GPU and oracle envs after 60 random decisions in lockstep (n = 192)."""
    conv_policy, spec_env = mods
    n, steps = 192, 60
    gpu, cpu = spec_env.SpecEnv(n, seed=11), oracle.OracleSpec(n, spec_env.DEFAULT, seed=11)
    acts = random_actions(77, steps, n, 12)
    dev = torch.from_numpy(acts).cuda()
    for k in range(steps):
        cpu.step(acts[k])
        gpu.step(dev[k].contiguous())
    assert np.array_equal(gpu.compact().cpu().numpy(), cpu.compact())
    return gpu, cpu


def test_crop_matches_oracle_under_all_d4_elements(mods, played):
    conv_policy, _ = mods
    gpu, cpu = played
    pol = conv_policy.ConvPolicy(seed=1)
    buf = pol.buffers(gpu.batch)
    for g in range(8):
        pol.encode(gpu.state, gpu.batch, buf, g)
        got = buf['crop'].cpu().numpy().view(np.uint16)
        ref = cpu.crop(g)
        assert np.array_equal(got, ref), (g, np.argwhere(got != ref)[:5].tolist())


def expand(crop):
    """u16 codes [n, 63, 64] -> the 10 input channels [n, 10, 63, 63]."""
    c = crop[:, :, :63].to(torch.int32) & 0xffff
    cls = c & 7
    ch = [(cls == k).float() for k in range(8)]
    ch += [((c >> 4) & 31).float() / 32, ((c >> 3) & 1).float()]
    return torch.stack(ch, 1)


def bf(x):
    return x.to(torch.bfloat16).float()


def conv_reference(pol, crop):
    x = expand(crop)
    for i in (1, 2, 3):
        w = bf(pol.params[f'c{i}w'])
        x = bf(F.relu(F.conv2d(x, w, pol.params[f'c{i}b'], stride=2)))
    return x.permute(0, 2, 3, 1).reshape(x.shape[0], -1)


def close(got, ref, what, tol=1e-2):
    scale = ref.abs().max().item()
    err = (got - ref).abs().max().item()
    assert err <= tol * max(scale, 1e-3), (what, err, scale)


def test_conv_stack_fc_and_head_match_torch(mods, played):
    conv_policy, _ = mods
    gpu, _ = played
    n = gpu.batch
    pol = conv_policy.ConvPolicy(seed=2, chunk=64)  # several chunks
    buf = pol.buffers(n)
    pol.encode(gpu.state, n, buf, 0)
    pol.features(buf, n)
    torch.cuda.synchronize()
    assert conv_policy.conv_error() == 0
    ref = conv_reference(pol, buf['crop'])
    got = buf['fc_in'].float()
    close(got, ref, 'conv stack')
    assert (got - ref).abs().mean().item() < 1e-3 * max(ref.abs().max().item(), 1e-3)
    # FC and head on the kernels' own inputs
    h_ref = F.relu(got @ bf(pol.params['fcw']).T + pol.params['fcb'])
    close(buf['h'].float(), h_ref, 'fc')
    hb_ref = buf['h'].float() @ bf(pol.params['hw']).T + pol.params['hb']
    close(buf['hb'], hb_ref, 'head', tol=1e-4)


def masks(legal):
    bits = legal.to(torch.int64) & 0xffff
    b = lambda k: ((bits >> k) & 1).bool()
    move = torch.stack([b(t) for t in range(8)] + [torch.zeros_like(b(0))], 1)
    att = torch.stack([b(t) & b(10) for t in range(8)] + [b(10)], 1)
    tvalid = torch.stack((move, att), 1)
    vmask = torch.zeros(bits.shape[0], 12, dtype=torch.bool, device=legal.device)
    vmask[:, 2], vmask[:, 3], vmask[:, 4] = b(8), b(9), b(11)
    return tvalid, vmask


class ReferenceActionDistribution:
    """The reference's ActionDistribution (autoregressive-actions-v1/scripts/
    tactical_models.py:8-30) restated for 12 verbs of which the first two carry a
    9-way target: type mask = any valid target for directional verbs; a safe
    dummy conditional when a directional verb has no valid target."""

    def __init__(self, verb_logits, target_logits, tvalid, vmask):
        type_mask = torch.cat((tvalid.any(-1), vmask[:, 2:]), -1)
        self.types = Categorical(logits=verb_logits.masked_fill(~type_mask, -1e9))
        safe = tvalid | ~tvalid.any(-1, keepdim=True)
        self.directions = Categorical(logits=target_logits.masked_fill(~safe, -1e9))
        self.probs = torch.cat(((self.types.probs[:, :2, None] * self.directions.probs).flatten(1),
                                self.types.probs[:, 2:]), -1)

    def log_prob(self, joint):
        kind = torch.where(joint < 18, joint // 9, joint - 16)
        t = joint % 9
        cond = self.directions.logits.gather(2, t[:, None, None].expand(-1, 2, 1)).squeeze(-1)
        cond = cond.gather(1, kind.clamp_max(1)[:, None]).squeeze(1)
        return self.types.log_prob(kind) + torch.where(kind < 2, cond, torch.zeros_like(cond))

    def entropy(self):
        return self.types.entropy() + (self.types.probs[:, :2] * self.directions.entropy()).sum(-1)


def test_ar_head_matches_reference_distribution_and_oracle(mods, played):
    conv_policy, _ = mods
    gpu, _ = played
    n = gpu.batch
    pol = conv_policy.ConvPolicy(seed=3)
    buf = pol.buffers(n)
    out = pol.act(gpu.state, gpu.legal, n, buf, seed=5, step=9, first_env=100, debug=True)
    torch.cuda.synchronize()
    hb = buf['hb']
    # target logits = W_t . tanh(pre + cond_k) + b_t
    pre = hb[:, 13:77]
    hid = torch.tanh(pre[:, None, :] + pol.cond[None])
    t_ref = hid @ pol.params['wt'].T + pol.params['bt']
    assert torch.allclose(out['target_logits'], t_ref, rtol=1e-5, atol=1e-5)
    assert torch.equal(out['verb_logits'], hb[:, :12])
    assert torch.equal(out['value'], hb[:, 12])
    tvalid, vmask = masks(gpu.legal)
    dist = ReferenceActionDistribution(out['verb_logits'], out['target_logits'], tvalid, vmask)
    joint = out['joint']
    assert (dist.probs.gather(1, joint[:, None]) > 0).all(), 'sampled an action of zero probability'
    assert torch.allclose(out['logp'], dist.log_prob(joint), rtol=1e-5, atol=1e-5)
    assert torch.allclose(out['entropy'], dist.entropy(), rtol=1e-5, atol=1e-5)
    j, a, lp, ent = oracle.sample_ar(out['verb_logits'].cpu().numpy(), out['target_logits'].cpu().numpy(),
                                     gpu.legal.cpu().numpy().view(np.uint16), 5, 9, 100)
    assert np.array_equal(joint.cpu().numpy(), j)
    assert np.array_equal(out['env_action'].cpu().numpy(), a)
    assert np.allclose(out['logp'].cpu().numpy(), lp, rtol=1e-6, atol=1e-6)
    assert np.allclose(out['entropy'].cpu().numpy(), ent, rtol=1e-5, atol=1e-5)


def test_ar_sampling_frequencies_follow_the_joint_distribution(mods):
    """One logits row replicated over 200,000 env ids: joint frequencies within
    5 standard errors of the probabilities (legal: all moves, wait, attack)."""
    from d1._lib import library
    n = 200_000
    g = torch.Generator(device='cuda').manual_seed(0)
    hb = torch.zeros((n, 80), device='cuda')
    hb[:, :12] = torch.randn(12, device='cuda', generator=g)
    hb[:, 13:77] = torch.randn(64, device='cuda', generator=g)
    cond = torch.randn(2, 64, device='cuda', generator=g)
    wt = torch.randn(9, 64, device='cuda', generator=g) / 8
    bt = torch.randn(9, device='cuda', generator=g)
    legal = torch.full((n,), 0xff | (1 << 8) | (1 << 10), dtype=torch.int16, device='cuda')
    joint = torch.empty(n, dtype=torch.int64, device='cuda')
    vl = torch.empty((n, 12), device='cuda')
    tl = torch.empty((n, 2, 9), device='cuda')
    assert library().d1_ar_head_sample(hb.data_ptr(), n, cond.data_ptr(), wt.data_ptr(), bt.data_ptr(),
                                       legal.data_ptr(), 7, 3, 0, joint.data_ptr(), None, None, None, None,
                                       vl.data_ptr(), tl.data_ptr(), torch.cuda.current_stream().cuda_stream) == 0
    tvalid, vmask = masks(legal[:1])
    p = ReferenceActionDistribution(vl[:1], tl[:1], tvalid, vmask).probs[0].double()
    freq = torch.bincount(joint, minlength=28).double() / n
    se = (p * (1 - p) / n).sqrt()
    assert ((freq - p).abs() <= 5 * se + 1e-9).all(), (freq - p).abs().max().item()


def test_conv_rollout_plays_legal_actions(mods):
    conv_policy, spec_env = mods
    n = 1024
    env = spec_env.SpecEnv(n, seed=4, observe=False)
    pol = conv_policy.ConvPolicy(seed=4, chunk=256)
    buf = pol.buffers(n)
    out = None
    for step in range(12):
        legal = env.legal.to(torch.int64) & 0xffff
        out = pol.act(env.state, env.legal, n, buf, seed=1, step=step, out=out)
        a = out['env_action']
        assert (a >= 0).all() and (a < 12).all()
        assert (((legal >> a) & 1) == 1).all(), 'env action outside the legal bits'
        env.step(a)
    torch.cuda.synchronize()
    assert conv_policy.conv_error() == 0
    assert torch.isfinite(out['logp']).all() and torch.isfinite(out['value']).all()

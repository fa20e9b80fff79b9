"""PPO path on the GPU against PyTorch restatements of the reference update
(gpu-d1/scripts/run_ring_ablations.py:354-372):

* GAE: mode 0 bit-exact with the reference's per-step tensor ops; mode 1 (warp
  segmented scan) within 1e-5 relative.
* One minibatch: loss terms and the flat gradient against torch autograd of the
  same loss with the kernels' bf16 rounding points (activations and the two
  hidden-layer gradients), tolerance 1e-3 relative on the loss and 1e-3
  relative L2 per gradient segment; the optimizer step against torch.optim.Adam.
* Config 2 sizes (minibatch 16,384 of a 65,536-env rollout): the same bounds on
  eight optimizer steps in a row.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def mods():
    from d1 import policy, ppo, rollout, spec_env
    return policy, ppo, rollout, spec_env


def small_setup(mods, B=512, T=32, mb=4096, seed=3):
    policy, ppo, rollout, spec_env = mods
    env = spec_env.SpecEnv(B, seed=seed)
    pol = policy.Policy(seed=seed)
    roll = rollout.Rollout(env, pol, T, seed=seed)
    roll.collect()
    trainer = ppo.PPO(pol, roll, minibatch=mb, epochs=1)
    return pol, roll, trainer


def torch_gae(rew, done, values, gamma, lam):
    T = rew.shape[0]
    adv = torch.empty_like(rew)
    nextv = values[T]
    gae = torch.zeros_like(nextv)
    for t in reversed(range(T)):
        live = 1 - done[t]
        delta = rew[t] + gamma * nextv * live - values[t]
        gae = delta + gamma * lam * live * gae
        adv[t], nextv = gae, values[t]
    return adv, adv + values[:T]


def test_gae_modes_against_the_reference_loop(mods):
    pol, roll, tr = small_setup(mods)
    rew, done = roll.out[:, :, 0], roll.out[:, :, 1]
    ref_adv, ref_ret = torch_gae(rew, done, roll.values, tr.gamma, tr.lam)
    tr.gae_mode = 0
    adv, ret = tr.advantages()
    assert torch.equal(adv, ref_adv) and torch.equal(ret, ref_ret)
    s = tr.stats.clone()
    assert abs(s[0].item() - ref_adv.double().sum().item()) <= 1e-6 * max(1.0, abs(s[0].item()))
    tr.gae_mode = 1
    adv1, ret1 = tr.advantages()
    scale = ref_adv.abs().max().item()
    assert (adv1 - ref_adv).abs().max().item() <= 1e-5 * max(scale, 1.0)
    assert (ret1 - ref_ret).abs().max().item() <= 1e-5 * max(ret1.abs().max().item(), 1.0)


@pytest.mark.parametrize('planes', [True, False])
@pytest.mark.parametrize('T,B', [(1, 40), (7, 33), (32, 96), (80, 64), (100, 70), (128, 1000), (256, 32), (300, 45),
                                 (1000, 130)])
def test_gae_scan_over_horizons_and_ragged_batches(T, B, planes):
    """d1_gae mode 1 against the reference loop: horizons from 1 to 1,000 (runs
    of one row to several chunks per warp), env counts that are not a multiple
    of an env group (odd ones take the one-env-per-lane form), outcome rows in
    the env's plane layout [T, 10, B] (reward and done rows contiguous over
    envs: read in pairs) and as [T, B, 10] rows; the statistics against float64
    sums of the same advantages (1e-6 of the absolute sum)."""
    from d1._lib import library
    lib = library()
    g = torch.Generator(device='cuda').manual_seed(T * 1000 + B)
    out = torch.zeros((T, 10, B), device='cuda').permute(0, 2, 1) if planes else torch.zeros((T, B, 10), device='cuda')
    out[:, :, 0] = torch.randn((T, B), device='cuda', generator=g)
    out[:, :, 1] = (torch.rand((T, B), device='cuda', generator=g) < 0.05).float()
    values = torch.randn((T + 1, B), device='cuda', generator=g)
    adv, ret = torch.empty((T, B), device='cuda'), torch.empty((T, B), device='cuda')
    stats = torch.zeros(2, dtype=torch.float64, device='cuda')
    assert lib.d1_gae(out.data_ptr(), out[:, :, 1].data_ptr(), out.stride(0), out.stride(1), values.data_ptr(), T, B,
                      0.999, 0.95, adv.data_ptr(), ret.data_ptr(), stats.data_ptr(), 1, 0) == 0
    torch.cuda.synchronize()
    ref_adv, ref_ret = torch_gae(out[:, :, 0], out[:, :, 1], values, 0.999, 0.95)
    scale = max(ref_adv.abs().max().item(), 1.0)
    assert (adv - ref_adv).abs().max().item() <= 1e-5 * scale
    assert (ret - ref_ret).abs().max().item() <= 1e-5 * max(ref_ret.abs().max().item(), 1.0)
    # each thread adds a chunk of 8 steps in float before the double totals:
    # error below 8 * 2^-24 of the absolute sum
    a64 = adv.double()
    assert abs(stats[0].item() - a64.sum().item()) <= 1e-6 * max(1.0, a64.abs().sum().item())
    assert abs(stats[1].item() - (a64 * a64).sum().item()) <= 1e-6 * (a64 * a64).sum().item()


def bf16_round(x):
    return x.to(torch.bfloat16).to(torch.float32)


class RoundGrad(torch.autograd.Function):
    """Identity forward; rounds the incoming gradient to bf16 (as the kernels
    store dh1 and dh2 in bf16)."""

    @staticmethod
    def forward(ctx, x):
        return x.view_as(x)

    @staticmethod
    def backward(ctx, g):
        return bf16_round(g)


def reference_minibatch(pol, roll, tr, idx, round_grads=True):
    T, B = roll.T, roll.env.batch
    from d1.spec_env import expand_cobs
    obs = expand_cobs(roll.cobs[:T].reshape(T * B, -1)[idx]).float()
    legal = roll.legal[:T].reshape(-1)[idx].to(torch.int32) & 0xffff
    act = roll.actions.reshape(-1)[idx]
    oldlp = roll.logp.reshape(-1)[idx]
    oldv = roll.values[:T].reshape(-1)[idx]
    adv_all = tr.adv.reshape(-1)
    mean = tr.stats[0].item() / tr.adv_count
    var = (tr.stats[1].item() - tr.stats[0].item() * mean) / (tr.adv_count - 1)
    adv = (adv_all[idx] - mean) / (var ** 0.5 + 1e-8)
    ret = tr.ret.reshape(-1)[idx]
    leaf = {k: (pol.bf16[k].float() if k in ('w1', 'w2', 'wh') else pol.params[k].clone()).requires_grad_(True)
            for k in ('w1', 'b1', 'w2', 'b2', 'wh', 'bh')}
    rg = RoundGrad.apply if round_grads else (lambda x: x)
    z1 = obs @ leaf['w1'].T + leaf['b1']
    h1 = torch.relu(rg(z1))
    h1 = h1 + (bf16_round(h1) - h1).detach()  # stored in bf16, gradient passes straight through
    z2 = h1 @ leaf['w2'].T + leaf['b2']
    h2 = torch.relu(rg(z2))
    h2 = h2 + (bf16_round(h2) - h2).detach()
    out = h2 @ leaf['wh'].T + leaf['bh']
    logits, v = out[:, :12], out[:, 12]
    mask = ((legal[:, None] >> torch.arange(12, device=legal.device)) & 1) == 0
    lp_all = torch.log_softmax(logits.masked_fill(mask, -1e9), -1)
    p = lp_all.exp()
    ent = -(p * lp_all.masked_fill(mask, 0)).sum(-1)
    la = lp_all.gather(1, act[:, None])[:, 0]
    ratio = (la - oldlp).exp()
    pg = -torch.minimum(ratio * adv, ratio.clamp(1 - tr.clip, 1 + tr.clip) * adv)
    vc = oldv + (v - oldv).clamp(-tr.vclip, tr.vclip)
    vf = torch.maximum((v - ret) ** 2, (vc - ret) ** 2)
    loss = pg.mean() + tr.vf_coef * vf.mean() - tr.ent_coef * ent.mean()
    loss.backward()
    grads = {k: leaf[k].grad for k in leaf}
    return loss.item(), pg.sum().item(), vf.sum().item(), ent.sum().item(), grads


def rel(a, b):
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def test_minibatch_loss_gradient_and_adam_match_torch(mods):
    pol, roll, tr = small_setup(mods)
    tr.advantages()
    g = torch.Generator(device='cuda').manual_seed(0)
    idx = torch.randperm(tr.total, device='cuda', generator=g)[:tr.mb]
    before = pol.flat.clone()
    bf_before = {k: v.clone() for k, v in pol.bf16.items()}
    loss_ref, pg_ref, vf_ref, ent_ref, grads = reference_minibatch(pol, roll, tr, idx)
    terms = tr.minibatch(idx).clone()
    torch.cuda.synchronize()
    n = tr.mb
    loss = terms[0].item() / n + tr.vf_coef * terms[1].item() / n - tr.ent_coef * terms[2].item() / n
    assert abs(loss - loss_ref) <= 1e-3 * max(1.0, abs(loss_ref)), (loss, loss_ref)
    assert abs(terms[1].item() - vf_ref) <= 1e-3 * abs(vf_ref)
    assert abs(terms[2].item() - ent_ref) <= 1e-3 * abs(ent_ref)
    off = tr.off
    for k, shape in [('w1', (256, 1832)), ('b1', (256,)), ('w2', (256, 256)), ('b2', (256,)), ('wh', (13, 256)),
                     ('bh', (13,))]:
        n_el = int(np.prod(shape))
        got = tr.grad[off[k]:off[k] + n_el].view(shape)
        print('segment', k, 'relative L2 error', rel(got, grads[k]))
        assert rel(got, grads[k]) < 1e-3, (k, rel(got, grads[k]))
    # optimizer step = torch.optim.Adam on the same gradient, after grad-norm clipping
    p = before.clone().requires_grad_(True)
    opt = torch.optim.Adam([p], lr=tr.lr, eps=tr.eps, betas=tr.betas)
    gg = tr.grad.clone()
    coef = tr.max_grad_norm / (gg.double().norm().item() + 1e-6)  # clip_grad_norm_ on the flat gradient
    if coef < 1:
        gg.mul_(coef)
    p.grad = gg
    opt.step()
    assert torch.allclose(pol.flat, p.detach(), rtol=1e-5, atol=1e-7)
    assert torch.equal(pol.bf16['w1'], pol.params['w1'].to(torch.bfloat16))
    assert torch.equal(pol.bf16['w2t'], pol.params['w2'].T.contiguous().to(torch.bfloat16))
    assert not torch.equal(pol.bf16['w1'], bf_before['w1'])


def test_reference_loss_switch_matches_plain_mse(mods):
    """vclip <= 0 and vf_coef 0.25 reproduce the reference's 0.25 * MSE value term."""
    pol, roll, tr = small_setup(mods, seed=5)
    tr.vclip, tr.vf_coef = 0.0, 0.25
    tr.advantages()
    idx = torch.arange(tr.mb, device='cuda')
    T, B = roll.T, roll.env.batch
    # value predictions of the pre-update policy on these samples, plain squared error
    from d1.spec_env import expand_cobs
    h1, h2 = pol.hidden_layers(expand_cobs(roll.cobs[:T].reshape(T * B, -1)[idx]).contiguous())
    v = (h2.float() @ pol.bf16['wh'][12].float() + pol.params['bh'][12])
    vf_ref = ((v - tr.ret.reshape(-1)[idx]) ** 2).sum().item()
    terms = tr.minibatch(idx).clone()
    torch.cuda.synchronize()
    assert torch.isfinite(terms).all()
    assert 0 <= terms[3].item() <= tr.mb
    assert abs(terms[1].item() - vf_ref) <= 1e-3 * abs(vf_ref)


def test_full_iteration_runs_and_learns_something(mods):
    pol, roll, tr = small_setup(mods, B=1024, T=32, mb=4096, seed=7)
    start = pol.flat.clone()
    tr.epochs = 2
    roll.roll()
    for _ in range(2):
        tr.iteration()
    torch.cuda.synchronize()
    from d1 import gemm
    assert gemm.gemm_error() == 0
    assert torch.isfinite(pol.flat).all()
    assert not torch.equal(pol.flat, start)


def test_gae_scan_at_the_bench_horizon(mods):
    """T = 128: the scan stages 48 KB of shared memory."""
    pol, roll, tr = small_setup(mods, B=1024, T=128, mb=4096, seed=9)
    rew, done = roll.out[:, :, 0], roll.out[:, :, 1]
    ref_adv, _ = torch_gae(rew, done, roll.values, tr.gamma, tr.lam)
    tr.gae_mode = 1
    adv, _ = tr.advantages()
    assert (adv - ref_adv).abs().max().item() <= 1e-5 * max(ref_adv.abs().max().item(), 1.0)
    s1 = tr.stats[0].item()
    assert abs(s1 - ref_adv.double().sum().item()) <= 1e-4 * max(1.0, abs(s1))


def test_compact_update_equals_the_materialised_update(mods):
    """The default update expands the compact history inside the layer-1 and dW1
    GEMMs; compact=False gathers X = [one-hot rows | ones column] first. Same
    gradients and parameters bit for bit over several minibatches."""
    policy, ppo, rollout, spec_env = mods
    env = spec_env.SpecEnv(512, seed=11)
    pa, pb = policy.Policy(seed=11), policy.Policy(seed=11)
    roll = rollout.Rollout(env, pa, 32, seed=11)
    roll.collect()
    ta = ppo.PPO(pa, roll, minibatch=4096, epochs=1, graph=False, compact=True)
    tb = ppo.PPO(pb, roll, minibatch=4096, epochs=1, graph=False, compact=False)
    ta.advantages()
    tb.advantages()
    g = torch.Generator(device='cuda').manual_seed(4)
    for _ in range(3):
        idx = torch.randperm(ta.total, device='cuda', generator=g)[:ta.mb]
        ta.minibatch(idx)
        tb.minibatch(idx)
        torch.cuda.synchronize()
        assert torch.equal(ta.grad, tb.grad)
        assert torch.equal(pa.flat, pb.flat)
    from d1 import gemm
    assert gemm.gemm_error() == 0


def test_config2_minibatches_match_torch_over_eight_steps(mods):
    """BASELINE config 2 sizes: minibatches of 16,384 drawn from a 65,536-env
    rollout, eight optimizer steps in a row. Every step: loss within 1e-3
    relative and every gradient segment within 1e-3 relative L2 of torch
    autograd at the kernels' bf16 rounding points (at the parameters the GPU
    reached); the step itself equal to clip_grad_norm_(0.5) + torch.optim.Adam
    fed the same gradient, carried over all eight steps. A torch model trained
    on its own autograd gradients for the same eight steps stays within 1e-2
    relative L2 of the GPU's total parameter change."""
    policy, ppo, rollout, spec_env = mods
    env = spec_env.SpecEnv(65536, seed=21)
    pol = policy.Policy(seed=21)
    roll = rollout.Rollout(env, pol, 8, seed=21)
    roll.collect()
    tr = ppo.PPO(pol, roll, minibatch=16384, epochs=1, graph=False)
    tr.advantages()
    start = pol.flat.clone()
    p_adam = start.clone().requires_grad_(True)
    opt = torch.optim.Adam([p_adam], lr=tr.lr, eps=tr.eps, betas=tr.betas)
    p_own = start.clone().requires_grad_(True)
    opt_own = torch.optim.Adam([p_own], lr=tr.lr, eps=tr.eps, betas=tr.betas)
    g = torch.Generator(device='cuda').manual_seed(5)
    perm = torch.randperm(tr.total, device='cuda', generator=g)
    off, n = tr.off, tr.mb
    shapes = [('w1', (256, 1832)), ('b1', (256,)), ('w2', (256, 256)), ('b2', (256,)), ('wh', (13, 256)),
              ('bh', (13,))]
    worst = {}
    for k in range(8):
        idx = perm[k * n:(k + 1) * n]
        loss_ref, _, vf_ref, ent_ref, grads = reference_minibatch(pol, roll, tr, idx)
        terms = tr.minibatch(idx).clone()
        torch.cuda.synchronize()
        loss = terms[0].item() / n + tr.vf_coef * terms[1].item() / n - tr.ent_coef * terms[2].item() / n
        assert abs(loss - loss_ref) <= 1e-3 * max(1.0, abs(loss_ref)), (k, loss, loss_ref)
        for name, shape in shapes:
            got = tr.grad[off[name]:off[name] + int(np.prod(shape))].view(shape)
            e = rel(got, grads[name])
            worst[name] = max(worst.get(name, 0.0), e)
            assert e < 1e-3, (k, name, e)
        # the optimizer on the GPU's own gradient
        gg = tr.grad.clone()
        p_adam.grad = gg
        torch.nn.utils.clip_grad_norm_([p_adam], tr.max_grad_norm)
        opt.step()
        assert torch.allclose(pol.flat, p_adam.detach(), rtol=1e-5, atol=1e-7), k
        # a torch model on its own autograd gradients (same minibatches)
        flat = torch.cat([grads[name].reshape(-1) for name, _ in
                          sorted(shapes, key=lambda s: off[s[0]])])
        p_own.grad = flat.clone()
        torch.nn.utils.clip_grad_norm_([p_own], tr.max_grad_norm)
        opt_own.step()
    drift = rel(pol.flat - start, p_own.detach() - start)
    print('worst gradient error per segment', worst, 'update drift vs autograd model', drift)
    assert drift < 1e-2, drift


def permute_restated(n, seed, epoch):
    """numpy restatement of d1_ppo_permute: alternating Feistel rounds (murmur3
    32-bit finaliser of round key ^ half; round keys from the splitmix64
    finaliser) over the smallest 2^m >= n, walked into [0, n)."""
    def h64(z):
        z = np.asarray(z, dtype=np.uint64)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xbf58476d1ce4e5b9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94d049bb133111eb)
        return z ^ (z >> np.uint64(31))

    def h32(v):
        v = np.asarray(v, dtype=np.uint32)
        v = (v ^ (v >> np.uint32(16))) * np.uint32(0x85ebca6b)
        v = (v ^ (v >> np.uint32(13))) * np.uint32(0xc2b2ae35)
        return v ^ (v >> np.uint32(16))

    with np.errstate(over='ignore'):
        key = h64(np.uint64(seed) ^ h64(np.uint64(epoch) + np.uint64(0x9e3779b97f4a7c15)))
        rk = [np.uint32(int(h64(key + np.uint64(r))) & 0xFFFFFFFF) for r in range(6)]
        m = max(0, int(n - 1).bit_length())
        hb, lb = m // 2, m - m // 2
        hmask, lmask = np.uint32((1 << hb) - 1), np.uint32((1 << lb) - 1)
        x = np.arange(n, dtype=np.uint64)
        todo = np.ones(n, dtype=bool)
        while todo.any():
            y = x[todo]
            hi, lo = (y >> np.uint64(lb)).astype(np.uint32), y.astype(np.uint32) & lmask
            for r in range(0, 6, 2):
                hi = hi ^ (h32(rk[r] ^ lo) & hmask)
                lo = lo ^ (h32(rk[r + 1] ^ hi) & lmask)
            x[todo] = (hi.astype(np.uint64) << np.uint64(lb)) | lo.astype(np.uint64)
            todo[todo] = x[todo] >= np.uint64(n)
        return x.astype(np.int64)


@pytest.mark.parametrize('n', [1, 2, 3, 1000, 4097, 65536])
def test_epoch_permutation_matches_its_restatement(n):
    from d1._lib import library
    lib = library()
    epoch = torch.tensor([7], dtype=torch.int64, device='cuda')
    perm = torch.empty(n, dtype=torch.int64, device='cuda')
    assert lib.d1_ppo_permute(perm.data_ptr(), n, 0x1234, epoch.data_ptr(), 0) == 0
    torch.cuda.synchronize()
    got = perm.cpu().numpy()
    assert np.array_equal(np.sort(got), np.arange(n))
    assert np.array_equal(got, permute_restated(n, 0x1234, 7))


def test_epoch_permutation_at_rollout_size_and_across_epochs(mods):
    """65,536 x 128 samples: every index exactly once, a fresh order for each
    epoch count, and no visible structure (a minibatch's indices spread over
    the whole rollout)."""
    from d1._lib import library
    lib = library()
    n, mb = 65536 * 128, 16384
    epoch = torch.zeros(1, dtype=torch.int64, device='cuda')
    perms = []
    for _ in range(2):
        p = torch.empty(n, dtype=torch.int64, device='cuda')
        assert lib.d1_ppo_permute(p.data_ptr(), n, 99, epoch.data_ptr(), 0) == 0
        assert lib.d1_counter_add(epoch.data_ptr(), 1, 0) == 0
        perms.append(p)
    torch.cuda.synchronize()
    assert epoch.item() == 2
    for p in perms:
        assert torch.equal(torch.sort(p).values, torch.arange(n, device='cuda'))
    assert (perms[0] == perms[1]).float().mean().item() < 1e-3
    first = perms[0][:mb].double()
    # a uniform draw of 16,384 indices has mean n/2 +- n / sqrt(12 * 16384)
    assert abs(first.mean().item() - n / 2) < 5 * n / (12 * mb) ** 0.5
    # the time step (index // B) of consecutive draws is uncorrelated
    t = (perms[0][:mb] // 65536).double()
    c = torch.corrcoef(torch.stack([t[:-1], t[1:]]))[0, 1].item()
    assert abs(c) < 0.05


def test_update_draws_its_order_on_the_device(mods):
    """update() without a generator advances the device epoch count once per
    epoch, eager and graph-replayed epochs alike."""
    pol, roll, tr = small_setup(mods, B=512, T=32, mb=4096, seed=4)
    tr.epochs = 2
    tr.advantages()
    tr.update()
    tr.update()
    torch.cuda.synchronize()
    assert tr.perm_epoch.item() == 4
    assert tr.graph is not None and tr.graph_perm is True
    assert np.array_equal(tr.perm.cpu().numpy(), permute_restated(tr.total, 0, 3))


@pytest.mark.parametrize('B,T,mb', [(512, 32, 4096), (100, 10, 500)])
def test_fused_tail_matches_the_three_launch_path(mods, B, T, mb):
    """d1_ppo_tail (layer 2, head, loss, dh2, dh1 in one launch) against the
    layer-2 GEMM + d1_ppo_loss + dh1 GEMM path on the same minibatch, from the
    same parameters: the flat gradient per segment (1e-3 relative L2), the loss
    terms (1e-5 relative), dh2 and dh1 (bf16 values computed in another
    summation order: nearly all equal, the rest within a rounding step). 500
    rows leave the last 128-row tile ragged."""
    policy, ppo, rollout, spec_env = mods
    from d1 import gemm
    env = spec_env.SpecEnv(B, seed=5)
    pol = policy.Policy(seed=5)
    roll = rollout.Rollout(env, pol, T, seed=5)
    roll.collect()
    fused = ppo.PPO(pol, roll, minibatch=mb, epochs=1, graph=False)
    plain = ppo.PPO(pol, roll, minibatch=mb, epochs=1, graph=False, fused_tail=False)
    assert fused.loss_blocks == (mb + 127) // 128
    fused.advantages()
    plain.advantages()
    g = torch.Generator(device='cuda').manual_seed(3)
    idx = torch.randperm(fused.total, device='cuda', generator=g)[:mb]
    start = pol.flat.clone()
    out = {}
    for name, tr in (('fused', fused), ('plain', plain)):
        pol.flat.copy_(start)
        pol.refresh()
        terms = tr.minibatch(idx).clone()
        torch.cuda.synchronize()
        out[name] = (terms, tr.grad.clone(), tr.dh2.clone(), tr.dh1.clone())
    assert fused.lib.d1_ppo_tail_error() == 0
    assert gemm.gemm_error() == 0
    (tf, gf, d2f, d1f), (tp, gp, d2p, d1p) = out['fused'], out['plain']
    for k in range(5):
        assert abs(tf[k].item() - tp[k].item()) <= 1e-5 * max(1.0, abs(tp[k].item())), (k, tf[k].item(), tp[k].item())
    off = fused.off
    for name, size in [('w1', 256 * 1832), ('b1', 256), ('w2', 256 * 256), ('b2', 256), ('wh', 13 * 256),
                       ('bh', 13)]:
        e = rel(gf[off[name]:off[name] + size], gp[off[name]:off[name] + size])
        assert e < 1e-3, (name, e)
    for a, b in ((d2f, d2p), (d1f, d1p)):
        a, b = a.float(), b.float()
        assert (a == b).float().mean().item() > 0.99
        assert (a - b).abs().max().item() <= 2e-2 * b.abs().max().item()

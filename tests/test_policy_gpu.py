"""Policy head + sampler on the GPU: logits/value against a PyTorch fp32
restatement (tolerance), actions given logits against the CPU oracle (exact)."""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def lib():
    from d1._lib import library
    oracle.build()
    return library()


def run_head(lib, h, wh, bh, legal, seed, step, first_env=0):
    n = h.shape[0]
    a = torch.empty(n, dtype=torch.int64, device='cuda')
    lp = torch.empty(n, device='cuda')
    v = torch.empty(n, device='cuda')
    lg = torch.empty((n, 12), device='cuda')
    code = lib.d1_policy_head_sample(h.data_ptr(), n, 256, wh.data_ptr(), bh.data_ptr(),
                                     None if legal is None else legal.data_ptr(), seed, step, first_env,
                                     a.data_ptr(), lp.data_ptr(), v.data_ptr(), lg.data_ptr(), 0)
    assert code == 0
    torch.cuda.synchronize()
    return a, lp, v, lg


def test_head_matches_fp32_reference_and_sampler_matches_oracle(lib):
    g = torch.Generator().manual_seed(0)
    n = 65536
    h = torch.relu(torch.randn(n, 256, generator=g)).to(torch.bfloat16).cuda()
    wh = (torch.randn(13, 256, generator=g) / 16).to(torch.bfloat16).cuda()
    bh = torch.randn(13, generator=g).cuda()
    legal = torch.randint(0, 1 << 12, (n,), generator=g).to(torch.int32)
    legal = (legal | (1 << 8)).to(torch.int16).cuda()
    a, lp, v, lg = run_head(lib, h, wh, bh, legal, seed=1234, step=77, first_env=5)
    ref = h.float() @ wh.float().T + bh
    assert torch.allclose(lg, ref[:, :12], rtol=1e-4, atol=1e-4)
    assert torch.allclose(v, ref[:, 12], rtol=1e-4, atol=1e-4)
    ora, olp = oracle.sample_actions(lg.cpu().numpy(), legal.cpu().numpy().view(np.uint16), 1234, 77, 5)
    assert np.array_equal(a.cpu().numpy(), ora)
    assert np.allclose(lp.cpu().numpy(), olp, rtol=1e-5, atol=1e-5)
    bits = legal.cpu().numpy().view(np.uint16).astype(np.int64)
    assert ((bits >> a.cpu().numpy()) & 1).all(), 'sampled an illegal action'
    # log-prob agrees with torch's masked log-softmax
    masked = lg.masked_fill(((legal.to(torch.int32)[:, None] >> torch.arange(12, device='cuda')) & 1) == 0, -1e9)
    ref_lp = torch.log_softmax(masked, -1).gather(1, a[:, None])[:, 0]
    assert torch.allclose(lp, ref_lp, rtol=1e-5, atol=1e-5)


def test_sampling_frequencies_follow_the_softmax(lib):
    n = 1 << 18
    g = torch.Generator().manual_seed(1)
    wh = torch.zeros(13, 256, dtype=torch.bfloat16, device='cuda')
    bh = torch.tensor([0.0, 1.0, -1.0, 2.0, 0.5, -3.0, 0.0, 1.5, 0.2, -0.5, 1.0, 0.0, 0.0], device='cuda')
    h = torch.zeros(n, 256, dtype=torch.bfloat16, device='cuda')
    legal = torch.full((n,), 0b101111111011, dtype=torch.int16, device='cuda')  # action 2 and 10 illegal
    a, _, _, _ = run_head(lib, h, wh, bh, legal, seed=9, step=3)
    counts = torch.bincount(a, minlength=12).double().cpu() / n
    p = torch.softmax(bh[:12].masked_fill(torch.tensor([(0b101111111011 >> j) & 1 == 0 for j in range(12)],
                                                          device='cuda'), -1e9), -1).double().cpu()
    assert counts[2] == 0 and counts[10] == 0
    assert torch.allclose(counts, p, atol=4e-3)


@pytest.mark.parametrize('n', [65536, 1000])
def test_fused_layer2_head_matches_the_unfused_path_and_the_oracle(lib, n):
    """d1_gemm_head_sample (layer 2 + head + sampler in the GEMM epilogue): logits
    and value against the separate GEMM + head kernel (same bf16 activations,
    another summation order: 1e-5), draws against the oracle given its logits
    (exact), and the same action as the unfused path for nearly every row."""
    from d1.policy import Policy
    from d1.spec_env import SpecEnv
    env = SpecEnv(n, seed=2)
    pol = Policy(seed=3)
    out = {}
    for name, fn in (('fused', pol.act_fused), ('unfused', pol.act)):
        lg = torch.empty((n, 12), device='cuda')
        a, lp, v = fn(env.obs, env.legal, 11, 5, 7, logits=lg)
        out[name] = (a.clone(), lp.clone(), v.clone(), lg)
    torch.cuda.synchronize()
    fa, flp, fv, flg = out['fused']
    ua, ulp, uv, ulg = out['unfused']
    assert torch.allclose(flg, ulg, rtol=1e-5, atol=1e-5)
    assert torch.allclose(fv, uv, rtol=1e-5, atol=1e-5)
    legal = env.legal.cpu().numpy().view(np.uint16)
    ora, olp = oracle.sample_actions(flg.cpu().numpy(), legal, 11, 5, 7)
    assert np.array_equal(fa.cpu().numpy(), ora)
    assert np.allclose(flp.cpu().numpy(), olp, rtol=1e-5, atol=1e-5)
    assert (fa == ua).float().mean().item() > 0.999
    vals = torch.empty(n, device='cuda')
    pol.value(env.obs, out=vals)
    assert torch.equal(vals, uv)
    from d1 import gemm
    assert gemm.gemm_error() == 0


@pytest.mark.parametrize('n', [4096, 8192])
def test_decision_graph_replays_the_eager_loop(lib, n):
    """DecisionGraph (one captured decision with host copies and a device step
    counter; at 8,192 envs as two env ranges on two streams) reproduces the
    eager host-driven loop exactly."""
    from d1.policy import Policy
    from d1.rollout import DecisionGraph
    from d1.spec_env import SpecEnv
    pol = Policy(seed=4)
    eager, graphed = SpecEnv(n, seed=6), SpecEnv(n, seed=6)
    dg = DecisionGraph(graphed, pol, seed=9, step=0)
    assert len(dg.ranges) == (1 if n < 8192 else 2)
    # An eager call on more rows regrows the policy's cached activation buffers;
    # the freed blocks are then handed out again. The graph holds its own
    # buffers, so its replays below are unaffected.
    big = SpecEnv(2 * n, seed=1)
    pol.act(big.obs, big.legal, 1, 0)
    filler = torch.full((8 * n, pol.hidden), 3.0, dtype=torch.bfloat16, device='cuda')
    # DecisionGraph ran one warm-up decision with zero actions and step 0
    act = torch.zeros(n, dtype=torch.int64, device='cuda')
    eager.step(act)
    a, _, _ = pol.act(eager.obs, eager.legal, 9, 0)
    dg.h_act.copy_(dg.h_next)
    act = a.clone()
    for k in range(1, 4):
        dg.replay()
        torch.cuda.synchronize()
        eager.step(act)
        a, _, _ = pol.act(eager.obs, eager.legal, 9, k)
        torch.cuda.synchronize()
        assert torch.equal(dg.h_out, eager.out.cpu()), k
        assert torch.equal(dg.h_next, a.cpu()), k
        dg.h_act.copy_(dg.h_next)
        act = a.clone()


def test_rollout_on_two_streams_equals_one_stream():
    """Rollout(parts=2) steps two env ranges on their own streams (each range's
    env kernel overlapping the other's policy GEMMs); every buffer equals the
    one-stream rollout's bit for bit."""
    from d1.policy import Policy
    from d1.rollout import Rollout
    from d1.spec_env import SpecEnv
    B, T = 8192, 12
    one = Rollout(SpecEnv(B, seed=21), Policy(seed=4), T, seed=21, parts=1)
    two = Rollout(SpecEnv(B, seed=21), Policy(seed=4), T, seed=21, parts=2)
    assert one.parts == 1 and two.parts == 2
    for r in (one, two):
        r.collect()
        r.roll()
        r.collect()
    torch.cuda.synchronize()
    for name in ('obs', 'cobs', 'legal', 'actions', 'logp', 'values', 'out'):
        assert torch.equal(getattr(one, name), getattr(two, name)), name
    assert torch.equal(one.env.state, two.env.state)


@pytest.mark.parametrize('parts', [1, 2])
def test_graphed_collection_equals_eager_collection(parts):
    """Rollout(graphs=True): the first collect() runs eagerly and captures the
    rollout as one graph; the later ones replay it. Over three rollouts, with the
    policy's weights changed in place between them (as a PPO update does), every
    buffer, the env rows and the sampling step equal the eager rollout's bit
    for bit."""
    from d1.policy import Policy
    from d1.rollout import Rollout
    from d1.spec_env import SpecEnv
    B, T = 8192, 6
    eager = Rollout(SpecEnv(B, seed=23), Policy(seed=5), T, seed=23, parts=parts)
    graph = Rollout(SpecEnv(B, seed=23), Policy(seed=5), T, seed=23, parts=parts, graphs=True)
    for k in range(3):
        for r in (eager, graph):
            r.collect()
            r.roll()
            with torch.no_grad():  # a stand-in for an update: new weights, same buffers
                r.policy.params['w1'].mul_(0.9)
                r.policy.refresh()
        torch.cuda.synchronize()
        for name in ('obs', 'cobs', 'legal', 'actions', 'logp', 'values', 'out'):
            assert torch.equal(getattr(eager, name), getattr(graph, name)), (k, name)
        assert torch.equal(eager.env.state, graph.env.state), k
        assert eager.global_step == graph.global_step == (k + 1) * T
    assert graph._graph is not None


@pytest.mark.parametrize('n', [65536, 1000])
def test_policy_tail_matches_the_unfused_path_and_the_oracle(lib, n):
    """d1_policy_tail_sample (layer 2, head and draw in one persistent launch)
    against the layer-2 GEMM + head kernel on the same observations: logits and
    value within 1e-5 (another summation order), draws exact against the oracle
    given the kernel's own logits, the same action as the unfused path for
    nearly every row; the device-step form equals the host-step form, and
    value() equals act()'s value bit for bit."""
    from d1.policy import Policy
    from d1.spec_env import SpecEnv
    env = SpecEnv(n, seed=2)
    pol, plain = Policy(seed=3), Policy(seed=3, tail=False)
    assert pol.tail and not plain.tail
    lt = torch.empty((n, 12), device='cuda')
    lu = torch.empty((n, 12), device='cuda')
    ta, tlp, tv = pol.act(env.obs, env.legal, 11, 5, 7, logits=lt)
    ua, ulp, uv = plain.act(env.obs, env.legal, 11, 5, 7, logits=lu)
    torch.cuda.synchronize()
    assert torch.allclose(lt, lu, rtol=1e-5, atol=1e-5)
    assert torch.allclose(tv, uv, rtol=1e-5, atol=1e-5)
    legal = env.legal.cpu().numpy().view(np.uint16)
    ora, olp = oracle.sample_actions(lt.cpu().numpy(), legal, 11, 5, 7)
    assert np.array_equal(ta.cpu().numpy(), ora)
    assert np.allclose(tlp.cpu().numpy(), olp, rtol=1e-5, atol=1e-5)
    assert (ta == ua).float().mean().item() > 0.999
    da, dlp, dv = pol.act(env.obs, env.legal, 11, torch.tensor([5], dtype=torch.int64, device='cuda'), 7)
    vals = pol.value(env.obs)
    torch.cuda.synchronize()
    assert torch.equal(da, ta) and torch.equal(dlp, tlp) and torch.equal(dv, tv)
    assert torch.equal(vals, tv)
    assert lib.d1_policy_tail_error() == 0

"""Failure detection of the peer gradient exchange on one GPU, without a fault.

The trainer is given a two-rank exchange whose second "rank" is a second local
buffer that nobody ever flags: the all-reduce's bounded waits run out after a
short poll limit, the library records the error, the optimizer step leaves the
parameters, Adam moments and step count exactly as they were, and
PPO.update() raises instead of training on a stale gradient. The wait that
runs out is a device-side bounded poll on a flag that nothing sets; the kernel
returns normally and the context stays usable (a later single-GPU update runs).
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize('exchange', ['oneshot', 'twophase'])
def test_peer_wait_runs_out_reports_and_changes_nothing(exchange):
    from d1._lib import D1Error
    from d1.policy import Policy
    from d1.ppo import PPO
    from d1.rollout import Rollout
    from d1.spec_env import SpecEnv
    B, T, mb = 512, 8, 2048
    roll = Rollout(SpecEnv(B, seed=3), Policy(seed=0), T, seed=3)
    roll.collect()
    tr = PPO(roll.policy, roll, minibatch=mb, epochs=1, graph=False, peer_wait_limit=2000, exchange=exchange)
    tr.advantages()
    nbytes = tr.peer_bytes(world=2)
    bufs = [torch.zeros(nbytes // 4, dtype=torch.int32, device='cuda') for _ in range(2)]
    tr.peer_attach(2, 0, [b.data_ptr() for b in bufs])
    before = [t.clone() for t in (tr.policy.flat, tr.m, tr.v, tr.step_dev, tr.policy.bf16['w1'])]
    assert tr.lib.d1_peer_error() == 0
    with pytest.raises(D1Error, match='peer gradient exchange'):
        tr.update(torch.Generator(device='cuda').manual_seed(1))
    after = (tr.policy.flat, tr.m, tr.v, tr.step_dev, tr.policy.bf16['w1'])
    for b, a in zip(before, after):
        assert torch.equal(b, a)
    assert tr.lib.d1_peer_error() == 0  # the raise consumed the report
    # the context is still usable: the same trainer without the exchange steps normally
    tr.peer = None
    tr.update(torch.Generator(device='cuda').manual_seed(1))
    torch.cuda.synchronize()
    assert tr.step_dev.item() == T * B // mb
    assert not torch.equal(tr.policy.flat, before[0])

"""Multi-GPU PPO update with the gradient all-reduce through peer memory
(d1_ppo_step_peer, one-shot; d1_ppo_step_peer2, two-phase; d1_ppo_step_nvls,
the one-shot exchange read through an NVLink multicast address, where the
system provides one) against the same
update with NCCL's all-reduce (peer=False), on 2 GPUs as 2 processes: after every minibatch both give the
same parameters bit for bit (the mean of two values is one add and one divide
either way), and every rank holds the same parameters. Several minibatches in a
row exercise both halves of the exchange buffer; a captured epoch exercises the
path inside a CUDA graph. Skipped with fewer than 2 GPUs."""
import os

import pytest
import torch

pytestmark = pytest.mark.gpu


def _worker(rank, world, port, results):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, 'dcss-auto_b200'))
    import datetime
    import torch.distributed as dist
    from d1 import policy, ppo, rollout, spec_env
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group('nccl', rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device('cuda', rank))
    try:
        B, T, mb = 512, 16, 2048

        def make(peer, graph, exchange='oneshot'):
            env = spec_env.SpecEnv(B, seed=3, first_env=rank * B, device=f'cuda:{rank}')
            pol = policy.Policy(seed=0, device=f'cuda:{rank}')
            roll = rollout.Rollout(env, pol, T, seed=3)
            roll.collect()
            tr = ppo.PPO(pol, roll, minibatch=mb, epochs=2, group=dist.group.WORLD, peer=peer, graph=graph,
                         exchange=exchange)
            tr.advantages()
            return tr

        a, b, a2 = make(True, False), make(False, False), make(True, False, 'twophase')
        assert a2.peer['two_phase'] and not a.peer['two_phase']
        try:
            a3 = make(True, False, 'nvls')
        except Exception:  # no multicast object on this system (torch or the trainer refuses)
            a3 = None
        have = torch.tensor([0 if a3 is None else 1], device=f'cuda:{rank}')
        dist.all_reduce(have, op=dist.ReduceOp.MIN)
        nvls = bool(have.item())
        if a3 is not None and not nvls:
            a3.release()  # every rank uses the multicast path, or none does
        g = torch.Generator(device=f'cuda:{rank}').manual_seed(7)
        same, ranks_agree = True, True
        for k in range(5):
            idx = torch.randperm(a.total, device=f'cuda:{rank}', generator=g)[:mb]
            a.minibatch(idx)
            b.minibatch(idx)
            a2.minibatch(idx)
            if nvls:
                a3.minibatch(idx)
            torch.cuda.synchronize()
            same &= torch.equal(a.policy.flat, b.policy.flat) and torch.equal(a.grad, b.grad)
            same &= torch.equal(a2.policy.flat, b.policy.flat) and torch.equal(a2.grad, b.grad)
            if nvls:
                same &= torch.equal(a3.policy.flat, b.policy.flat) and torch.equal(a3.grad, b.grad)
            both = [torch.empty_like(a.policy.flat) for _ in range(world)]
            dist.all_gather(both, a.policy.flat)
            ranks_agree &= all(torch.equal(both[0], x) for x in both)
        # a captured epoch (the second update epoch replays a CUDA graph)
        c, d, c2 = make(True, True), make(False, True), make(True, True, 'twophase')
        gens = [torch.Generator(device=f'cuda:{rank}').manual_seed(9) for _ in range(3)]
        c.update(gens[0])
        d.update(gens[1])
        c2.update(gens[2])
        torch.cuda.synchronize()
        graphed_same = torch.equal(c.policy.flat, d.policy.flat) and torch.equal(c2.policy.flat, d.policy.flat)
        if nvls:
            c3 = make(True, True, 'nvls')
            c3.update(torch.Generator(device=f'cuda:{rank}').manual_seed(9))
            torch.cuda.synchronize()
            graphed_same &= torch.equal(c3.policy.flat, d.policy.flat)
        err = a.lib.d1_peer_error()
        for tr in (a, b, a2, c, d, c2) + ((a3, c3) if nvls else ()):
            tr.release()
        results[rank] = dict(same=bool(same), ranks_agree=bool(ranks_agree), graphed_same=bool(graphed_same),
                             err=int(err), nvls=nvls)
    finally:
        dist.destroy_process_group()


def test_peer_allreduce_update_equals_the_nccl_update():
    if torch.cuda.device_count() < 2:
        pytest.skip('needs 2 GPUs')
    import torch.multiprocessing as mp
    ctx = mp.get_context('spawn')
    manager = ctx.Manager()
    results = manager.dict()
    port = 29600 + os.getpid() % 200
    procs = [ctx.Process(target=_worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0, 0], codes
    for r in range(2):
        nv = results[r]['nvls']
        assert results[r] == dict(same=True, ranks_agree=True, graphed_same=True, err=0, nvls=nv), results[r]
    print('NVLS exchange tested:', results[0]['nvls'])

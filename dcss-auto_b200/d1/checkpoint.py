"""Checkpoint and exact resume of a PPO run (reference: gpu-d1/scripts/
run_ring_ablations.py:277-309, scripts/test_resume.py): the fp32 master weights,
Adam moments and step count, the live env state rows, the rollout's current
observation/legal slot and sampling step, the permutation's device epoch count,
and the permutation generator when the caller draws the order from one. A run
resumed from a checkpoint continues bit-for-bit like the uninterrupted run
(every kernel on the path is deterministic, including the advantage statistics
and the gradient-norm sum). The file is written atomically (temp + rename)."""
import os
import pathlib

import torch

FORMAT = 3


def job_of(trainer):
    r, env = trainer.rollout, trainer.rollout.env
    return dict(batch=env.batch, first_env=env.first_env, config=dict(env.values), horizon=r.T,
                sample_seed=r.sample_seed, minibatch=trainer.mb, epochs=trainer.epochs, lr=trainer.lr,
                clip=trainer.clip, vclip=trainer.vclip, vf_coef=trainer.vf_coef, ent_coef=trainer.ent_coef,
                max_grad_norm=trainer.max_grad_norm, gamma=trainer.gamma, lam=trainer.lam, eps=trainer.eps,
                betas=tuple(trainer.betas), gae_mode=trainer.gae_mode, params=trainer.policy.size,
                perm_seed=trainer.perm_seed)


def state_dict(trainer, generator=None, extra=None):
    r, env, p = trainer.rollout, trainer.rollout.env, trainer.policy
    r.join()  # the rollout's env-range streams
    return dict(format=FORMAT, job=job_of(trainer), params=p.flat.cpu(), adam_m=trainer.m.cpu(),
                adam_v=trainer.v.cpu(), adam_step=trainer.step_dev.cpu(), perm_epoch=trainer.perm_epoch.cpu(),
                env_state=env.state.cpu(),
                obs=r.obs.cpu(), cobs=r.cobs[0].cpu(), legal=r.legal[0].cpu(), global_step=r.global_step,
                generator=None if generator is None else generator.get_state(), extra=extra)


def load_state_dict(trainer, data, generator=None):
    if data.get('format') != FORMAT:
        raise ValueError('unknown checkpoint format')
    if data['job'] != job_of(trainer):
        raise ValueError('Resume job does not match checkpoint')
    r, env, p = trainer.rollout, trainer.rollout.env, trainer.policy
    r.join()  # a range stream still stepping must not race the overwrite below
    p.flat.copy_(data['params'])
    p.refresh()
    trainer.m.copy_(data['adam_m'])
    trainer.v.copy_(data['adam_v'])
    trainer.step_dev.copy_(data['adam_step'])
    trainer.perm_epoch.copy_(data['perm_epoch'])
    env.state.copy_(data['env_state'])
    r.obs.copy_(data['obs'])
    r.cobs[0].copy_(data['cobs'])
    r.legal[0].copy_(data['legal'])
    r.global_step = data['global_step']
    if generator is not None:
        if data['generator'] is None:
            raise ValueError('checkpoint holds no generator state')
        generator.set_state(data['generator'])
    return data['extra']


def save(path, trainer, generator=None, extra=None):
    path = pathlib.Path(path)
    tmp = path.with_name(path.name + '.tmp')
    torch.save(state_dict(trainer, generator, extra), tmp)
    os.replace(tmp, path)


def load(path, trainer, generator=None):
    return load_state_dict(trainer, torch.load(path, map_location='cpu', weights_only=False), generator)

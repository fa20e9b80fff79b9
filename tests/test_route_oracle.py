"""Route-cue task, host side: the reference's own build of the task
(oracle/_ref/learn_route.so, gpu-d1/src/learn.cu with the route-cue fast flags)
reproduces the committed golden digests, the corpus the tests use is the one
the digests were made on, and the reference's own route-cue known-answer
program (gpu-d1/src/test_route_cue.cu, built by `make -C oracle ref`) passes."""
import pathlib
import subprocess

import numpy as np
import pytest

import oracle

HERE = pathlib.Path(__file__).resolve().parent
GOLD = np.load(HERE / 'golden' / 'route_trajectories.npz')


def test_corpus_is_the_golden_one():
    from golden.make_golden_route import corpus, corpus_digest
    assert np.array_equal(corpus_digest(corpus()), GOLD['corpus_digest'])


@pytest.mark.skipif(oracle.route_library() is None, reason='oracle/_ref/learn_route.so not built here')
@pytest.mark.parametrize('name,steps', [('h40', 200), ('r1', 200), ('h8', 600)])
def test_reference_build_reproduces_golden(name, steps):
    from golden.make_golden_route import corpus, ref_digest
    from golden.schedule import random_actions
    batch, enemies, seed, total, heur, mf = map(int, GOLD[f'{name}_meta'])
    env = oracle.ReferenceRoute(batch, corpus(), enemies=enemies, seed=seed, map_filter=mf)
    assert np.array_equal(ref_digest(env), GOLD[f'{name}_init'])
    rand = random_actions(2000 + enemies + batch, total, batch, 9)
    for k in range(steps):
        env.step(env.heuristic().copy() if (heur and k % 2 == 0) else rand[k])
        assert np.array_equal(ref_digest(env), GOLD[f'{name}_digests'][k]), (name, k)


@pytest.mark.skipif(not (oracle.HERE / '_ref' / 'test_route_cue').exists(), reason='reference test not built here')
def test_reference_route_cue_program_passes():
    r = subprocess.run([str(oracle.HERE / '_ref' / 'test_route_cue')], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and 'PASS route cue' in r.stdout, r.stdout + r.stderr

"""Per-episode D4 camera augmentation (reference: gpu-d1/branches/
vision15-symmetry-v1/scripts/symmetry.py:19-102) against a torch restatement
of the reference's D4 tables laid out for the spec observation: cell-major
one-hot planes (element 8 * cell + channel) and the scalar coordinate pairs at
1800 + (4, 5), (9, 10), (15, 16), (26, 27). The restatement builds index /
scale / offset exactly as the reference does (float64 arithmetic, float32
tables) and applies obs.gather(index) * scale + offset in fp32; the kernel's
bf16 output must equal its bf16 rounding bit for bit."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DIRECTIONS = [(0, -1), (1, 0), (0, 1), (-1, 0), (1, -1), (1, 1), (-1, 1), (-1, -1), (0, 0)]
OBS = 1832


def xy(x, y, group):
    if group // 4:
        x = -x
    for _ in range(group % 4):
        x, y = -y, x
    return x, y


class ReferenceD4:
    """symmetry.py:19-57 with the spec observation's feature positions."""

    def __init__(self, device='cuda'):
        index = torch.arange(OBS).repeat(8, 1)
        scale = torch.ones(8, OBS)
        offset = torch.zeros(8, OBS)
        forward = torch.arange(12).repeat(8, 1)
        for g in range(8):
            for y in range(-7, 8):
                for x in range(-7, 8):
                    xx, yy = xy(x, y, g)
                    for c in range(8):
                        index[g, 8 * ((yy + 7) * 15 + xx + 7) + c] = 8 * ((y + 7) * 15 + x + 7) + c
            pairs = [(1804, 80., 70., 39.5, 34.5), (1809, 7., 7., 0., 0.), (1815, 80., 70., 0., 0.),
                     (1826, 7., 7., 0., 0.)]
            ex, ey = xy(1, 0, g), xy(0, 1, g)
            for j, sx, sy, cx, cy in pairs:
                units, center = [sx, sy], [cx, cy]
                for dst in range(2):
                    src = 0 if ex[dst] else 1
                    sign = ex[dst] if ex[dst] else ey[dst]
                    index[g, j + dst] = j + src
                    scale[g, j + dst] = sign * units[src] / units[dst]
                    offset[g, j + dst] = (center[dst] - sign * center[src]) / units[dst]
            for a, (x, y) in enumerate(DIRECTIONS[:8]):
                forward[g, a] = DIRECTIONS.index(xy(x, y, g))
        inverse = forward.argsort(1)
        self.index, self.scale, self.offset, self.forward, self.inverse = [
            t.to(device) for t in (index, scale, offset, forward, inverse)]

    def observation(self, obs, groups):
        g = groups.long()
        return (obs.float().gather(1, self.index[g]) * self.scale[g] + self.offset[g]).to(torch.bfloat16)

    def mask(self, mask, groups):
        return mask.gather(1, self.inverse[groups.long()])

    def to_world(self, actions, groups):
        return self.inverse[groups.long()].gather(1, actions[:, None]).squeeze(1)


def bits_to_mask(legal):
    bits = legal.to(torch.int64) & 0xffff
    return ((bits[:, None] >> torch.arange(12, device=bits.device)) & 1).float()


@pytest.fixture(scope='module')
def mods():
    from d1 import spec_env, symmetry
    from d1._lib import library
    return spec_env, symmetry, library()


def run(lib, obs, legal, groups, out=None, legal_out=None):
    out = torch.empty_like(obs) if out is None else out
    legal_out = torch.empty_like(legal) if legal_out is None else legal_out
    s = torch.cuda.current_stream().cuda_stream
    assert lib.d1_spec_d4_observe(obs.data_ptr(), legal.data_ptr(), groups.data_ptr(), obs.shape[0], out.data_ptr(),
                                  legal_out.data_ptr(), s) == 0
    return out, legal_out


def test_transform_matches_the_reference_tables(mods):
    spec_env, _, lib = mods
    ref = ReferenceD4()
    n = 1024
    env = spec_env.SpecEnv(n, seed=4)
    g = torch.Generator(device='cuda').manual_seed(3)
    for k in range(6):
        env.step(torch.randint(0, 12, (n,), device='cuda', generator=g))
    groups = (torch.arange(n, device='cuda') % 8).to(torch.uint8)
    got, legal = run(lib, env.obs, env.legal, groups)
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int16), ref.observation(env.obs, groups).view(torch.int16))
    assert torch.equal(bits_to_mask(legal), ref.mask(bits_to_mask(env.legal), groups))
    assert torch.equal(legal.to(torch.int64) & ~0xff, env.legal.to(torch.int64) & ~0xff)
    # arbitrary values in every element (the coordinate pairs with non-trivial inputs)
    rnd = (torch.randn(n, OBS, device='cuda', generator=g) * 3).to(torch.bfloat16)
    legal_rnd = torch.randint(0, 1 << 12, (n,), device='cuda', generator=g).to(torch.int16)
    got, legal = run(lib, rnd, legal_rnd, groups)
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int16), ref.observation(rnd, groups).view(torch.int16))
    assert torch.equal(bits_to_mask(legal), ref.mask(bits_to_mask(legal_rnd), groups))


def test_in_place_and_actions(mods):
    _, _, lib = mods
    ref = ReferenceD4()
    n = 4096
    g = torch.Generator(device='cuda').manual_seed(8)
    obs = (torch.randn(n, OBS, device='cuda', generator=g)).to(torch.bfloat16)
    legal = torch.randint(0, 1 << 12, (n,), device='cuda', generator=g).to(torch.int16)
    groups = torch.randint(0, 8, (n,), device='cuda', generator=g).to(torch.uint8)
    want, want_legal = run(lib, obs, legal, groups)
    inplace, inplace_legal = obs.clone(), legal.clone()
    run(lib, inplace, inplace_legal, groups, out=inplace, legal_out=inplace_legal)
    torch.cuda.synchronize()
    assert torch.equal(inplace.view(torch.int16), want.view(torch.int16)) and torch.equal(inplace_legal, want_legal)
    acts = torch.randint(0, 12, (n,), device='cuda', generator=g)
    world = torch.empty_like(acts)
    assert lib.d1_spec_d4_actions(acts.data_ptr(), groups.data_ptr(), n, world.data_ptr(),
                                  torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    assert torch.equal(world, ref.to_world(acts, groups))
    # the identity group changes nothing
    ident = torch.zeros(n, dtype=torch.uint8, device='cuda')
    same, same_legal = run(lib, obs, legal, ident)
    torch.cuda.synchronize()
    assert torch.equal(same.view(torch.int16), obs.view(torch.int16)) and torch.equal(same_legal, legal)


def test_episode_wrapper(mods):
    spec_env, symmetry, _ = mods
    ref = ReferenceD4()
    n = 512
    base = spec_env.SpecEnv(n, seed=6)
    wrap = symmetry.EpisodeSymmetry(base, seed=11)
    counts = torch.bincount(wrap.groups.long(), minlength=8)
    assert (counts > 0).all()
    g = torch.Generator(device='cuda').manual_seed(2)
    twin = spec_env.SpecEnv(n, seed=6)  # steps on the world actions directly
    ended_any = False
    for k in range(120):
        cam = torch.randint(0, 12, (n,), device='cuda', generator=g)
        before = wrap.groups.clone()
        world = ref.to_world(cam, before)
        obs, out = wrap.step(cam)
        twin.step(world.contiguous())
        torch.cuda.synchronize()
        assert torch.equal(base.compact(), twin.compact())
        ended = out[:, 1] > 0
        ended_any |= bool(ended.any())
        assert torch.equal(wrap.groups[~ended], before[~ended])
        assert torch.equal(obs.view(torch.int16), ref.observation(base.obs, wrap.groups).view(torch.int16))
        assert torch.equal(bits_to_mask(wrap.legal), ref.mask(base.legal_mask(), wrap.groups))
    assert ended_any
    snap = wrap.snapshot()
    other = symmetry.EpisodeSymmetry(spec_env.SpecEnv(n, seed=6), seed=11)
    other.base.state.copy_(base.state)
    other.base.obs.copy_(base.obs)
    other.base.legal.copy_(base.legal)
    other.restore(snap)
    torch.cuda.synchronize()
    assert torch.equal(other.obs.view(torch.int16), wrap.obs.view(torch.int16))

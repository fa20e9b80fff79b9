"""Per-episode D4 camera augmentation of the BASELINE task (the EpisodeSymmetry
wrapper of gpu-d1/branches/vision15-symmetry-v1/scripts/symmetry.py:59-102).

Every env sees its world through one of the 8 D4 elements, fixed for the
episode and redrawn when the episode ends. The wrapped env keeps stepping in
world coordinates: camera actions are mapped to the world (d1_spec_d4_actions),
and after every step the world observation and legal bits are transformed into
the camera frame (d1_spec_d4_observe). Group draws come from Philox purpose 4
keyed by (global env id, seed, draw index) instead of torch's generator, so a
shard of a multi-GPU run draws the same groups as the whole batch would.
Attributes other than obs, legal and legal_mask pass through to the wrapped env."""
import torch

from ._lib import check, library, launch_stream


class EpisodeSymmetry:
    def __init__(self, base, seed):
        if base.obs is None:
            raise ValueError('the wrapped env must write observations')
        self.base, self.seed = base, seed
        self.lib = library()
        dev, n = base.device, base.batch
        self.groups = torch.empty(n, dtype=torch.uint8, device=dev)
        self.obs = torch.empty_like(base.obs)
        self.legal = torch.empty_like(base.legal)
        self._world = torch.empty(n, dtype=torch.int64, device=dev)
        self.draws = 0
        self._draw(None, None)
        self.refresh()

    def __getattr__(self, name):
        return getattr(self.base, name)

    def _stream(self):
        return launch_stream(self.base.device)

    def _draw(self, out, active):
        p = lambda t: None if t is None else t.data_ptr()
        check(self.lib.d1_spec_d4_draw(self.groups.data_ptr(), self.base.batch, p(out),
                                       0 if out is None else out.shape[1], p(active), self.seed, self.draws,
                                       self.base.first_env, self._stream()), 'd1_spec_d4_draw')
        self.draws += 1

    def refresh(self):
        check(self.lib.d1_spec_d4_observe(self.base.obs.data_ptr(), self.base.legal.data_ptr(), self.groups.data_ptr(),
                                          self.base.batch, self.obs.data_ptr(), self.legal.data_ptr(), self._stream()),
              'd1_spec_d4_observe')

    def legal_mask(self):
        """Camera-frame legal actions as a float [n, 12] mask."""
        bits = self.legal.to(torch.int64) & 0xffff
        return ((bits[:, None] >> torch.arange(12, device=bits.device)) & 1).float()

    def to_world(self, actions):
        check(self.lib.d1_spec_d4_actions(actions.data_ptr(), self.groups.data_ptr(), self.base.batch,
                                          self._world.data_ptr(), self._stream()), 'd1_spec_d4_actions')
        return self._world

    def reset(self, seed):
        self.base.reset(seed)
        self._draw(None, None)
        self.refresh()
        return self.obs

    def step(self, actions, active=None):
        assert actions.dtype == torch.int64 and actions.is_contiguous()
        world = self.to_world(actions)
        _, out = self.base.step(world) if active is None else self.base.step(world, active=active)
        self._draw(out, active)
        self.refresh()
        return self.obs, out

    def snapshot(self):
        return dict(groups=self.groups.cpu(), draws=self.draws)

    def restore(self, state):
        self.groups.copy_(state['groups'].to(self.base.device))
        self.draws = int(state['draws'])
        self.refresh()

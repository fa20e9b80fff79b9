"""Fixed observation history (gpu-d1/branches/vision15-centered-map-v1/scripts/
frame_stack.py:5-32): `frames` observations per env, oldest first, duplicated at
reset and refilled with the new observation when an episode ends. One kernel
(d1_frame_stack) shifts every env's history in place and appends the new frame.
Wraps either task's env; attributes other than obs pass through to it."""
import torch

from ._lib import check, library, launch_stream


class FrameStack:
    def __init__(self, base, frames=4):
        if frames < 2:
            raise ValueError('FrameStack requires at least two frames')
        if base.obs is None:
            raise ValueError('the wrapped env must write observations')
        self.base, self.frames = base, frames
        self.width = base.obs.shape[1]
        self.row_bytes = self.width * base.obs.element_size()
        self.obs = torch.empty((base.batch, frames * self.width), dtype=base.obs.dtype, device=base.obs.device)
        self._fill()

    def __getattr__(self, name):
        return getattr(self.base, name)

    def _stream(self):
        return launch_stream(self.obs.device)

    def _fill(self):
        check(library().d1_frame_stack(self.obs.data_ptr(), self.base.obs.data_ptr(), self.row_bytes, self.frames,
                                       self.base.batch, None, 0, None, self._stream()), 'd1_frame_stack')

    def reset(self, seed):
        self.base.reset(seed)
        self._fill()
        return self.obs

    def step(self, actions, active=None):
        _, out = self.base.step(actions) if active is None else self.base.step(actions, active=active)
        check(library().d1_frame_stack(self.obs.data_ptr(), self.base.obs.data_ptr(), self.row_bytes, self.frames,
                                       self.base.batch, out.data_ptr(), out.shape[1],
                                       None if active is None else active.data_ptr(), self._stream()),
              'd1_frame_stack')
        return self.obs, out

    def restore_raw_observation(self):
        self.base.obs.copy_(self.obs[:, -self.width:])

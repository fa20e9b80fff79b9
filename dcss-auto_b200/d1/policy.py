"""MLP policy of BASELINE config 1: obs 1832 -> 256 -> 256 (ReLU) -> 12 logits + value.

Parameters live in one flat fp32 buffer (the optimizer's master copy and the
unit of the multi-GPU gradient all-reduce), laid out as
W1 [256, 1832], b1 [256], W2 [256, 256], Wh [13, 256], bh [13], b2 [256];
Wh rows 0-11 are the action logits and row 12 the value. bf16 copies of W1,
W2, W2^T and Wh feed the tensor-core GEMMs and the head kernel. Initialisation:
N(0, 1/fan_in) weights, zero biases, from a torch CPU generator seed.
"""
import torch

from ._lib import check, library, launch_stream, resolve_device
from . import gemm

OBS, HID, NACT = 1832, 256, 12
NOUT = NACT + 1


def layout(obs=OBS, hidden=HID):
    shapes = [('w1', (hidden, obs)), ('b1', (hidden,)), ('w2', (hidden, hidden)), ('wh', (NOUT, hidden)),
              ('bh', (NOUT,)), ('b2', (hidden,))]
    out, off = {}, 0
    for name, shape in shapes:
        n = 1
        for d in shape:
            n *= d
        out[name] = (off, shape)
        off += n
    return out, off


class Policy:
    def __init__(self, device='cuda', seed=0, obs=OBS, hidden=HID, tail=True):
        self.device = resolve_device(device)
        # act() and value() run layer 2, the head and the draw as one fused kernel
        self.tail = tail and hidden == HID
        self.obs, self.hidden = obs, hidden
        self.layout, self.size = layout(obs, hidden)
        self.flat = torch.zeros(self.size, device=self.device)
        self.params = {k: self.flat[o:o + torch.Size(s).numel()].view(s) for k, (o, s) in self.layout.items()}
        g = torch.Generator(device='cpu').manual_seed(seed)
        for k in ('w1', 'w2', 'wh'):
            fan_out, fan_in = self.params[k].shape
            self.params[k].copy_(torch.randn(fan_out, fan_in, generator=g) / fan_in ** 0.5)
        self.bf16 = {
            'w1': torch.empty((hidden, obs), dtype=torch.bfloat16, device=self.device),
            'w2': torch.empty((hidden, hidden), dtype=torch.bfloat16, device=self.device),
            'w2t': torch.empty((hidden, hidden), dtype=torch.bfloat16, device=self.device),
            'wh': torch.empty((NOUT, hidden), dtype=torch.bfloat16, device=self.device),
        }
        self.lib = library()
        self.refresh()

    def refresh(self):
        """Re-derive the bf16 compute copies from the fp32 masters."""
        self.bf16['w1'].copy_(self.params['w1'])
        self.bf16['w2'].copy_(self.params['w2'])
        self.bf16['w2t'].copy_(self.params['w2'].T)
        self.bf16['wh'].copy_(self.params['wh'])

    def hidden_layers(self, obs, h1=None, h1t=None, h2=None):
        """(h1, h2) bf16 activations for obs bf16 [n, 1832]; h1t (feature-major)
        is written too when given (the backward pass needs it)."""
        n = obs.shape[0]
        if h1 is None:
            h1 = torch.empty((n, self.hidden), dtype=torch.bfloat16, device=self.device)
        gemm.gemm(obs, self.bf16['w1'], bias=self.params['b1'], relu=True, out=h1, out_t=h1t)
        if h2 is None:
            h2 = torch.empty((n, self.hidden), dtype=torch.bfloat16, device=self.device)
        gemm.gemm(h1, self.bf16['w2'], bias=self.params['b2'], relu=True, out=h2)
        return h1, h2

    def head(self, h2, legal, seed, step, first_env, action, logp, value, logits=None):
        """`step` is an int, or an int64 device tensor of one element read when
        the kernel runs (for CUDA graphs that advance it themselves)."""
        stream = launch_stream(self.device)
        n = h2.shape[0]
        if isinstance(step, torch.Tensor):
            check(self.lib.d1_policy_head_sample_dev(
                h2.data_ptr(), n, self.hidden, self.bf16['wh'].data_ptr(), self.params['bh'].data_ptr(),
                None if legal is None else legal.data_ptr(), seed, step.data_ptr(), first_env,
                None if action is None else action.data_ptr(), None if logp is None else logp.data_ptr(),
                None if value is None else value.data_ptr(), None if logits is None else logits.data_ptr(), stream),
                'd1_policy_head_sample_dev')
            return
        check(self.lib.d1_policy_head_sample(h2.data_ptr(), n, self.hidden, self.bf16['wh'].data_ptr(),
                                             self.params['bh'].data_ptr(),
                                             None if legal is None else legal.data_ptr(), seed, step, first_env,
                                             None if action is None else action.data_ptr(),
                                             None if logp is None else logp.data_ptr(),
                                             None if value is None else value.data_ptr(),
                                             None if logits is None else logits.data_ptr(), stream),
              'd1_policy_head_sample')

    def _h1(self, obs):
        h1 = self._h1_buffer(obs.shape[0])
        gemm.gemm(obs, self.bf16['w1'], bias=self.params['b1'], relu=True, out=h1)
        return h1

    def fused_head(self, h1, legal, seed, step, first_env, action, logp, value, logits=None):
        """Layer 2 with the head and sampler in its epilogue (h2 is never stored)."""
        stream = launch_stream(self.device)
        ptr = lambda t: None if t is None else t.data_ptr()
        check(self.lib.d1_gemm_head_sample(h1.data_ptr(), h1.stride(0), self.bf16['w2'].data_ptr(), self.hidden,
                                           h1.shape[0], self.hidden, self.params['b2'].data_ptr(),
                                           self.bf16['wh'].data_ptr(), self.params['bh'].data_ptr(), ptr(legal),
                                           seed, step, first_env, ptr(action), ptr(logp), ptr(value), ptr(logits),
                                           stream), 'd1_gemm_head_sample')

    def act(self, obs, legal, seed, step, first_env=0, action=None, logp=None, value=None, logits=None, part=0,
            h1=None, h2=None):
        """Forward + sample: layer 1 on the tcgen05 pair GEMM, then layer 2, the
        head and the draw in one persistent kernel (d1_policy_tail_sample; with
        tail=False: the layer-2 GEMM and the head + sampler kernel). Writes into
        the given buffers (allocated if None). `part` selects the policy's
        cached activation buffers, so that parts of a batch can run on
        different streams at the same time; a caller that captures this call in
        a CUDA graph passes its own h1/h2 ([n, hidden] bf16) instead, because the
        cached buffers are reallocated when a later call needs more rows."""
        n = obs.shape[0]
        h1 = self._h1_buffer(n, part) if h1 is None else h1
        if action is None:
            action = torch.empty(n, dtype=torch.int64, device=self.device)
        if logp is None:
            logp = torch.empty(n, device=self.device)
        if value is None:
            value = torch.empty(n, device=self.device)
        if self.tail:
            gemm.gemm(obs, self.bf16['w1'], bias=self.params['b1'], relu=True, out=h1)
            self.tail_sample(h1, legal, seed, step, first_env, action, logp, value, logits)
        else:
            h2 = self._h2_buffer(n, part) if h2 is None else h2
            self.hidden_layers(obs, h1=h1, h2=h2)
            self.head(h2, legal, seed, step, first_env, action, logp, value, logits)
        return action, logp, value

    def tail_sample(self, h1, legal, seed, step, first_env, action, logp, value, logits=None):
        """Layer 2 + head + draw from h1 (d1_policy_tail_sample). `step` is an int
        or an int64 device tensor of one element read when the kernel runs;
        action None: value (and logits) only."""
        dev_step = isinstance(step, torch.Tensor)
        ptr = lambda t: None if t is None else t.data_ptr()
        check(self.lib.d1_policy_tail_sample(h1.data_ptr(), h1.shape[0], h1.stride(0), self.bf16['w2'].data_ptr(),
                                             self.params['b2'].data_ptr(), self.bf16['wh'].data_ptr(),
                                             self.params['bh'].data_ptr(), ptr(legal), seed,
                                             0 if dev_step else step, step.data_ptr() if dev_step else None,
                                             first_env, ptr(action), ptr(logp), value.data_ptr(), ptr(logits),
                                             launch_stream(self.device)), 'd1_policy_tail_sample')

    def act_fused(self, obs, legal, seed, step, first_env=0, action=None, logp=None, value=None, logits=None):
        """The same draw with layer 2, the head and the sampler in one GEMM
        (d1_gemm_head_sample). Measured slower than act() on B200 at 65,536
        rows: the 13 x 256 head FMAs per row then run on the GEMM's 8 epilogue
        warps only."""
        n = obs.shape[0]
        if action is None:
            action = torch.empty(n, dtype=torch.int64, device=self.device)
        if logp is None:
            logp = torch.empty(n, device=self.device)
        if value is None:
            value = torch.empty(n, device=self.device)
        self.fused_head(self._h1(obs), legal, seed, step, first_env, action, logp, value, logits)
        return action, logp, value

    def _buffer(self, kind, n, part):
        bufs = self.__dict__.setdefault('_act_bufs', {})
        b = bufs.get((kind, part))
        if b is None or b.shape[0] < n:
            b = bufs[(kind, part)] = torch.empty((n, self.hidden), dtype=torch.bfloat16, device=self.device)
        return b[:n]

    def _h2_buffer(self, n, part=0):
        return self._buffer('h2', n, part)

    def _h1_buffer(self, n, part=0):
        return self._buffer('h1', n, part)

    def value(self, obs, out=None):
        """The value head alone (the rollout's bootstrap), by the same kernels
        as act() so that both agree bit for bit."""
        n = obs.shape[0]
        value = torch.empty(n, device=self.device) if out is None else out
        if self.tail:
            h1 = self._h1_buffer(n)
            gemm.gemm(obs, self.bf16['w1'], bias=self.params['b1'], relu=True, out=h1)
            self.tail_sample(h1, None, 0, 0, 0, None, None, value)
            return value
        _, h2 = self.hidden_layers(obs, h1=self._h1_buffer(n), h2=self._h2_buffer(n))
        self.head(h2, None, 0, 0, 0, None, None, value)
        return value

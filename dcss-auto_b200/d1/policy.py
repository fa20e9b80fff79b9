"""MLP policy of BASELINE config 1: obs 1832 -> 256 -> 256 (ReLU) -> 12 logits + value.

Parameters live in one flat fp32 buffer (the optimizer's master copy and the
unit of the multi-GPU gradient all-reduce), laid out as
W1 [256, 1832], b1 [256], W2 [256, 256], Wh [13, 256], bh [13], b2 [256];
Wh rows 0-11 are the action logits and row 12 the value. bf16 copies of W1,
W2, W2^T and Wh feed the tensor-core GEMMs and the head kernel. Initialisation:
N(0, 1/fan_in) weights, zero biases, from a torch CPU generator seed.
"""
import torch

from ._lib import check, library
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
    def __init__(self, device='cuda', seed=0, obs=OBS, hidden=HID):
        self.device = torch.device(device)
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
        stream = torch.cuda.current_stream(self.device).cuda_stream
        n = h2.shape[0]
        check(self.lib.d1_policy_head_sample(h2.data_ptr(), n, self.hidden, self.bf16['wh'].data_ptr(),
                                             self.params['bh'].data_ptr(),
                                             None if legal is None else legal.data_ptr(), seed, step, first_env,
                                             None if action is None else action.data_ptr(),
                                             None if logp is None else logp.data_ptr(),
                                             None if value is None else value.data_ptr(),
                                             None if logits is None else logits.data_ptr(), stream),
              'd1_policy_head_sample')

    def act(self, obs, legal, seed, step, first_env=0, action=None, logp=None, value=None, logits=None):
        """Forward + sample. Writes into the given buffers (allocated if None)."""
        n = obs.shape[0]
        _, h2 = self.hidden_layers(obs)
        if action is None:
            action = torch.empty(n, dtype=torch.int64, device=self.device)
        if logp is None:
            logp = torch.empty(n, device=self.device)
        if value is None:
            value = torch.empty(n, device=self.device)
        self.head(h2, legal, seed, step, first_env, action, logp, value, logits)
        return action, logp, value

    def value(self, obs, out=None):
        n = obs.shape[0]
        _, h2 = self.hidden_layers(obs)
        value = torch.empty(n, device=self.device) if out is None else out
        self.head(h2, None, 0, 0, 0, None, None, value)
        return value

"""MLP policy of BASELINE config 1: obs 1832 -> 256 -> 256 (ReLU) -> 12 logits + value.

Weights are fp32 masters with bf16 copies for the tensor-core GEMMs, initialised
N(0, 1/fan_in) from a torch seed. The head and the masked categorical sampler are
the fused d1_policy_head_sample kernel.
"""
import torch

from ._lib import check, library
from . import gemm

OBS, HID, NACT = 1832, 256, 12


class Policy:
    def __init__(self, device='cuda', seed=0, obs=OBS, hidden=HID):
        self.device = torch.device(device)
        g = torch.Generator(device='cpu').manual_seed(seed)

        def w(fan_out, fan_in):
            return (torch.randn(fan_out, fan_in, generator=g) / fan_in ** 0.5).to(self.device)
        self.params = {
            'w1': w(hidden, obs), 'b1': torch.zeros(hidden, device=self.device),
            'w2': w(hidden, hidden), 'b2': torch.zeros(hidden, device=self.device),
            'wh': w(NACT + 1, hidden), 'bh': torch.zeros(NACT + 1, device=self.device),
        }
        self.obs, self.hidden = obs, hidden
        self.lib = library()
        self.refresh()

    def refresh(self):
        """Re-derive the bf16 compute copies from the fp32 masters."""
        self.bf16 = {k: v.to(torch.bfloat16).contiguous() for k, v in self.params.items() if k.startswith('w')}

    def hidden_layers(self, obs, out=None):
        """(h1, h2) bf16 activations for obs bf16 [n, 1832]."""
        h1 = gemm.linear_relu(obs, self.bf16['w1'], self.params['b1'])
        h2 = gemm.linear_relu(h1, self.bf16['w2'], self.params['b2'])
        return h1, h2

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
        stream = torch.cuda.current_stream(self.device).cuda_stream
        check(self.lib.d1_policy_head_sample(h2.data_ptr(), n, self.hidden, self.bf16['wh'].data_ptr(),
                                             self.params['bh'].data_ptr(), legal.data_ptr(), seed, step, first_env,
                                             action.data_ptr(), logp.data_ptr(), value.data_ptr(),
                                             None if logits is None else logits.data_ptr(), stream),
              'd1_policy_head_sample')
        return action, logp, value

    def value(self, obs, out=None):
        n = obs.shape[0]
        _, h2 = self.hidden_layers(obs)
        value = torch.empty(n, device=self.device) if out is None else out
        stream = torch.cuda.current_stream(self.device).cuda_stream
        check(self.lib.d1_policy_head_sample(h2.data_ptr(), n, self.hidden, self.bf16['wh'].data_ptr(),
                                             self.params['bh'].data_ptr(), None, 0, 0, 0, None, None,
                                             value.data_ptr(), None, stream), 'd1_policy_head_sample')
        return value

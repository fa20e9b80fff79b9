"""Centered-map conv policy with the autoregressive verb x target head
(BASELINE config 3).

    crop 63x63 (u16 codes -> 10 channels)
      conv 3x3/2 10->32, ReLU; conv 3x3/2 32->64, ReLU; conv 3x3/2 64->64, ReLU
      (tcgen05 implicit GEMM, d1_conv_layer)           -> 7x7x64 = 3136 (NHWC)
      FC 3136->512, ReLU                               (tcgen05 GEMM, d1_gemm)
      head 512->80: verb logits 12, value 1, direction pre-activation 64
                                                       (tcgen05 GEMM, fp32 out)
      verb ~ 12-way, target ~ 9-way | verb via tanh(pre + cond_verb) . W_t + b_t
                                                       (d1_ar_head_sample)

The reference builds the recentred map with an encode kernel and runs torch
Conv2d/Linear layers (gpu-d1/branches/vision15-centered-map-v1/src/
fast_maps.cu:4-17, scripts/tactical_models.py:11-62); its autoregressive head is
ActionDistribution + the type-embedding direction MLP
(autoregressive-actions-v1/scripts/tactical_models.py:8-48). Sizes follow
BASELINE config 3 (63x63x10 crop, 32-64-64 convs, FC 512, 12 verbs x 9 targets).

Weights are fp32 masters initialised N(0, 1/fan_in) (biases N(0, 0.01^2) so the
bias paths are exercised) from a torch CPU generator; bf16 copies in operand
layout feed the kernels. Activations between conv layers go through buffers
sized for `chunk` envs at a time (64 KB + 32 KB per env); 16,384 keeps each
launch many waves deep, which measured faster than L2-sized chunks.
"""
import torch

from ._lib import check, library, launch_stream, resolve_device
from . import gemm as G

CROP, CROP_PITCH, FC_IN, WIDTH, HEAD, PRE, NV, NT = 63, 64, 3136, 512, 80, 64, 12, 9
# joint action -> spec env action (MOVE t, ATTACK t / nearest, WAIT, REST, DESCEND)
ENV_ACTION = [0, 1, 2, 3, 4, 5, 6, 7, -1, 0, 1, 2, 3, 4, 5, 6, 7, 10, 8, 9, 11, -1, -1, -1, -1, -1, -1, -1]
CONV = [(10, 32), (32, 64), (64, 64)]


class ConvPolicy:
    def __init__(self, device='cuda', seed=0, chunk=16384):
        self.device = resolve_device(device)
        self.lib = library()
        self.chunk = chunk
        g = torch.Generator(device='cpu').manual_seed(seed)

        def w(shape, fan_in):
            return (torch.randn(shape, generator=g) / fan_in ** 0.5).to(self.device)

        def b(k):
            return (0.01 * torch.randn(k, generator=g)).to(self.device)

        p = {}
        for i, (cin, cout) in enumerate(CONV, 1):
            p[f'c{i}w'] = w((cout, cin, 3, 3), cin * 9)
            p[f'c{i}b'] = b(cout)
        p['fcw'], p['fcb'] = w((WIDTH, FC_IN), FC_IN), b(WIDTH)
        hw = w((HEAD, WIDTH), WIDTH)
        hw[NV + 1 + PRE:] = 0
        hb = b(HEAD)
        hb[NV + 1 + PRE:] = 0
        p['hw'], p['hb'] = hw, hb
        p['emb'] = (0.1 * torch.randn(2, 16, generator=g)).to(self.device)   # MOVE, ATTACK type embeddings
        p['wemb'] = w((PRE, 16), WIDTH + 16)                                  # their first-layer columns
        p['wt'], p['bt'] = w((NT, PRE), PRE), b(NT)
        self.params = p
        self.packed = {i: torch.empty(self.lib.d1_conv_weight_bytes(i), dtype=torch.uint8, device=self.device)
                       for i in (1, 2, 3)}
        self.bf16 = {}
        self.refresh()

    def refresh(self):
        """Re-derive the kernel copies (operand-layout bf16 conv weights, bf16 FC
        and head weights, the type-embedding terms) from the fp32 masters."""
        s = launch_stream(self.device)
        for i in (1, 2, 3):
            wt = self.params[f'c{i}w'].contiguous()
            check(self.lib.d1_conv_pack_weights(i, wt.data_ptr(), self.packed[i].data_ptr(), s),
                  'd1_conv_pack_weights')
        self.bf16['fcw'] = self.params['fcw'].to(torch.bfloat16)
        self.bf16['hw'] = self.params['hw'].to(torch.bfloat16)
        self.cond = (self.params['emb'] @ self.params['wemb'].T).contiguous()

    def buffers(self, n):
        """Device buffers for a batch of n envs (allocated once by the caller)."""
        dev, c = self.device, min(self.chunk, n)
        return {
            'crop': torch.empty((n, CROP, CROP_PITCH), dtype=torch.int16, device=dev),
            'a1': torch.empty(c * self.lib.d1_conv_in_bytes(2), dtype=torch.uint8, device=dev),
            'a2': torch.empty(c * self.lib.d1_conv_in_bytes(3), dtype=torch.uint8, device=dev),
            'fc_in': torch.empty((n, FC_IN), dtype=torch.bfloat16, device=dev),
            'h': torch.empty((n, WIDTH), dtype=torch.bfloat16, device=dev),
            'hb': torch.empty((n, HEAD), dtype=torch.float32, device=dev),
        }

    def encode(self, state, n, buf, g=0):
        """Crops of n env state rows (u16 codes) under D4 element g."""
        s = launch_stream(self.device)
        check(self.lib.d1_spec_crop(state.data_ptr(), n, g, buf['crop'].data_ptr(), s), 'd1_spec_crop')

    def features(self, buf, n):
        """conv stack + FC + head GEMM: fills buf['fc_in'], buf['h'], buf['hb']."""
        lib, s = self.lib, launch_stream(self.device)
        p, pk = self.params, self.packed
        crop, fc_in = buf['crop'], buf['fc_in']
        for c0 in range(0, n, self.chunk):
            m = min(self.chunk, n - c0)
            check(lib.d1_conv_layer(1, crop[c0].data_ptr(), m, pk[1].data_ptr(), p['c1b'].data_ptr(),
                                    buf['a1'].data_ptr(), s), 'd1_conv_layer 1')
            check(lib.d1_conv_layer(2, buf['a1'].data_ptr(), m, pk[2].data_ptr(), p['c2b'].data_ptr(),
                                    buf['a2'].data_ptr(), s), 'd1_conv_layer 2')
            check(lib.d1_conv_layer(3, buf['a2'].data_ptr(), m, pk[3].data_ptr(), p['c3b'].data_ptr(),
                                    fc_in[c0].data_ptr(), s), 'd1_conv_layer 3')
        G.gemm(fc_in[:n], self.bf16['fcw'], bias=p['fcb'], relu=True, out=buf['h'][:n])
        G.gemm(buf['h'][:n], self.bf16['hw'], bias=p['hb'], out_f32=buf['hb'][:n])

    def act(self, state, legal, n, buf, seed, step, first_env=0, out=None, g=0, debug=False):
        """Sample joint actions for n envs from their state rows: returns a dict of
        device tensors joint, env_action (int64), logp, value (fp32) and, with
        debug=True, entropy, verb_logits [n, 12], target_logits [n, 2, 9]."""
        self.encode(state, n, buf, g)
        self.features(buf, n)
        return self.act_from_features(legal, n, buf, seed, step, first_env, out, debug)

    def act_from_features(self, legal, n, buf, seed, step, first_env=0, out=None, debug=False):
        """The autoregressive head on buf['hb'] (filled by features())."""
        dev = self.device
        if out is None:
            out = {k: torch.empty(n, dtype=torch.int64, device=dev) for k in ('joint', 'env_action')}
            out.update({k: torch.empty(n, device=dev) for k in ('logp', 'value')})
            if debug:
                out['entropy'] = torch.empty(n, device=dev)
                out['verb_logits'] = torch.empty((n, NV), device=dev)
                out['target_logits'] = torch.empty((n, 2, NT), device=dev)
        s = launch_stream(dev)
        ptr = lambda k: out[k].data_ptr() if k in out else None
        p = self.params
        check(self.lib.d1_ar_head_sample(buf['hb'].data_ptr(), n, self.cond.data_ptr(), p['wt'].data_ptr(),
                                         p['bt'].data_ptr(), legal.data_ptr(), seed, step, first_env, ptr('joint'),
                                         ptr('env_action'), ptr('logp'), ptr('value'), ptr('entropy'),
                                         ptr('verb_logits'), ptr('target_logits'), s), 'd1_ar_head_sample')
        return out


def conv_error():
    return library().d1_conv_error()

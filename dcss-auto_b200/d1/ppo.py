"""GAE and the PPO update of gpu-d1/scripts/run_ring_ablations.py:354-372 on the
B200 kernels, with BASELINE config 2's loss (value clipping, vf/entropy
coefficients) and a switch for the reference loss (0.25 * MSE, no value clip).

Per minibatch (all device work is libd1 kernels, launched on the current stream):

  layer 1    h1 = relu(X W1^T + b1)                d1_gemm_cobs_a (tcgen05, K = 1832; X's
             rows are the one-hot expansion of the rollout's compact history
             rows cobs[idx], written into the operand tiles in shared memory)
  tail       h2 = relu(h1 W2^T + b2), head, PPO    d1_ppo_tail (one tcgen05 launch: W2 and
             loss, dlogits/dvalue, dh2 = dhead Wh  an activation tile in shared memory,
             * relu'(h2), dh1 = (dh2 W2) * relu'(h1),  accumulators in TMEM)
             partials of dWh, dbh, db2
  dW2        dh2^T h1 (split-K fp32 slabs)         d1_gemm_ex
  (fused_tail=False: layer 2 by d1_gemm, the loss by d1_ppo_loss on warp MMAs,
  dh1 by d1_gemm with a mask epilogue -- three launches for the same products)
  dW1, db1   dh1^T [X | 1] (split-K fp32 slabs;    d1_gemm_cobs_b (the B operand expanded
             column 1832 = db1)                    from cobs[idx] the same way)
  step       slab and loss-partial reductions      d1_ppo_step (a reduction
             into the flat gradient, its norm,     launch, then the Adam launch)
             clip + Adam + bf16 copies
  (multi-GPU, default: d1_ppo_step_peer -- the reduction publishes each rank's
  gradient in an exchange buffer that the other ranks map through CUDA IPC, a
  kernel sums all ranks' buffers over NVLink peer loads after per-rank flags,
  then Adam; peer=False: d1_grad_reduce, NCCL all-reduce, d1_ppo_step)

compact=False runs the same update with X materialised: d1_ppo_gather_cobs
writes [one-hot rows | ones column] (pitch 1840) and layer 1 and dW1 read it
through d1_gemm / d1_gemm_ex. The products are the same bit for bit; the
compact path skips the 60 MB gather and one launch (measured: 0.132 vs 0.142 ms
per 16,384-sample minibatch).

The weight-gradient GEMMs read dh2, h1, dh1 and X as stored (row-major, so
[K, M] / [K, N] with K = samples): their tensor-core operands are MN-major and
no kernel writes a transposed copy.

The gradient of every minibatch is a mean over that rank's minibatch; with R
ranks the all-reduced gradient is divided by R, so it equals the gradient of the
union minibatch (every rank uses equal-size minibatches).
"""
import ctypes as C

import torch

from ._lib import D1Error, check, library, launch_stream
from . import gemm as G
from .policy import HID, NOUT, OBS

LOSS_TERMS = ('pg', 'vf', 'entropy', 'clip_count', 'approx_kl')


class AdamSegment(C.Structure):
    _fields_ = [('offset', C.c_int64), ('count', C.c_int64), ('rows', C.c_int), ('cols', C.c_int),
                ('bf16', C.c_void_p), ('bf16_t', C.c_void_p)]


class GradJob(C.Structure):
    _fields_ = [('src', C.c_void_p), ('stride', C.c_int64), ('nsrc', C.c_int), ('rows', C.c_int),
                ('cols_in', C.c_int), ('cols_out', C.c_int), ('in_norm', C.c_int), ('dst', C.c_void_p),
                ('dst_extra', C.c_void_p)]


class PPO:
    def __init__(self, policy, rollout, minibatch=16384, epochs=4, lr=3e-4, clip=0.2, vclip=0.2, vf_coef=0.5,
                 ent_coef=0.01, max_grad_norm=0.5, gamma=0.999, lam=0.95, adam_eps=1e-5, betas=(0.9, 0.999),
                 gae_mode=1, splits=8, group=None, graph=True, peer=True, compact=True, peer_wait_limit=0,
                 exchange='auto', splits2=None, perm_seed=0, fused_tail=True, dw2_stream=True):
        self.policy, self.rollout = policy, rollout
        self.fused_tail = fused_tail  # layer 2 + loss + dh1 as one launch (d1_ppo_tail)
        self.perm_seed = perm_seed  # key of the epoch permutation (with the device epoch count)
        self.peer_wait_limit = peer_wait_limit  # polls per flag wait; 0 = the library default (~1 s)
        if exchange not in ('auto', 'oneshot', 'twophase', 'nvls'):
            raise ValueError("exchange must be 'auto', 'oneshot', 'twophase' or 'nvls'")
        self.exchange = exchange
        self.compact = compact
        self.mb, self.epochs = minibatch, epochs
        self.lr, self.clip, self.vclip, self.vf_coef, self.ent_coef = lr, clip, vclip, vf_coef, ent_coef
        self.max_grad_norm, self.gamma, self.lam, self.eps, self.betas = max_grad_norm, gamma, lam, adam_eps, betas
        self.gae_mode, self.group = gae_mode, group
        self.lib = library()
        dev = policy.device
        T, B = rollout.T, rollout.env.batch
        self.total = T * B
        if self.total % minibatch:
            raise ValueError('rollout size must be a multiple of the minibatch')
        f32, bf = dict(device=dev), dict(device=dev, dtype=torch.bfloat16)
        self.adv = torch.empty((T, B), **f32)
        self.ret = torch.empty((T, B), **f32)
        self.stats = torch.zeros(2, dtype=torch.float64, device=dev)
        self.grad = torch.zeros(policy.size, **f32)
        self.m = torch.zeros(policy.size, **f32)
        self.v = torch.zeros(policy.size, **f32)
        self.step_dev = torch.zeros(1, dtype=torch.int64, device=dev)  # Adam step count
        self.use_graph, self.graph = graph, None
        self.perm = torch.empty(self.total, dtype=torch.int64, device=dev)
        self.perm_epoch = torch.zeros(1, dtype=torch.int64, device=dev)  # epochs drawn by d1_ppo_permute
        self.graph_perm = None  # whether the captured epoch draws its own permutation
        mb = minibatch
        self.xw = OBS + 8  # X row pitch: the 8-column tail carries the ones column
        self.x = None if compact else torch.empty((mb, self.xw), **bf)
        self.h1 = torch.empty((mb, HID), **bf)
        self.h2 = torch.empty((mb, HID), **bf)
        self.dh2 = torch.empty((mb, HID), **bf)
        self.dh1 = torch.empty((mb, HID), **bf)
        self.s1 = G.splits_for(mb, splits)
        self.slab1 = torch.empty((self.s1, HID, self.xw), **f32)
        # dW2 is 256 x 256: one 2-SM tile. Alone it needs 8x the K splits of dW1
        # to put ~128 CTAs to work; on its own stream beside dW1 (whose 64 CTA
        # pairs leave 20 SMs idle) 8 splits = 16 CTAs run in those gaps.
        self.side = torch.cuda.Stream(dev) if dw2_stream else None
        self.s2 = G.splits_for(mb, (splits if dw2_stream else splits * 8) if splits2 is None else splits2)
        self.slab2 = torch.empty((self.s2, HID, HID), **f32)
        self.part_len = self.lib.d1_ppo_loss_part_len()
        if fused_tail:
            self.loss_blocks = self.lib.d1_ppo_tail_blocks(mb)  # one partial per 128 rows
        else:
            batches = (mb + 63) // 64                 # the loss kernel takes 64 rows per pass
            per = (batches + 591) // 592              # passes per block with four blocks per SM
            self.loss_blocks = (batches + per - 1) // per
        self.part = torch.empty((self.loss_blocks, self.part_len), **f32)
        self.terms = torch.zeros(8, **f32)
        self.history = []
        lay = policy.layout
        self.off = {k: lay[k][0] for k in lay}
        head_len = NOUT * HID + NOUT + HID
        assert self.off['bh'] == self.off['wh'] + NOUT * HID and self.off['b2'] == self.off['bh'] + NOUT
        self.head_len = head_len
        bfc = policy.bf16
        segs = [AdamSegment(self.off['w1'], HID * OBS, HID, OBS, bfc['w1'].data_ptr(), None),
                AdamSegment(self.off['w2'], HID * HID, HID, HID, bfc['w2'].data_ptr(), bfc['w2t'].data_ptr()),
                AdamSegment(self.off['wh'], NOUT * HID, NOUT, HID, bfc['wh'].data_ptr(), None)]
        self.segs = (AdamSegment * len(segs))(*segs)
        g, ptr = self.grad, lambda t: t.data_ptr()
        jobs = [GradJob(ptr(self.slab1), HID * self.xw, self.s1, HID, self.xw, OBS, 1, ptr(g[self.off['w1']:]),
                        ptr(g[self.off['b1']:])),
                GradJob(ptr(self.slab2), HID * HID, self.s2, 1, HID * HID, HID * HID, 1, ptr(g[self.off['w2']:]), None),
                GradJob(ptr(self.part), self.part_len, self.loss_blocks, 1, head_len, head_len, 1,
                        ptr(g[self.off['wh']:]), None),
                GradJob(ptr(self.part[:, head_len:]), self.part_len, self.loss_blocks, 1, 8, 8, 0, ptr(self.terms),
                        None)]
        self.jobs = (GradJob * len(jobs))(*jobs)
        self.peer = None
        if group is not None and peer:
            self._peer_setup(group)

    def _peer_setup(self, group):
        """Exchange buffers for the peer all-reduce: each rank allocates two
        halves of the flat gradient plus one flag per rank, shares the CUDA IPC
        handle over the process group and maps every peer's buffer."""
        import torch.distributed as dist
        lib, world, rank = self.lib, dist.get_world_size(group), dist.get_rank(group)
        if world > 8:
            raise ValueError('the peer all-reduce supports up to 8 ranks')
        if self.exchange == 'nvls':
            self._nvls_setup(group, world, rank)
            return
        P = self.grad.numel()
        self.xstride = (P + 3) // 4 * 4
        flag_off = 2 * self.xstride * 4
        base, handle = C.c_void_p(), (C.c_char * lib.d1_peer_handle_bytes())()
        with torch.cuda.device(self.policy.device):
            check(lib.d1_peer_alloc(self.peer_bytes(world), C.byref(base), handle), 'd1_peer_alloc')
            handles = [None] * world
            dist.all_gather_object(handles, bytes(handle), group=group)
            ptrs = []
            for p, h in enumerate(handles):
                if p == rank:
                    ptrs.append(base.value)
                else:
                    q = C.c_void_p()
                    check(lib.d1_peer_open(h, C.byref(q)), 'd1_peer_open')
                    ptrs.append(q.value)
        self.peer_attach(world, rank, ptrs)
        self.peer['base'] = base.value

    def _nvls_setup(self, group, world, rank):
        """The exchange buffer as torch symmetric memory bound to an NVLink
        multicast object: the one-shot layout (two gradient halves, flags),
        peer pointers for the flags, and the multicast address the all-reduce
        reads the summed gradient through (multimem.ld_reduce)."""
        import torch.distributed._symmetric_memory as symm
        dev = self.policy.device
        self.exchange_nvls = True
        nbytes = self.peer_bytes(world)
        buf = symm.empty((nbytes + 15) // 16 * 4, dtype=torch.float32, device=dev)
        buf.zero_()
        torch.cuda.synchronize(dev)
        hdl = symm.rendezvous(buf, group)
        mc = int(getattr(hdl, 'multicast_ptr', 0) or 0)
        if not mc:
            raise D1Error('exchange="nvls": this system gives the exchange buffer no NVLink multicast address')
        self.peer_attach(world, rank, [int(p) for p in hdl.buffer_ptrs])
        self.peer['mc'] = mc
        self.peer['symm'] = (buf, hdl)  # keeps the mapping alive

    def two_phase(self, world):
        """Whether the peer exchange of `world` ranks is the two-phase one
        (each rank reduces a slice, then gathers) rather than the one-shot
        one (each rank reads every peer's whole gradient). 'auto' is the
        one-shot exchange: measured on 8 B200s, a minibatch took 0.194 ms with
        it and 0.199 ms with the two-phase one (2 GPUs: 0.153 and 0.168 ms);
        the extra flag round costs more than the smaller transfer saves."""
        return self.exchange == 'twophase' and not getattr(self, 'exchange_nvls', False)

    def _peer_layout(self, world):
        """(stride, flag offset in bytes): one-shot -- two halves of the flat
        gradient; two-phase -- inbox and gather areas of [2][world][slice]."""
        P = self.grad.numel()
        if self.two_phase(world):
            slice_ = ((P + world - 1) // world + 3) // 4 * 4
            return slice_, 4 * world * slice_ * 4
        xstride = (P + 3) // 4 * 4
        return xstride, 2 * xstride * 4

    def peer_bytes(self, world=None):
        """Size of one rank's exchange buffer: the gradient areas and 16 u64
        flags."""
        import torch.distributed as dist
        world = world if world is not None else dist.get_world_size(self.group)
        return self._peer_layout(world)[1] + 16 * 8

    def peer_attach(self, world, rank, ptrs):
        """Use the exchange buffers ptrs[p] (rank p's, as mapped here) for the
        gradient all-reduce of every minibatch."""
        self.xstride, flag_off = self._peer_layout(world)
        self.peer = dict(world=world, rank=rank, base=None, ptrs=list(ptrs), two_phase=self.two_phase(world),
                         xbufs=(C.c_void_p * world)(*ptrs),
                         flags=(C.c_void_p * world)(*[q + flag_off for q in ptrs]))

    @property
    def stream(self):
        return launch_stream(self.policy.device)

    # ------------------------------------------------------------------ GAE
    def advantages(self):
        r = self.rollout
        r.join()  # a caller may have driven r.step() itself
        out = r.out  # [T, B, OUT]: reward at column 0, done at column 1
        self.stats.zero_()
        check(self.lib.d1_gae(out.data_ptr(), out[:, :, 1].data_ptr(), out.stride(0), out.stride(1),
                              r.values.data_ptr(), r.T, r.env.batch, self.gamma, self.lam, self.adv.data_ptr(),
                              self.ret.data_ptr(), self.stats.data_ptr(), self.gae_mode, self.stream), 'd1_gae')
        count = float(self.total)
        if self.group is not None:
            import torch.distributed as dist
            dist.all_reduce(self.stats, group=self.group)
            count *= dist.get_world_size(self.group)
        self.adv_count = count
        return self.adv, self.ret

    # ------------------------------------------------------------------ update
    def minibatch(self, idx):
        """One gradient step on the rollout samples `idx` (int64, length mb)."""
        p, r, lib, s = self.policy, self.rollout, self.lib, self.stream
        mb = self.mb
        cobs = r.cobs[:r.T].reshape(self.total, r.cobs.shape[2])
        if self.compact:
            G.gemm_cobs_a(cobs, p.bf16['w1'], idx=idx, bias=p.params['b1'], relu=True, out=self.h1)
        else:
            check(lib.d1_ppo_gather_cobs(cobs.data_ptr(), idx.data_ptr(), mb, self.x.data_ptr(), self.xw, 1, s),
                  'd1_ppo_gather_cobs')
            G.gemm(self.x[:, :OBS], p.bf16['w1'], bias=p.params['b1'], relu=True, out=self.h1)
        g = self.grad
        if self.fused_tail:
            # layer 2, head, loss, dh2 and dh1 in one launch
            check(lib.d1_ppo_tail(self.h1.data_ptr(), p.bf16['w2'].data_ptr(), p.params['b2'].data_ptr(),
                                  p.bf16['wh'].data_ptr(), p.params['bh'].data_ptr(), idx.data_ptr(),
                                  r.legal.data_ptr(), r.actions.data_ptr(), r.logp.data_ptr(), self.adv.data_ptr(),
                                  self.ret.data_ptr(), r.values.data_ptr(), self.stats.data_ptr(), self.adv_count,
                                  mb, self.clip, self.vclip, self.vf_coef, self.ent_coef, self.dh2.data_ptr(),
                                  self.dh1.data_ptr(), self.part.data_ptr(), s), 'd1_ppo_tail')
        else:
            G.gemm(self.h1, p.bf16['w2'], bias=p.params['b2'], relu=True, out=self.h2)
            check(lib.d1_ppo_loss(self.h2.data_ptr(), p.bf16['wh'].data_ptr(), p.params['bh'].data_ptr(),
                                  idx.data_ptr(), r.legal.data_ptr(), r.actions.data_ptr(), r.logp.data_ptr(),
                                  self.adv.data_ptr(), self.ret.data_ptr(), r.values.data_ptr(),
                                  self.stats.data_ptr(), self.adv_count, mb, self.clip, self.vclip, self.vf_coef,
                                  self.ent_coef, self.dh2.data_ptr(), None, mb, self.part.data_ptr(),
                                  self.loss_blocks, s), 'd1_ppo_loss')
            # dh1 = (dh2 W2) * relu'(h1)
            G.gemm(self.dh2, p.bf16['w2t'], mask=self.h1, out=self.dh1)
        # dW2 = dh2^T h1, beside dW1 when it has its own stream
        main = torch.cuda.current_stream(p.device)
        if self.side is not None:
            self.side.wait_stream(main)
            with torch.cuda.stream(self.side):
                G.gemm_ex(self.dh2, self.h1, a_kn=True, b_kn=True, out_f32=self.slab2, splits=self.s2)
        else:
            G.gemm_ex(self.dh2, self.h1, a_kn=True, b_kn=True, out_f32=self.slab2, splits=self.s2)
        # dW1 = dh1^T X; X's ones column makes slab column 1832 the column sums of dh1 (db1)
        if self.compact:
            G.gemm_cobs_b(self.dh1, cobs, idx, self.xw, self.slab1, splits=self.s1)
        else:
            G.gemm_ex(self.dh1, self.x, a_kn=True, b_kn=True, out_f32=self.slab1, splits=self.s1)
        if self.side is not None:
            main.wait_stream(self.side)
        jobs, njobs = self.jobs, len(self.jobs)
        if self.peer is not None and self.peer.get('mc'):
            pr = self.peer
            check(lib.d1_ppo_step_nvls(jobs, njobs, p.flat.data_ptr(), g.data_ptr(), self.m.data_ptr(),
                                       self.v.data_ptr(), g.numel(), self.lr, self.betas[0], self.betas[1], self.eps,
                                       self.max_grad_norm, self.step_dev.data_ptr(), self.segs, len(self.segs),
                                       pr['xbufs'], pr['flags'], self.xstride, C.c_void_p(pr['mc']), pr['world'],
                                       pr['rank'], self.peer_wait_limit, s), 'd1_ppo_step_nvls')
            return self.terms
        if self.peer is not None:
            pr = self.peer
            fn = lib.d1_ppo_step_peer2 if pr['two_phase'] else lib.d1_ppo_step_peer
            check(fn(jobs, njobs, p.flat.data_ptr(), g.data_ptr(), self.m.data_ptr(), self.v.data_ptr(), g.numel(),
                     self.lr, self.betas[0], self.betas[1], self.eps, self.max_grad_norm, self.step_dev.data_ptr(),
                     self.segs, len(self.segs), pr['xbufs'], pr['flags'], self.xstride, pr['world'], pr['rank'],
                     self.peer_wait_limit, s),
                  'd1_ppo_step_peer2' if pr['two_phase'] else 'd1_ppo_step_peer')
            return self.terms
        if self.group is not None:
            import torch.distributed as dist
            check(lib.d1_grad_reduce(jobs, njobs, s), 'd1_grad_reduce')
            dist.all_reduce(g, group=self.group)
            g.div_(dist.get_world_size(self.group))
            jobs, njobs = None, 0
        check(lib.d1_ppo_step(jobs, njobs, p.flat.data_ptr(), g.data_ptr(), self.m.data_ptr(), self.v.data_ptr(),
                              g.numel(), self.lr, self.betas[0], self.betas[1], self.eps, self.max_grad_norm,
                              self.step_dev.data_ptr(), self.segs, len(self.segs), s), 'd1_ppo_step')
        return self.terms

    def _permute(self):
        """This epoch's minibatch order: d1_ppo_permute keyed by perm_seed and the
        device epoch count, which it then advances (both on the stream, so a
        captured epoch draws a fresh order on every replay)."""
        s = self.stream
        check(self.lib.d1_ppo_permute(self.perm.data_ptr(), self.total, self.perm_seed & (2 ** 64 - 1),
                                      self.perm_epoch.data_ptr(), s), 'd1_ppo_permute')
        check(self.lib.d1_counter_add(self.perm_epoch.data_ptr(), 1, s), 'd1_counter_add')

    def _epoch(self, own_perm):
        if own_perm:
            self._permute()
        for i in range(0, self.total, self.mb):
            self.minibatch(self.perm[i:i + self.mb])

    def update(self, generator=None):
        """epochs x (total / mb) minibatch steps over a fresh permutation each epoch.

        The order comes from d1_ppo_permute (a keyed bijection, one pass, no
        sort) unless a torch generator is given: then it is
        torch.randperm(total, generator=generator), the reference's own draw
        (gpu-d1/scripts/run_ring_ablations.py:364), so the minibatches follow
        the reference's order for the same generator state.

        With graph=True the first epoch runs eagerly (it also initialises every
        kernel's attributes) and the second is captured once into a CUDA graph
        (with the permutation when it is d1_ppo_permute's); later epochs replay
        it, so a whole epoch of ~15 launches per minibatch costs one host call."""
        dev = self.policy.device
        own = generator is None
        if self.graph is not None and self.graph_perm != own:
            self.graph = None  # captured for the other permutation source
        for _ in range(self.epochs):
            if not own:
                torch.randperm(self.total, device=dev, generator=generator, out=self.perm)
            if not self.use_graph:
                self._epoch(own)
            elif self.graph is None and not getattr(self, '_warm', False):
                self._epoch(own)
                self._warm = True
            else:
                if self.graph is None:
                    self.graph = torch.cuda.CUDAGraph()
                    self.graph_perm = own
                    side = torch.cuda.Stream(dev)
                    side.wait_stream(torch.cuda.current_stream(dev))
                    with torch.cuda.stream(side), torch.cuda.graph(self.graph, stream=side):
                        self._epoch(own)
                    torch.cuda.current_stream(dev).wait_stream(side)
                self.graph.replay()
        self.check_peer()

    def check_peer(self):
        """Raise if a gradient exchange since the last check gave up waiting for
        a peer (that minibatch's step then changed no parameter on this rank, so
        the ranks' parameters no longer agree). Synchronises the device."""
        if self.peer is not None and self.lib.d1_peer_error():
            raise D1Error('peer gradient exchange: a rank did not publish its gradient in time; '
                          'this rank skipped the optimizer step and training cannot continue')

    def release(self):
        """Free the captured graph (before destroying a process group it uses)
        and, after every rank has finished with them, the exchange buffers."""
        self.graph = None
        if self.peer is not None:
            import torch.distributed as dist
            torch.cuda.synchronize(self.policy.device)
            dist.barrier(group=self.group)
            pr = self.peer
            if pr['base'] is not None:
                for p, q in enumerate(pr['ptrs']):
                    if p != pr['rank']:
                        self.lib.d1_peer_close(C.c_void_p(q))
                dist.barrier(group=self.group)
                self.lib.d1_peer_free(C.c_void_p(pr['base']))
            self.peer = None

    def iteration(self, generator=None):
        """Collect a rollout, compute advantages, update: one PPO iteration."""
        r = self.rollout
        r.collect()
        self.advantages()
        self.update(generator)
        r.roll()

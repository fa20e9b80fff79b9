"""Rollout buffer and collection loop of gpu-d1/scripts/run_ring_ablations.py:332-353
on the B200 kernels.

Every step the policy reads the current one-hot observation (`obs`, one
[B, 1832] bf16 buffer) and writes action/log-prob/value slot t; the env step
writes the next one-hot observation over it, its compact form (320 B per env)
into history slot `cobs[t+1]`, the legal mask into slot t+1 and its outcome row
into out[t]. The history is kept compact -- 320 instead of 3,664 bytes per
sample, 2.7 instead of 31 GB at 65,536 envs x 128 steps -- and the update's
layer-1 and dW1 GEMMs expand the minibatch's rows into their operand tiles.
Nothing is copied between kernels.
"""
import torch

OBS, COBS = 1832, 320


def env_ranges(batch, parts):
    """Contiguous env ranges for `parts` streams (one range below 8,192 envs,
    and ranges of at least 4,096 envs: smaller launches lose more to their
    tails than the overlap gains)."""
    parts = max(1, min(parts, batch // 4096)) if batch >= 8192 else 1
    edges = [batch * i // parts for i in range(parts + 1)]
    return [(edges[i], edges[i + 1]) for i in range(parts)]


class Rollout:
    """parts > 1 splits the batch into that many contiguous env ranges, each
    stepped (policy, then env) on its own stream: one range's env kernel then
    overlaps another's policy GEMMs (measured on one B200 at 65,536 envs: 0.373
    -> 0.342 ms per step with two ranges). The ranges' streams follow the
    current stream's earlier work at every step and are joined back into it by
    join(), which roll(), bootstrap() and collect() call; a caller that drives
    step() itself calls join() before reading the buffers on another stream.
    Trajectories do not depend on `parts`.

    graphs=True: collect() runs its first rollout eagerly, then captures the
    whole rollout (every slot's policy and env launches on the ranges' streams,
    with the same fork/join structure, so consecutive steps still overlap as
    they do eagerly) as one CUDA graph, and later collect() calls replay it: one
    launch per rollout from the host instead of a dozen per step, the same
    kernels and the same trajectories. Slot t reads its sampling step from
    element t of a device array that collect() fills with global_step + t. The
    graph reads the policy's weights and the env rows in place, so training
    between rollouts is seen; step() outside collect() stays eager."""

    def __init__(self, env, policy, horizon, seed=0, sample_seed=None, parts=2, graphs=False):
        self.env, self.policy, self.T = env, policy, horizon
        B, dev = env.batch, env.device
        self.seed = seed
        self.sample_seed = seed if sample_seed is None else sample_seed
        self.obs = torch.empty((B, OBS), dtype=torch.bfloat16, device=dev)
        self.cobs = torch.empty((horizon + 1, B, COBS), dtype=torch.uint8, device=dev)
        self.legal = torch.empty((horizon + 1, B), dtype=torch.int16, device=dev)
        self.actions = torch.empty((horizon, B), dtype=torch.int64, device=dev)
        self.logp = torch.empty((horizon, B), device=dev)
        self.values = torch.empty((horizon + 1, B), device=dev)
        # outcomes stored as planes [T, 10, B] (GAE reads rewards and dones
        # coalesced); self.out is the [T, B, 10] view of them
        self.out_planes = torch.zeros((horizon, env.out.shape[1], B), device=dev)
        self.out = self.out_planes.permute(0, 2, 1)
        self.global_step = 0
        self.ranges = env_ranges(B, parts)
        self.streams = [torch.cuda.Stream(dev) for _ in self.ranges] if len(self.ranges) > 1 else []
        self.graphs = graphs
        self._graph = None
        env.reset(seed, obs_out=self.obs, legal_out=self.legal[0], cobs_out=self.cobs[0])

    @property
    def parts(self):
        return len(self.ranges)

    def join(self):
        """Make the current stream wait for the ranges' streams."""
        main = torch.cuda.current_stream(self.env.device)
        for s in self.streams:
            main.wait_stream(s)

    def step(self, t, step=None, h1=None, h2=None):
        """Slot t's policy and env step. `step` (the sampling step: an int, or an
        int64 device tensor of one element) defaults to global_step; h1 and h2
        give the policy's activation rows (the graphs pass their own)."""
        step = self.global_step if step is None else step
        if not self.streams:
            self.policy.act(self.obs, self.legal[t], self.sample_seed, step, self.env.first_env,
                            action=self.actions[t], logp=self.logp[t], value=self.values[t], h1=h1, h2=h2)
            self.env.step(self.actions[t], obs_out=self.obs, legal_out=self.legal[t + 1], out_out=self.out[t],
                          cobs_out=self.cobs[t + 1])
        else:
            main = torch.cuda.current_stream(self.env.device)
            for i, (lo, hi) in enumerate(self.ranges):
                s = self.streams[i]
                s.wait_stream(main)
                with torch.cuda.stream(s):
                    self.policy.act(self.obs[lo:hi], self.legal[t][lo:hi], self.sample_seed, step,
                                    self.env.first_env + lo, action=self.actions[t][lo:hi],
                                    logp=self.logp[t][lo:hi], value=self.values[t][lo:hi], part=i,
                                    h1=None if h1 is None else h1[lo:hi], h2=None if h2 is None else h2[lo:hi])
                    self.env.step(self.actions[t], obs_out=self.obs, legal_out=self.legal[t + 1],
                                  out_out=self.out[t], cobs_out=self.cobs[t + 1], rows=(lo, hi))
        self.global_step += 1

    def bootstrap(self):
        self.join()
        self.policy.value(self.obs, out=self.values[self.T])

    def collect(self):
        if self.graphs and self._graph is not None:
            torch.add(self._slots, self.global_step, out=self._steps)
            self._graph.replay()
            self.global_step += self.T
        else:
            for t in range(self.T):
                self.step(t)
            if self.graphs:
                self._capture()
        self.bootstrap()

    def _capture(self):
        """The whole rollout as one graph (the first, eager rollout has set up
        every kernel's attributes); capturing runs nothing."""
        dev = self.env.device
        self._slots = torch.arange(self.T, dtype=torch.int64, device=dev)
        self._steps = torch.empty(self.T, dtype=torch.int64, device=dev)
        # the graph's own activation rows: the policy's cached ones may be
        # reallocated by a later eager call with more rows
        self._h1 = torch.empty((self.env.batch, self.policy.hidden), dtype=torch.bfloat16, device=dev)
        self._h2 = torch.empty_like(self._h1)
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side), torch.cuda.graph(g, stream=side):
            for t in range(self.T):
                self.step(t, step=self._steps[t:t + 1], h1=self._h1, h2=self._h2)
            self.join()
        torch.cuda.current_stream(dev).wait_stream(side)
        self.global_step -= self.T
        self._graph = g

    def roll(self):
        """Start the next rollout from the last observation (the one-hot buffer
        already holds it)."""
        self.join()
        self.cobs[0].copy_(self.cobs[self.T])
        self.legal[0].copy_(self.legal[self.T])

    @property
    def rewards(self):
        return self.out[:, :, 0]

    @property
    def dones(self):
        return self.out[:, :, 1]


class DecisionGraph:
    """One decision of a host-driven loop captured once as a CUDA graph:
    copy the actions in from pinned host memory, step the env, run the policy on
    the new observation (two GEMMs + head + masked draw) and copy the outcome
    rows and the next actions back to pinned host memory. As in Rollout, the
    batch runs as contiguous env ranges on their own streams (the first range's
    policy overlaps the next range's env kernel), and each range's outcome rows
    are copied back on a further stream while its policy runs; the graph joins
    them all before it ends. The sampling step is a device counter that the
    graph advances after the draws, so every replay draws fresh uniforms.
    replay() launches it; the caller synchronises before reading the host
    buffers."""

    def __init__(self, env, policy, seed, first_env=0, step=0, parts=2):
        import torch
        from ._lib import check, library, launch_stream
        dev, n = env.device, env.batch
        self.env, self.policy = env, policy
        self.h_act = torch.zeros(n, dtype=torch.int64).pin_memory()
        self.h_out = torch.empty((n, env.out.shape[1])).pin_memory()
        self.h_next = torch.empty(n, dtype=torch.int64).pin_memory()
        self.d_act = torch.empty(n, dtype=torch.int64, device=dev)
        self.next = torch.empty(n, dtype=torch.int64, device=dev)
        self.logp = torch.empty(n, device=dev)
        self.value = torch.empty(n, device=dev)
        self.step = torch.full((1,), step, dtype=torch.int64, device=dev)
        # The graph's own activation buffers: the policy's cached ones are
        # reallocated when a later eager call needs more rows, which would leave
        # the captured pointers dangling.
        self.h1 = torch.empty((n, policy.hidden), dtype=torch.bfloat16, device=dev)
        self.h2 = torch.empty((n, policy.hidden), dtype=torch.bfloat16, device=dev)
        lib = library()
        self.ranges = env_ranges(n, parts)
        split = len(self.ranges) > 1
        streams = [torch.cuda.Stream(dev) for _ in self.ranges] if split else []
        copies = [torch.cuda.Stream(dev) for _ in self.ranges]  # outcome rows back while the policy runs

        def body():
            main = torch.cuda.current_stream(dev)
            self.d_act.copy_(self.h_act, non_blocking=True)
            for i, (lo, hi) in enumerate(self.ranges):
                st = streams[i] if split else main
                st.wait_stream(main)
                with torch.cuda.stream(st):
                    env.step(self.d_act, rows=(lo, hi))
                    copies[i].wait_stream(st)
                    with torch.cuda.stream(copies[i]):
                        self.h_out[lo:hi].copy_(env.out[lo:hi], non_blocking=True)
                    policy.act(env.obs[lo:hi], env.legal[lo:hi], seed, self.step, first_env + lo,
                               action=self.next[lo:hi], logp=self.logp[lo:hi], value=self.value[lo:hi],
                               h1=self.h1[lo:hi], h2=self.h2[lo:hi])
                    self.h_next[lo:hi].copy_(self.next[lo:hi], non_blocking=True)
            for i in range(len(self.ranges)):
                if split:
                    main.wait_stream(streams[i])
                main.wait_stream(copies[i])
            check(lib.d1_counter_add(self.step.data_ptr(), 1, launch_stream(dev)), 'd1_counter_add')

        body()  # warm-up: kernel attributes and workspaces exist before capture
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side), torch.cuda.graph(self.graph, stream=side):
            body()
        torch.cuda.current_stream(dev).wait_stream(side)

    def replay(self):
        self.graph.replay()

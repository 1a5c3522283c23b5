"""CUDA-graph runner for the packed linears of one decode token.

The reference lost most of its decode time to per-call host work (253
matmuls per token, 43 ms device vs 149 ms wall on an A100; CHANGELOG 0.2.2,
epure/kernels/cuda.py:58-85).  ``GraphedLinearStack`` removes it: the launches
of a whole token are recorded once in a CUDA graph over static buffers, and
``__call__`` only copies the token's input in, replays the graph and copies
the result out.

The stack is a ``LinearStack`` (epure.synthetic): per layer, q/k/v share the
layer input (one launch), o reads q, gate/up read o (one launch), down reads
up, and down's output feeds the next layer.
"""
import torch

from . import _native


class GraphedLinearStack:
    def __init__(self, stack, m=1, dtype=torch.bfloat16, device=None):
        self.stack = stack
        self.m = m
        self.dtype = dtype
        self.device = torch.device(device or stack.device)
        b0 = stack.blocks[0]
        h, inter = b0["q_proj"].in_features, b0["gate_proj"].out_features
        mk = lambda n: torch.zeros((m, n), dtype=dtype, device=self.device)  # noqa: E731
        self.x = mk(h)
        self.q, self.k, self.v = mk(b0["q_proj"].out_features), mk(b0["k_proj"].out_features), \
            mk(b0["v_proj"].out_features)
        self.o = mk(b0["o_proj"].out_features)
        self.g, self.u = mk(inter), mk(inter)
        self.d = [mk(b0["down_proj"].out_features), mk(b0["down_proj"].out_features)]
        self.out = None
        self.graph = None
        self.stream = torch.cuda.Stream(device=self.device)
        self.launches_per_step = 4 * len(stack.blocks)

    def step_eager(self):
        """Issue one token's launches on the current stream (no graph)."""
        h = self.x
        for li, b in enumerate(self.stack.blocks):
            _native.linear_multi(h, [b["q_proj"], b["k_proj"], b["v_proj"]],
                                 outs=[self.q, self.k, self.v])
            _native.linear_multi(self.q, [b["o_proj"]], outs=[self.o])
            _native.linear_multi(self.o, [b["gate_proj"], b["up_proj"]], outs=[self.g, self.u])
            dst = self.d[li & 1]
            _native.linear_multi(self.u, [b["down_proj"]], outs=[dst])
            h = dst
        self.out = h
        return h

    def capture(self):
        """Record one step in a CUDA graph (warms up and reserves workspaces first)."""
        with torch.cuda.stream(self.stream):
            for grp in self.stack.groups()[:4]:
                _native.reserve_workspace(grp, self.m, self.device)
            self.step_eager()
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=self.stream):
            self.step_eager()
        self.graph = g
        return self

    def replay(self):
        self.graph.replay()
        return self.out

    def __call__(self, x_host, out_host=None):
        """Host input -> host output for one token: H2D copy, graph replay, D2H copy."""
        if self.graph is None:
            self.capture()
        self.x.copy_(x_host, non_blocking=True)
        self.graph.replay()
        if out_host is None:
            out_host = torch.empty(self.out.shape, dtype=self.out.dtype, pin_memory=True)
        out_host.copy_(self.out, non_blocking=True)
        return out_host


class ChainedLinearStack:
    """The same token chain as GraphedLinearStack, as ONE persistent launch.

    ``epq_chain_run`` walks all launches of the token inside one cooperative
    kernel: weights stream continuously through each SM's TMA ring, layers
    synchronise through grid barriers, and intermediate outputs stay as fp32
    partial sums (they are never rounded to the activation dtype).  The stack's
    stores must use the "tiled" GPU layout.  The launch is captured in a CUDA
    graph; ``__call__`` copies the token in, replays and copies the result out.
    """

    def __init__(self, stack, dtype=torch.bfloat16, device=None):
        self.stack = stack
        self.device = torch.device(device or stack.device)
        steps = stack.chain_steps()
        self.ws = _native.chain_prepare(steps)
        k0 = steps[0][0][0].in_features
        last, feed = steps[-1]
        self.x = torch.zeros((1, k0), dtype=dtype, device=self.device)
        self.out = torch.zeros((1, last[feed].out_features), dtype=dtype, device=self.device)
        self.graph = None
        self.stream = torch.cuda.Stream(device=self.device)
        self.launches_per_step = 1

    def step_eager(self):
        _native.chain_run(self.ws, self.x, self.out)
        return self.out

    def capture(self):
        with torch.cuda.stream(self.stream):
            self.step_eager()
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=self.stream):
            self.step_eager()
        self.graph = g
        return self

    def replay(self):
        self.graph.replay()
        return self.out

    def __call__(self, x_host, out_host=None):
        if self.graph is None:
            self.capture()
        self.x.copy_(x_host, non_blocking=True)
        self.graph.replay()
        if out_host is None:
            out_host = torch.empty(self.out.shape, dtype=self.out.dtype, pin_memory=True)
        out_host.copy_(self.out, non_blocking=True)
        return out_host

"""Compressed-state fine-tuning step over the packed linears of a decoder.

The fine-tuning path of the reference (epure/finetune.py:49-102: make_trainable
promotes every store's scales and codebook to fp32 parameters, indices stay
frozen) spends its linear-layer time in three contractions per packed linear:
the forward ``y = x W^T``, the activation gradient ``dX = dY W`` and the
parameter gradients ``dscale`` / ``dcb`` reduced from ``dY^T X``.
``PackedTrainStep`` runs exactly those, through libepq.so, for every packed
linear of a ``LinearStack`` (epure.synthetic), chained the way a token batch
visits them: forward q/k/v (fused) -> o -> gate/up (fused) -> down per layer;
backward in reverse, where the gradient reaching a linear's output is the
activation gradient of the linear that reads it (down -> up -> o -> q) and the
linears whose outputs the packed path does not consume (k, v, gate: attention
and the SwiGLU product are not packed linears) receive a fixed synthetic
output gradient.  Attention, norms, the loss and the optimizer update are not
part of the packed path.
"""
import torch

from . import _native


class PackedTrainStep:
    def __init__(self, stack, m, dtype=torch.bfloat16, device=None, seed=0):
        self.stack = stack
        self.m = m
        self.dtype = dtype
        self.device = torch.device(device or stack.device)
        b0 = stack.blocks[0]
        g = torch.Generator(device=self.device).manual_seed(seed)
        rnd = lambda n: (torch.randn(m, n, generator=g, device=self.device) * 0.05).to(dtype)  # noqa: E731
        # fixed output gradients for the outputs the packed path does not consume
        self.dk, self.dv = rnd(b0["k_proj"].out_features), rnd(b0["v_proj"].out_features)
        self.dg = rnd(b0["gate_proj"].out_features)
        self.dout = rnd(b0["down_proj"].out_features)
        self.grads = None

    def step(self, x):
        """Forward + backward of every packed linear; returns the input gradient.

        ``self.grads`` holds, per layer, {name: (dscale [n, ng] f32, dcb f32)}.
        """
        acts = []
        h = x
        for b in self.stack.blocks:
            q, _, _ = _native.linear_multi(h, [b["q_proj"], b["k_proj"], b["v_proj"]])
            o = _native.linear(q, b["o_proj"])
            _, u = _native.linear_multi(o, [b["gate_proj"], b["up_proj"]])
            d = _native.linear(u, b["down_proj"])
            acts.append((h, q, o, u))
            h = d
        grads = [None] * len(self.stack.blocks)
        dh = self.dout
        for li in range(len(self.stack.blocks) - 1, -1, -1):
            b = self.stack.blocks[li]
            hin, q, o, u = acts[li]
            gl = {}
            du, *gl["down_proj"] = _native.linear_bwd(u, dh, b["down_proj"])
            do_u, *gl["up_proj"] = _native.linear_bwd(o, du, b["up_proj"])
            do_g, *gl["gate_proj"] = _native.linear_bwd(o, self.dg, b["gate_proj"])
            dq, *gl["o_proj"] = _native.linear_bwd(q, do_u + do_g, b["o_proj"])
            dh_q, *gl["q_proj"] = _native.linear_bwd(hin, dq, b["q_proj"])
            dh_k, *gl["k_proj"] = _native.linear_bwd(hin, self.dk, b["k_proj"])
            dh_v, *gl["v_proj"] = _native.linear_bwd(hin, self.dv, b["v_proj"])
            dh = dh_q + dh_k + dh_v
            grads[li] = gl
        self.grads = grads
        return dh

    def flops(self):
        """Forward + dX + dW contractions of one step."""
        return 3 * self.stack.flops(self.m)

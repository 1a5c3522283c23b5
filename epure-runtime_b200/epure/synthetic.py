"""Seeded synthetic packed stores and decoder-shaped stacks of them.

The benchmark configurations use random-init weights (there is no network for
checkpoints): indices uniform over the codebook, a 256x4 fp16 codebook with
N(0,1) entries, fp16 scales |N(0, 0.02)| per output row per 128-weight group.
``make_store`` draws exactly that; ``DecoderShapes`` lists the packed linears
of the decoder families the benchmark names; ``LinearStack`` chains them the
way one decode token visits them.
"""
from dataclasses import dataclass

import torch

from .runtime import PackedWeight


def make_store(n, k, *, vec=4, levels=256, group=128, device="cuda", seed=0,
               cb_dtype=torch.float16, scale_dtype=torch.float16, gpu_layout=None):
    """A random PackedWeight [n, k] with the benchmark's value distributions."""
    gen = torch.Generator(device=device).manual_seed(int(seed))
    ng = -(-k // group)
    idx = torch.randint(0, levels, (n, k // vec), dtype=torch.uint8, device=device,
                        generator=gen)
    cb = torch.randn(levels, vec, generator=gen, device=device).to(cb_dtype)
    if vec == 1:
        cb = cb.reshape(-1).float()
        if levels <= 16:
            lo = idx[:, 0::2] & 0x0F
            hi = (idx[:, 1::2] & 0x0F) if k % 2 == 0 else None
            idx = (lo | (hi << 4)) if hi is not None else lo
    scale = (torch.randn(n, ng, generator=gen, device=device) * 0.02).abs().to(scale_dtype)
    return PackedWeight((n, k), idx.reshape(-1), scale, cb, group, levels, vec=vec,
                        gpu_layout=gpu_layout)


def store_bytes(st):
    """Bytes of a store the op must read: indices, scales, codebook."""
    n, k = st.out_features, st.in_features
    ng = -(-k // st.group)
    idx = n * k // st.vec if (st.vec == 4 or st.levels > 16) else n * ((k + 1) // 2)
    return idx + n * ng * st.scale.element_size() + st.cb.numel() * st.cb.element_size()


@dataclass(frozen=True)
class DecoderShapes:
    name: str
    layers: int
    hidden: int
    intermediate: int
    heads: int
    kv_heads: int
    head_dim: int
    vocab: int

    def linears(self):
        """(name, out_features, in_features) of one layer's packed linears."""
        h, i, hd = self.hidden, self.intermediate, self.head_dim
        return [
            ("q_proj", self.heads * hd, h),
            ("k_proj", self.kv_heads * hd, h),
            ("v_proj", self.kv_heads * hd, h),
            ("o_proj", h, self.heads * hd),
            ("gate_proj", i, h),
            ("up_proj", i, h),
            ("down_proj", h, i),
        ]

    def packed_weights(self):
        return self.layers * sum(n * k for _, n, k in self.linears())


QWEN3_1_7B = DecoderShapes("qwen3-1.7b", 28, 2048, 6144, 16, 8, 128, 151936)
LLAMA3_8B = DecoderShapes("llama3-8b", 32, 4096, 14336, 32, 8, 128, 128256)
LLAMA3_70B = DecoderShapes("llama3-70b", 80, 8192, 28672, 64, 8, 128, 128256)
SHAPES = {s.name: s for s in (QWEN3_1_7B, LLAMA3_8B, LLAMA3_70B)}


class LinearStack:
    """Every packed linear of a decoder, visited in decode order.

    Per layer: q/k/v share the layer input (one fused launch), o reads q's
    output, gate/up share o's output (one fused launch), down reads up's
    output, and down's output is the next layer's input.  Attention, norms,
    activations and residuals are not part of the packed-linear path and are
    left out, so a step moves exactly the packed bytes plus activations.
    """

    def __init__(self, shapes, layers=None, device="cuda", seed=0, tp=None, **store_kw):
        """``tp=(rank, world)`` draws only this rank's tensor-parallel shards:
        column-parallel linears (q/k/v, gate/up) with out_features / world rows,
        row-parallel ones (o, down) with in_features / world columns."""
        self.shapes = shapes
        self.layers = layers if layers is not None else shapes.layers
        self.device = torch.device(device)
        self.blocks = []
        s = seed
        for _ in range(self.layers):
            blk = {}
            for name, n, k in shapes.linears():
                if tp is not None and tp[1] > 1:
                    world = tp[1]
                    if name in ("o_proj", "down_proj"):
                        if k % (world * 128):
                            raise ValueError(f"{name}: in_features {k} not splittable into {world} groups")
                        k //= world
                    else:
                        if n % world:
                            raise ValueError(f"{name}: out_features {n} not divisible by {world}")
                        n //= world
                blk[name] = make_store(n, k, device=device, seed=s, **store_kw)
                s += 1
            self.blocks.append(blk)

    @classmethod
    def from_blocks(cls, shapes, blocks, device):
        """A stack over given per-layer stores (e.g. tensor-parallel shards of another stack)."""
        self = cls.__new__(cls)
        self.shapes, self.blocks, self.layers = shapes, blocks, len(blocks)
        self.device = torch.device(device)
        return self

    def chain_steps(self):
        """(stores, feed) per launch: the store that feeds the next launch.

        q feeds o, up feeds down, down feeds the next layer's q/k/v.
        """
        steps = []
        for b in self.blocks:
            steps += [([b["q_proj"], b["k_proj"], b["v_proj"]], 0), ([b["o_proj"]], 0),
                      ([b["gate_proj"], b["up_proj"]], 1), ([b["down_proj"]], 0)]
        return steps

    def groups(self):
        """The launches of one step: lists of stores that share an input."""
        out = []
        for b in self.blocks:
            out += [[b["q_proj"], b["k_proj"], b["v_proj"]], [b["o_proj"]],
                    [b["gate_proj"], b["up_proj"]], [b["down_proj"]]]
        return out

    def algorithmic_bytes(self, m=1, act_bytes=2):
        """Bytes one step must move: indices, scales, codebooks, activations in and out.

        A launch reads its shared activation once and writes each store's output.
        """
        total = 0
        for grp in self.groups():
            total += m * grp[0].in_features * act_bytes
            for st in grp:
                total += store_bytes(st) + m * st.out_features * act_bytes
        return total

    def flops(self, m=1):
        return 2 * m * sum(st.out_features * st.in_features
                           for b in self.blocks for st in b.values())

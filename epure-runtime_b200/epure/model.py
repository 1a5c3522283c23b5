"""A decoder around the packed linears, for whole-model greedy decoding.

The reference runs Hugging Face decoders whose ``nn.Linear`` modules ``apply_to``
swapped for ``PackedLinear`` (epure/runtime.py:214-305, 98-126); attention,
norms, embedding and lm_head stay dense.  ``PackedDecoder`` is that model family
written out directly -- the Llama-3 / Qwen3 block: RMSNorm, q/k/v, (Qwen3:
per-head q/k RMSNorm), RoPE, grouped-query attention over a static KV cache, o,
residual, RMSNorm, SwiGLU gate/up/down, residual; final RMSNorm; lm_head -- so
that a decode step has static shapes and can be captured in one CUDA graph.
Per token the ``7 x layers`` packed linears run through libepq.so, and so do the
block's non-linear parts at decode (include/epq_decode.h: RMSNorm, q/k norm +
RoPE + KV write, attention, SiLU * up, the residual adds): by default every
layer is five launches (epq_decode_linear / epq_attn_rope_decode); with
``program=True`` the same steps of all layers run inside ONE persistent kernel
per token (epq_program_run); ``fused_glue=False`` runs the glue as torch ops.  The prompt (prefill) and the lm_head use torch.

Weights are random (no checkpoints offline): the packed stores of
``synthetic.LinearStack``, a bf16 N(0, 0.02) embedding (tied to lm_head for
Qwen3, a separate one for Llama-3), RMSNorm weights 1.

``linear_mode`` picks how the packed linears are computed, on the same stores:

* ``"ours"``: libepq.so (tensor-core GEMV up to 16 rows, tcgen05 GEMM above);
* ``"reference"``: the reference's fallback, ``F.linear(x, store.materialize(x.dtype))``
  (runtime.py:123-124), bf16 activations;
* ``"fp32"``: the same model in float32 throughout (weights materialised in
  float32: cb * scale exactly), the arithmetic both others approximate.

Logits are float32 in every mode: by default from a float32 lm_head (the parity
checks compare argmaxes); ``fp32_logits=False`` runs the bf16 lm_head GEMV as a
serving stack would (lm_head is not a packed linear).
"""
import math

import torch
import torch.nn.functional as F

from . import _native
from .synthetic import LinearStack

_ROPE_THETA = {"qwen3-1.7b": 1.0e6, "llama3-8b": 5.0e5, "llama3-70b": 5.0e5}
_EPS = {"qwen3-1.7b": 1e-6, "llama3-8b": 1e-5, "llama3-70b": 1e-5}


class PackedDecoder:
    def __init__(self, shapes, layers=None, device="cuda", seed=0, max_len=512,
                 linear_mode="ours", stack=None, embed=None, lm_head=None, fp32_logits=True,
                 fused_glue=True, gpu_layout="mma16", program=False):
        if linear_mode not in ("ours", "reference", "fp32"):
            raise ValueError("linear_mode must be 'ours', 'reference' or 'fp32'")
        self.shapes = shapes
        self.device = torch.device(device)
        self.mode = linear_mode
        self.dtype = torch.float32 if linear_mode == "fp32" else torch.bfloat16
        self.stack = stack if stack is not None else LinearStack(
            shapes, layers=layers, device=device, seed=seed, gpu_layout=gpu_layout)
        self.layers = self.stack.layers
        self.max_len = max_len
        h, hd = shapes.hidden, shapes.head_dim
        self.qk_norm = shapes.name.startswith("qwen3")
        self.eps = _EPS.get(shapes.name, 1e-6)
        if embed is None:
            g = torch.Generator(device=self.device).manual_seed(seed + 7919)
            embed = (torch.randn(shapes.vocab, h, generator=g, device=self.device) * 0.02
                     ).to(torch.bfloat16)
            if not shapes.name.startswith("qwen3"):
                lm_head = (torch.randn(shapes.vocab, h, generator=g, device=self.device) * 0.02
                           ).to(torch.bfloat16)
        self.embed = embed
        self.lm_head = lm_head if lm_head is not None else embed      # tied for Qwen3
        self.lm_head_f32 = None
        self.fp32_logits = fp32_logits
        self.fused_glue = fused_glue and linear_mode == "ours"
        theta = _ROPE_THETA.get(shapes.name, 1.0e6)
        inv = 1.0 / (theta ** (torch.arange(0, hd, 2, device=self.device, dtype=torch.float64) / hd))
        ang = torch.arange(max_len, device=self.device, dtype=torch.float64)[:, None] * inv[None, :]
        self.cos, self.sin = torch.cos(ang).float(), torch.sin(ang).float()   # [max_len, hd/2]
        kv = (self.layers, max_len, shapes.kv_heads, hd)
        self.k_cache = torch.zeros(kv, dtype=self.dtype, device=self.device)
        self.v_cache = torch.zeros(kv, dtype=self.dtype, device=self.device)
        self.key_pos = torch.arange(max_len, device=self.device)
        self._graph = None
        if self.fused_glue:
            self.attn_ws = _native.attn_decode_workspace(shapes.heads, shapes.kv_heads, hd, self.device)
            self.arg_ws = _native.argmax_workspace(self.device)
        self._fusable = all(st.layout == "mma16" for b in self.stack.blocks for st in b.values())
        # One persistent kernel per token (epq_program_*) instead of five launches per layer.
        self.use_program = program and self._fusable and self.fused_glue and self.dtype == torch.bfloat16
        self._program = None

    def share_weights(self, linear_mode):
        """The same model (stores, embedding, lm_head) with another linear mode."""
        return PackedDecoder(self.shapes, device=self.device, max_len=self.max_len,
                             linear_mode=linear_mode, stack=self.stack, embed=self.embed,
                             lm_head=self.lm_head, fp32_logits=self.fp32_logits,
                             fused_glue=self.fused_glue or linear_mode != "ours")

    # -- pieces ------------------------------------------------------------------
    def _lin(self, x, stores):
        if self.mode == "ours":
            return _native.linear_multi(x, stores)
        wdt = torch.float32 if self.mode == "fp32" else x.dtype
        return [F.linear(x, st.materialize(wdt)) for st in stores]

    def _rms(self, x):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)).to(x.dtype)

    def _rope(self, x, pos):
        # x [T, heads, hd] (rotate-half convention), pos [T]
        c, s = self.cos[pos][:, None, :], self.sin[pos][:, None, :]
        xf = x.float()
        half = x.shape[-1] // 2
        x1, x2 = xf[..., :half], xf[..., half:]
        return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1).to(x.dtype)

    def _logits(self, hl):
        if not self.fp32_logits:                    # bf16 lm_head GEMV, float32 result
            return F.linear(hl.to(self.lm_head.dtype), self.lm_head)[0].float()
        if self.lm_head_f32 is None:
            self.lm_head_f32 = self.lm_head.float()
        return (hl.float() @ self.lm_head_f32.T)[0]

    def _decode_fused(self, ids, pos):
        """One token with libepq.so's fused decode kernels.  With the tensor-core
        layout (``gpu_layout="mma16"``) a layer is five launches of
        epq_decode_linear / epq_attn_rope_decode (include/epq_decode.h):

        * q/k/v with the input RMSNorm as its prologue;
        * RoPE + KV write + attention;
        * o, added into the residual stream in its epilogue;
        * gate/up with the RMSNorm prologue and a SiLU(gate) * up epilogue;
        * down, added into the residual stream.

        The rounding points are the reference block's: every linear output,
        the residual after each add, the normed input and SiLU * up are rounded
        to bf16.  Other layouts use the unfused launches (linear_multi + glue)."""
        sh = self.shapes
        H, hd = sh.heads, sh.head_dim
        if not self._fusable:
            return self._decode_unfused(ids, pos)
        h = self.embed[ids].contiguous()                               # residual stream [1, hidden]
        for li, b in enumerate(self.stack.blocks):
            q, k, v = _native.decode_linear(h, [b["q_proj"], b["k_proj"], b["v_proj"]],
                                            prologue=_native.PRO_RMSNORM, eps=self.eps)
            att = _native.attn_rope_decode(q.view(H, hd), k.view(-1, hd), v.view(-1, hd), pos, self.cos,
                                           self.sin, self.k_cache[li], self.v_cache[li], self.qk_norm,
                                           self.eps, 1.0 / math.sqrt(hd), self.attn_ws)
            _native.decode_linear(att.view(1, H * hd), [b["o_proj"]], epilogue=_native.EPI_RESIDUAL,
                                  outs=[h])
            (a,) = _native.decode_linear(h, [b["gate_proj"], b["up_proj"]], prologue=_native.PRO_RMSNORM,
                                         epilogue=_native.EPI_SILU_MUL, eps=self.eps)
            _native.decode_linear(a, [b["down_proj"]], epilogue=_native.EPI_RESIDUAL, outs=[h])
        return self._logits(_native.add_rmsnorm(h, eps=self.eps))

    def _build_program(self):
        """Records every layer's five fused steps (as ``_decode_fused`` launches
        them) into one decode program over fixed buffers."""
        sh = self.shapes
        H, KV, hd = sh.heads, sh.kv_heads, sh.head_dim
        dev, bf = self.device, torch.bfloat16
        self._ph = torch.zeros(1, sh.hidden, dtype=bf, device=dev)        # residual stream
        self._ppos = torch.zeros(1, dtype=torch.long, device=dev)
        q = torch.empty(H * hd, dtype=bf, device=dev)
        k = torch.empty(KV * hd, dtype=bf, device=dev)
        v = torch.empty(KV * hd, dtype=bf, device=dev)
        att = torch.empty(H * hd, dtype=bf, device=dev)
        act = torch.empty(sh.intermediate, dtype=bf, device=dev)
        prog = _native.DecodeProgram(dev)
        for li, b in enumerate(self.stack.blocks):
            prog.linear(self._ph, [b["q_proj"], b["k_proj"], b["v_proj"]], [q, k, v],
                        prologue=_native.PRO_RMSNORM, eps=self.eps)
            prog.attention(q.view(H, hd), k.view(KV, hd), v.view(KV, hd), self._ppos, self.cos, self.sin,
                           self.k_cache[li], self.v_cache[li], self.qk_norm, self.eps, 1.0 / math.sqrt(hd),
                           att.view(H, hd))
            prog.linear(att, [b["o_proj"]], [self._ph], epilogue=_native.EPI_RESIDUAL)
            prog.linear(self._ph, [b["gate_proj"], b["up_proj"]], [act], prologue=_native.PRO_RMSNORM,
                        epilogue=_native.EPI_SILU_MUL, eps=self.eps)
            prog.linear(act, [b["down_proj"]], [self._ph], epilogue=_native.EPI_RESIDUAL)
        self._program = prog.finalize()

    def _decode_program(self, ids, pos):
        """One token as ONE persistent kernel (epq_program_run) plus the final
        RMSNorm, lm_head and the token's input copies: the same steps and
        rounding points as ``_decode_fused``."""
        if self._program is None:
            self._build_program()
        torch.index_select(self.embed, 0, ids.reshape(-1), out=self._ph)
        self._ppos.copy_(pos.reshape(-1)[:1])
        self._program.run()
        return self._logits(_native.add_rmsnorm(self._ph, eps=self.eps))

    def _decode_unfused(self, ids, pos):
        """One token with the per-linear launches and the separate glue kernels
        (residual add + RMSNorm, RoPE + KV write + attention, SiLU * up)."""
        sh = self.shapes
        H, hd = sh.heads, sh.head_dim
        x = self.embed[ids]                                            # [1, hidden]
        y = _native.add_rmsnorm(x, eps=self.eps)
        for li, b in enumerate(self.stack.blocks):
            q, k, v = _native.linear_multi(y, [b["q_proj"], b["k_proj"], b["v_proj"]])
            att = _native.attn_rope_decode(q.view(H, hd), k.view(-1, hd), v.view(-1, hd), pos, self.cos,
                                           self.sin, self.k_cache[li], self.v_cache[li], self.qk_norm,
                                           self.eps, 1.0 / math.sqrt(hd), self.attn_ws)
            (o,) = _native.linear_multi(att.view(1, H * hd), [b["o_proj"]])
            y = _native.add_rmsnorm(x, add=o, h_out=x, eps=self.eps)   # x += o; y = rms(x)
            g, u = _native.linear_multi(y, [b["gate_proj"], b["up_proj"]])
            (d,) = _native.linear_multi(_native.silu_mul(g, u), [b["down_proj"]])
            y = _native.add_rmsnorm(x, add=d, h_out=x, eps=self.eps)   # next layer's input norm
        return self._logits(y)

    def forward(self, ids, pos):
        """Logits (float32) of the last position of ``ids`` [T] at positions ``pos`` [T];
        writes the KV cache at those positions.  Static shapes for a fixed T."""
        if self.mode == "ours" and ids.shape[0] == 1 and self.fused_glue:
            if self.use_program:
                return self._decode_program(ids, pos)
            return self._decode_fused(ids, pos)
        sh = self.shapes
        T = ids.shape[0]
        H, KV, hd = sh.heads, sh.kv_heads, sh.head_dim
        x = self.embed[ids].to(self.dtype)
        allowed = (self.key_pos[None, :] <= pos[:, None])[None, None]     # [1, 1, T, max_len]
        for li, b in enumerate(self.stack.blocks):
            hcur = self._rms(x)
            q, k, v = self._lin(hcur, [b["q_proj"], b["k_proj"], b["v_proj"]])
            q, k, v = q.view(T, H, hd), k.view(T, KV, hd), v.view(T, KV, hd)
            if self.qk_norm:
                q, k = self._rms(q), self._rms(k)
            q, k = self._rope(q, pos), self._rope(k, pos)
            self.k_cache[li].index_copy_(0, pos, k)
            self.v_cache[li].index_copy_(0, pos, v)
            att = F.scaled_dot_product_attention(
                q.transpose(0, 1)[None], self.k_cache[li].transpose(0, 1)[None],
                self.v_cache[li].transpose(0, 1)[None], attn_mask=allowed,
                scale=1.0 / math.sqrt(hd), enable_gqa=True)               # [1, H, T, hd]
            att = att[0].transpose(0, 1).reshape(T, H * hd)
            (o,) = self._lin(att, [b["o_proj"]])
            x = x + o
            hcur = self._rms(x)
            g, u = self._lin(hcur, [b["gate_proj"], b["up_proj"]])
            (d,) = self._lin((F.silu(g.float()) * u.float()).to(self.dtype), [b["down_proj"]])
            x = x + d
        return self._logits(self._rms(x[-1:]))

    # -- decoding ------------------------------------------------------------------
    def _check_capacity(self, positions, what):
        if positions > self.max_len:
            raise ValueError(f"epure: {what} needs {positions} KV-cache positions; this decoder holds "
                             f"max_len={self.max_len}")

    def prefill(self, prompt):
        """Runs the prompt (long tensor [T]); returns the logits after its last token."""
        self._check_capacity(prompt.shape[0], "the prompt")
        pos = torch.arange(prompt.shape[0], device=self.device)
        return self.forward(prompt.to(self.device), pos)

    def step(self, token, pos):
        """One decode step for a device scalar token at device position ``pos`` ([1] each)."""
        return self.forward(token, pos)

    def capture(self, warmup=2):
        """Captures one greedy step in a CUDA graph: reads ``self.tok`` / ``self.pos``,
        writes the argmax into ``self.tok`` and advances ``self.pos``."""
        self.tok = torch.zeros(1, dtype=torch.long, device=self.device)
        self.pos = torch.zeros(1, dtype=torch.long, device=self.device)
        self.logits = None
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(warmup):
                self._greedy_body()
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._greedy_body()
        self._graph = g
        return self

    def _greedy_body(self):
        self.logits = self.step(self.tok, self.pos)
        if self.fused_glue:
            _native.argmax(self.logits, self.tok, self.arg_ws)
        else:
            self.tok.copy_(torch.argmax(self.logits).view(1))
        self.pos.add_(1)

    def generate(self, prompt, n_new, graph=True):
        """Greedy decode: ``n_new`` tokens after ``prompt`` (returns a long tensor).

        The prompt and the new tokens must fit the KV cache (``max_len``); the
        graphed step also checks its device-side position on every replay."""
        self._check_capacity(prompt.shape[0] + n_new, f"a {prompt.shape[0]}-token prompt + {n_new} new tokens")
        first = int(torch.argmax(self.prefill(prompt)))
        out = [first]
        if graph:
            if self._graph is None:
                raise RuntimeError("call capture() first")
            self.tok.fill_(first)
            self.pos.fill_(prompt.shape[0])
            toks = torch.empty(n_new, dtype=torch.long, device=self.device)
            toks[0] = first
            for t in range(1, n_new):
                self._graph.replay()
                toks[t:t + 1].copy_(self.tok)
            return toks
        tok = torch.tensor([first], device=self.device)
        for t in range(n_new - 1):
            pos = torch.tensor([prompt.shape[0] + t], device=self.device)
            tok = torch.argmax(self.step(tok, pos)).view(1)
            out.append(int(tok))
        return torch.tensor(out, device=self.device)

    def teacher_forced_logits(self, prompt, tokens):
        """Float32 logits [len(tokens), vocab] after the prompt and after each of
        ``tokens[:-1]`` fed in order: the prediction for every position of ``tokens``
        given the true prefix."""
        self._check_capacity(prompt.shape[0] + tokens.shape[0], "teacher forcing")
        out = torch.empty(tokens.shape[0], self.shapes.vocab, device=self.device)
        out[0] = self.prefill(prompt)
        T0 = prompt.shape[0]
        for t in range(tokens.shape[0] - 1):
            pos = torch.tensor([T0 + t], device=self.device)
            out[t + 1] = self.step(tokens[t:t + 1].to(self.device), pos)
        return out

    def teacher_forced_argmax(self, prompt, tokens):
        return torch.argmax(self.teacher_forced_logits(prompt, tokens), dim=-1).cpu()


class PackedCausalLM(torch.nn.Module):
    """The same decoder as a trainable module tree, for compressed-state fine-tuning.

    The reference fine-tunes a Hugging Face causal LM whose linears ``apply_to``
    swapped for PackedLinear (epure/finetune.py:49-176, fine-tuning/codebook.py):
    ``make_trainable`` promotes every store's scales and codebook to fp32
    parameters, the indices stay frozen, and the loss is next-token
    cross-entropy.  This is that model family written out: a bf16 embedding
    (tied to the lm_head for Qwen3, a separate one for Llama-3; both frozen),
    per layer RMSNorm, q/k/v (with per-head q/k RMSNorm for Qwen3), RoPE,
    causal grouped-query attention (torch SDPA), o, residual, RMSNorm, SwiGLU
    gate/up/down, residual; final RMSNorm, lm_head, cross-entropy.  Every
    projection is a ``PackedLinear`` over the stores of ``decoder.stack``, so on
    a GPU it runs libepq.so's tensor-core GEMM forward and its fused
    compressed-state backward (dX, dscale, dcb; dW never formed).
    ``linear_mode="reference"`` instead differentiates the reference's fallback
    ``F.linear(x, materialize(bf16))`` (runtime.py:78-89, 123-124) with torch
    ops, the formulation the gradients are checked against.

    ``forward(input_ids [B, T], labels=None)`` returns an object with ``.loss``
    (labels default to the inputs, shifted by one inside), so ``ScaleTuner``
    can drive it."""

    def __init__(self, decoder, linear_mode="ours"):
        super().__init__()
        import types
        from .runtime import PackedLinear
        if linear_mode not in ("ours", "reference"):
            raise ValueError("linear_mode must be 'ours' or 'reference'")
        self._types = types
        self.shapes = decoder.shapes
        self.mode = linear_mode
        self.eps = decoder.eps
        self.qk_norm = decoder.qk_norm
        self.cos, self.sin = decoder.cos, decoder.sin
        self.register_buffer("embed_w", decoder.embed.detach(), persistent=False)
        self.register_buffer("head_w", decoder.lm_head.detach(), persistent=False)
        self.layers = torch.nn.ModuleList()
        for b in decoder.stack.blocks:
            blk = torch.nn.Module()
            for name, st in b.items():
                setattr(blk, name, PackedLinear(st))
            self.layers.append(blk)

    def _lin(self, mod, x):
        if self.mode == "ours":
            return mod(x)
        return F.linear(x, mod.store.materialize(x.dtype))

    def _rms(self, x):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)).to(x.dtype)

    def _rope(self, x):
        # x [B, T, heads, hd], positions 0..T-1 (rotate-half)
        T = x.shape[1]
        c, s = self.cos[:T][None, :, None, :], self.sin[:T][None, :, None, :]
        xf = x.float()
        half = x.shape[-1] // 2
        x1, x2 = xf[..., :half], xf[..., half:]
        return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1).to(x.dtype)

    def logits(self, input_ids):
        """bf16 logits [B, T, vocab] of every position (causal)."""
        sh = self.shapes
        B, T = input_ids.shape
        H, KV, hd = sh.heads, sh.kv_heads, sh.head_dim
        if T > self.cos.shape[0]:
            raise ValueError(f"epure: sequence of {T} tokens exceeds the rotary table ({self.cos.shape[0]})")
        x = F.embedding(input_ids, self.embed_w)                              # [B, T, hidden] bf16
        for blk in self.layers:
            h = self._rms(x)
            q = self._lin(blk.q_proj, h).view(B, T, H, hd)
            k = self._lin(blk.k_proj, h).view(B, T, KV, hd)
            v = self._lin(blk.v_proj, h).view(B, T, KV, hd)
            if self.qk_norm:
                q, k = self._rms(q), self._rms(k)
            q, k = self._rope(q), self._rope(k)
            att = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                                 is_causal=True, scale=1.0 / math.sqrt(hd), enable_gqa=True)
            att = att.transpose(1, 2).reshape(B, T, H * hd)
            x = x + self._lin(blk.o_proj, att)
            h = self._rms(x)
            g, u = self._lin(blk.gate_proj, h), self._lin(blk.up_proj, h)
            x = x + self._lin(blk.down_proj, (F.silu(g.float()) * u.float()).to(x.dtype))
        return F.linear(self._rms(x), self.head_w)

    def forward(self, input_ids, labels=None):
        """Next-token cross-entropy (fp32 softmax over bf16 logits) of ``labels``
        (default ``input_ids``) shifted by one."""
        logits = self.logits(input_ids)
        labels = input_ids if labels is None else labels
        loss = F.cross_entropy(logits[:, :-1].reshape(-1, logits.shape[-1]).float(),
                               labels[:, 1:].reshape(-1))
        return self._types.SimpleNamespace(loss=loss)

"""Benchmark: batch-1 greedy decode of a Llama-3-8B-shaped codebook-quantized model.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N = 1 (the headline).  One step is one whole decode
token of ``epure.model.PackedDecoder`` on Llama-3-8B shapes with random weights
in the benchmark's format (u8 index per 4-weight vector, 256x4 fp16 codebook,
fp16 scale per row per 128 weights; bf16 embedding and lm_head): the embedding
row, then per layer five launches of libepq.so -- q/k/v with the input RMSNorm
fused in, RoPE + KV-cache write + attention, o added into the residual, gate/up
with the RMSNorm and SiLU(gate)*up fused in, down added into the residual --
then the final RMSNorm, the bf16 lm_head (cuBLAS), argmax and the position
update, all replayed from one CUDA graph after a 128-token prompt.  Every
packed weight is decoded exactly as the reference's bf16 path decodes it.  The
2.9 GB the step streams are far larger than the 126 MB L2, so no flush is
needed.
  value      tokens/s over K graph replays (the token stays on the device);
  e2e        the same through the public step with the token copied in from
             pinned host memory and the next token read back every step;
  roofline   the dominant kernel, gemv_mma_kernel: the token's 128 packed
             launches replayed alone (epure.decode.GraphedLinearStack over the
             same stores), algorithmic bytes / their CUDA-event time;
  token_roofline  the whole token's bytes (packed + lm_head + embedding row +
             KV read) / token time -- the north-star basis (2,904.6 MB/token);
  cpu_baseline    the reference's CPU path on whole tokens (below), rank 0.

N > 1.  Llama-3-70B shapes (config 4) tensor-parallel over the N GPUs: every
packed linear of a token on each rank's shards in ONE persistent launch of the
chain kernel per rank, the all-reduce after o and down done inside the kernel
over NVLink (peer loads; no NCCL launch on the data path); strong scaling.
Before timing, rank 0 checks the TP chain against the single-GPU chain on a
2-layer slice of the same model (full width) and prints the error as
``tp_check``; past 1e-4 every rank exits non-zero.  ``--replicas`` runs N
independent copies of the N = 1 workload instead (weak scaling).

Reference arm (--impl reference; rank 0 alone, the other ranks exit 0): the
reference's CPU implementation of the path on every host thread -- each packed
linear through the C restatement of its fused Rust kernel (kernel/src/lib.rs,
oracle/epq_oracle.c; f32 activations, as lib.rs takes), the rest of the block
(RMSNorm, RoPE, attention over the KV cache, SiLU, lm_head) in numpy float32.
N = 1: one whole 8B token per step.  N > 1: the 70B shapes' packed linears of
8 of the 80 layers per step (tok/s = 1 / (10 x step)); the sample is named in
``cpu_baseline.sample``.  It imports nothing from the epure package.

Other workloads (each prints its own metric): --mode chain (the packed linears
only, as one persistent chain launch per token, fp32 between layers), --mode
per-linear [--batch B] (the per-linear GEMV / GEMM launches), --mode prefill
[--tokens 2048], --mode finetune [--batch 8 --seq 2048] (the whole Qwen3-1.7B
model: forward, cross-entropy, backward, AdamW), --mode embedding;
--model / --layers pick the shapes; --fallback also times the reference's bf16
GPU fallback (materialize + F.linear, torch ops) on the same step.
"""
import argparse
import json
import os
import statistics
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "epure-runtime_b200"))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s bs1 @8B; dequant-GEMV HBM GB/s as % of B200 peak"
UNIT = "tok/s"
PROMPT = 128

# The decoder shapes (name, layers, hidden, intermediate, heads, kv heads, head dim,
# vocab) -- copied here so the reference arm needs nothing from the epure package.
SHAPES = {
    "qwen3-1.7b": ("qwen3-1.7b", 28, 2048, 6144, 16, 8, 128, 151936),
    "llama3-8b": ("llama3-8b", 32, 4096, 14336, 32, 8, 128, 128256),
    "llama3-70b": ("llama3-70b", 80, 8192, 28672, 64, 8, 128, 128256),
}
ROPE_THETA = {"qwen3-1.7b": 1.0e6, "llama3-8b": 5.0e5, "llama3-70b": 5.0e5}
RMS_EPS = {"qwen3-1.7b": 1e-6, "llama3-8b": 1e-5, "llama3-70b": 1e-5}

# DRAM traffic / algorithmic bytes of the dominant kernel, from one ncu capture
# (profiles/): per-linear = gemv_mma_kernel on a Llama-3-8B gate+up launch
# (dram__bytes_read.sum + dram__bytes_write.sum over the launch's algorithmic
# bytes); chain = chain_kernel on a 4-layer chain.
NCU_TRAFFIC_RATIO = {"per-linear": 31249152 / 31264768,
                     "chain": (232708096 + 5034240) / 232349696,
                     "program": None}


def _traffic(ratio, algorithmic_bytes, full):
    """The roofline's `traffic`: the ncu-measured DRAM bytes / algorithmic bytes of
    the kernel (a small capture, profiles/) times this launch's algorithmic bytes."""
    if ratio is None or not full:
        return {"traffic": None, "traffic_note": "no ncu capture of this kernel at this size"}
    return {"traffic": int(algorithmic_bytes * ratio),
            "traffic_note": "ncu dram bytes / algorithmic bytes of a small capture (profiles/), "
                            "times this launch's algorithmic bytes"}


def linears(shape):
    """(name, out_features, in_features) of one layer's packed linears."""
    _, _, h, i, heads, kv, hd, _ = shape
    return [("q_proj", heads * hd, h), ("k_proj", kv * hd, h), ("v_proj", kv * hd, h),
            ("o_proj", h, heads * hd), ("gate_proj", i, h), ("up_proj", i, h), ("down_proj", h, i)]


def workload(args, world):
    """(workload name, config dict) shared by both arms, so the two lines compare."""
    shape = SHAPES[args.model]
    layers = args.layers or shape[1]
    part = f" (first {layers} of {shape[1]} layers)" if layers != shape[1] else ""
    if args.mode == "model":
        name = f"{args.model} whole-model greedy decode token, batch 1, after a {PROMPT}-token prompt{part}"
        par = f"replicas x{world}" if world > 1 else "single GPU"
    else:   # tp chain
        name = f"{args.model} packed linears of one batch-1 decode token, tensor-parallel{part}"
        par = f"tp{world}"
    cfg = {"workload": name, "mode": args.mode if not args.tp else "tp-chain", "model": args.model,
           "layers": layers, "global_batch": world if (args.mode == "model" and world > 1) else 1,
           "seq_len": PROMPT + args.warmup + args.steps + 2 if args.mode == "model" else 1,
           "parallelism": par, "l2": "inputs larger than L2 (no flush needed)"}
    return name, cfg


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def _tensor_peak():
    """Sustained bf16 tensor throughput (a kernel timed inside a long step)."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["bf16_tflops_sustained"]), "measured (sustained)"
    except Exception:
        return 1400.0, "fallback (sustained)"


class ClockSampler:
    """SM clock, power and clock-event reasons of one GPU, polled from NVML every
    few milliseconds while the timed region runs (nvidia-smi's 200 ms loop sees
    too few samples of a tens-of-milliseconds region)."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, device_index, interval_s=0.004):
        self.device_index, self.interval = device_index, interval_s
        self.samples, self.max_mhz, self._thread, self._stop = [], None, None, False

    def _handle(self, nv):
        import torch
        try:
            p = torch.cuda.get_device_properties(self.device_index)
            bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
            return nv.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return nv.nvmlDeviceGetHandleByIndex(self.device_index)

    def _sample(self):
        nv, h = self._nv, self._h
        try:
            sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
            reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
            power = nv.nvmlDeviceGetPowerUsage(h) / 1000.0
            self.samples.append((sm, reasons, power))
        except Exception:
            pass

    def _run(self):
        while not self._stop:
            self._sample()
            time.sleep(self.interval)

    def __enter__(self):
        # The sampler thread competes for the GIL with the launching loop: a
        # 1 ms switch interval lets it in, and the region opens only once the
        # first sample is in; __exit__ adds one more taken before the GPU idles.
        self._switch = sys.getswitchinterval()
        try:
            import threading
            import pynvml as nv
            nv.nvmlInit()
            self._nv, self._h = nv, self._handle(nv)
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(self._h, nv.NVML_CLOCK_SM)
            sys.setswitchinterval(0.001)
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
            t0 = time.time()
            while not self.samples and time.time() - t0 < 0.5:
                time.sleep(0.001)
        except Exception:
            self._thread = None
        return self

    def __exit__(self, *a):
        if self._thread is not None:
            self._sample()
        self._stop = True
        if self._thread is not None:
            self._thread.join(timeout=2)
        sys.setswitchinterval(self._switch)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["no samples"]}
        reasons = set()
        for _, bits, _ in self.samples:
            reasons |= {name for bit, name in self.REASONS.items() if bits & bit}
        return {"sm_mhz": statistics.median(s for s, _, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(self.samples),
                "power_w_max": round(max(p for _, _, p in self.samples), 1), "source": "nvml"}


# ---------------------------------------------------------------------------
# the reference's CPU path (reference arm and cpu_baseline)
# ---------------------------------------------------------------------------
def host_threads():
    """Every host thread this process may run on (torchrun sets OMP_NUM_THREADS=1
    for its ranks; the reference's rayon pool ignores that and uses all cores)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


class CpuReferenceDecoder:
    """One batch-1 decode token the way the reference runs it on the CPU.

    Every packed linear is the reference's fused CPU kernel (kernel/src/lib.rs:
    96-151, restated in C in oracle/epq_oracle.c: per output row and group a
    table of cb * scale, an f32 sum over the group, group sums in order), with
    f32 activations as that kernel takes them; the rest of the Llama / Qwen3
    block (RMSNorm, RoPE, grouped-query attention over a KV cache, SiLU * up,
    residuals, final norm, lm_head, argmax) is numpy float32, standing in for
    the Hugging Face modules around the reference's PackedLinear.  Weights are
    seeded random in the benchmark's format.  ``linears_only`` keeps just the
    packed linears chained output to input (the tensor-parallel workload)."""

    def __init__(self, shape, layers, threads, max_len=PROMPT + 64, seed=0, linears_only=False):
        import numpy as np
        from oracle import oracle as O
        self.np, self.O = np, O
        O.build_c_oracle()
        self.shape, self.layers, self.threads = shape, layers, threads
        self.linears_only = linears_only
        name, _, h, inter, heads, kv, hd, vocab = shape
        rng = np.random.default_rng(seed)
        self.blocks = []
        for _ in range(layers):
            blk = {}
            for lname, n, k in linears(shape):
                idx = rng.integers(0, 256, (n, k // 4), dtype=np.uint8)
                cb = rng.standard_normal((256, 4), dtype=np.float32).astype(np.float16).astype(np.float32)
                sc = np.abs(rng.normal(0, 0.02, (n, k // 128))).astype(np.float16).astype(np.float32)
                blk[lname] = (idx, sc, cb, n, k)
            self.blocks.append(blk)
        self.h, self.heads, self.kv, self.hd = h, heads, kv, hd
        self.eps, self.qk_norm = RMS_EPS.get(name, 1e-6), name.startswith("qwen3")
        if not linears_only:
            self.embed = (rng.standard_normal((vocab, h), dtype=np.float32) * 0.02).astype(np.float32)
            self.lm_head = self.embed if name.startswith("qwen3") else \
                (rng.standard_normal((vocab, h), dtype=np.float32) * 0.02).astype(np.float32)
            inv = 1.0 / (ROPE_THETA.get(name, 1e6) ** (np.arange(0, hd, 2, dtype=np.float64) / hd))
            ang = np.arange(max_len, dtype=np.float64)[:, None] * inv[None, :]
            self.cos, self.sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
            self.kc = np.zeros((layers, max_len, kv, hd), np.float32)
            self.vc = np.zeros((layers, max_len, kv, hd), np.float32)
            # a filled prompt: random K/V rows stand in for the 128 prefill positions
            self.kc[:, :PROMPT] = rng.standard_normal((layers, PROMPT, kv, hd), dtype=np.float32)
            self.vc[:, :PROMPT] = rng.standard_normal((layers, PROMPT, kv, hd), dtype=np.float32)
            self.pos = PROMPT

    def _lin(self, x, st):
        idx, sc, cb, n, k = st
        return self.O.c_dequant_matmul(x, idx, sc, cb, n, k, 4, 128, 256, threads=self.threads)

    def _rms(self, x):
        np = self.np
        return x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + self.eps)

    def _rope(self, x, p):
        np = self.np
        half = self.hd // 2
        c, s = self.cos[p], self.sin[p]
        x1, x2 = x[..., :half], x[..., half:]
        return np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s], axis=-1)

    def step_linears(self, x):
        for b in self.blocks:
            q = self._lin(x, b["q_proj"])
            self._lin(x, b["k_proj"])
            self._lin(x, b["v_proj"])
            o = self._lin(q, b["o_proj"])
            self._lin(o, b["gate_proj"])
            u = self._lin(o, b["up_proj"])
            x = self._lin(u, b["down_proj"])
        return x

    def step(self, token):
        """One greedy token (numpy int) -> the next token."""
        np = self.np
        if self.linears_only:
            return self.step_linears(np.ones((1, self.h), np.float32))
        p = self.pos
        x = self.embed[token][None, :].copy()
        g = self.heads // self.kv
        for li, b in enumerate(self.blocks):
            y = self._rms(x)
            q = self._lin(y, b["q_proj"]).reshape(self.heads, self.hd)
            k = self._lin(y, b["k_proj"]).reshape(self.kv, self.hd)
            v = self._lin(y, b["v_proj"]).reshape(self.kv, self.hd)
            if self.qk_norm:
                q, k = self._rms(q), self._rms(k)
            q, k = self._rope(q, p), self._rope(k, p)
            self.kc[li, p], self.vc[li, p] = k, v
            keys, vals = self.kc[li, :p + 1], self.vc[li, :p + 1]          # [T, kv, hd]
            qg = q.reshape(self.kv, g, self.hd)
            s = np.einsum("kgd,tkd->kgt", qg, keys) / np.sqrt(self.hd)
            s = np.exp(s - s.max(-1, keepdims=True))
            s /= s.sum(-1, keepdims=True)
            att = np.einsum("kgt,tkd->kgd", s, vals).reshape(1, -1)
            x = x + self._lin(att, b["o_proj"])
            y = self._rms(x)
            gt, up = self._lin(y, b["gate_proj"]), self._lin(y, b["up_proj"])
            x = x + self._lin(gt / (1.0 + np.exp(-gt)) * up, b["down_proj"])
        logits = self.lm_head @ self._rms(x)[0]
        self.pos = p + 1 if p + 1 < self.kc.shape[1] else PROMPT
        return int(np.argmax(logits))


def cpu_reference(shape, layers, threads, steps=None, seconds=None, warmup=1, linears_only=False):
    """(seconds per step list, decoder): timed steps of CpuReferenceDecoder."""
    dec = CpuReferenceDecoder(shape, layers, threads, linears_only=linears_only,
                              max_len=PROMPT + warmup + (steps or 64) + 2)
    tok = 1
    for _ in range(warmup):
        tok = dec.step(tok)
    times, t_all = [], time.perf_counter()
    while True:
        t0 = time.perf_counter()
        tok = dec.step(tok)
        times.append(time.perf_counter() - t0)
        if steps is not None and len(times) >= steps:
            break
        if seconds is not None and time.perf_counter() - t_all >= seconds:
            break
    return times, dec


def run_reference(args, rank, world):
    """The reference arm: rank 0 times the reference's CPU path on every host thread."""
    if rank != 0:
        return 0
    threads = host_threads()
    os.environ["OMP_NUM_THREADS"] = str(threads)
    shape = SHAPES[args.model]
    if args.mode == "model":
        layers = args.layers or shape[1]
        times, _ = cpu_reference(shape, layers, threads, steps=args.steps, warmup=args.warmup)
        per_tok = sum(times) / len(times)
        sample = (f"whole {args.model} decode tokens ({layers} layers, all {7 * layers} packed linears "
                  f"+ attention, norms, lm_head) on {threads} threads, {len(times)} timed steps")
    else:
        total = args.layers or shape[1]
        layers = min(8, total)
        times, _ = cpu_reference(shape, layers, threads, steps=args.steps, warmup=args.warmup,
                                 linears_only=True)
        scale = total / layers
        per_tok = scale * sum(times) / len(times)
        sample = (f"{args.model} packed linears of {layers} of {total} layers per step on {threads} "
                  f"threads ({len(times)} timed steps); tok/s = 1 / ({scale:g} x step time)")
    tok_s = 1.0 / per_tok
    _, cfg = workload(args, world)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(tok_s, 4), "unit": UNIT,
        "n_gpus": world, "steps": len(times), "warmup": args.warmup,
        "ms_per_step": round(1000.0 * sum(times) / len(times), 3), "higher_is_better": True,
        "scaling": "weak" if args.mode == "model" else "strong", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic", "config": cfg,
        "cpu_baseline": {"value": round(tok_s, 4), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(tok_s, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# other workloads
# ---------------------------------------------------------------------------
def time_fallback(stack, x, steps):
    """The reference's GPU path without its Triton kernel, on the same step.

    PackedLinear.forward falls back to F.linear(x, materialize(x.dtype))
    (epure/runtime.py:78-89, 123-124): the codebook cast to the activation type,
    gathered by index, multiplied by the row's group scale (repeat_interleave
    over the group), then one cuBLAS GEMM.  Run with torch ops, store by store,
    in the step's order; CUDA events around `steps` steps.
    """
    import torch
    import torch.nn.functional as F

    def weight(st):
        dt = x.dtype
        idx = st.index_rows().long()                                   # [n, k/4]
        w = st.cb.to(dt)[idx].reshape(st.out_features, -1)[:, :st.in_features]
        sc = st.scale.to(dt).repeat_interleave(st.group, dim=1)[:, :st.in_features]
        return w * sc

    def step():
        h = x
        for grp, feed in zip(stack.groups(), [0, 0, 1, 0] * len(stack.blocks)):
            outs = [F.linear(h, weight(st)) for st in grp]
            h = outs[feed]
        return h

    step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    return {"what": "reference bf16 fallback: F.linear(x, materialize(bf16)) per store (torch ops)",
            "ms_per_step": round(ms, 4), "value": round(x.shape[0] * 1000.0 / ms, 2), "unit": UNIT,
            "steps": steps}


def run_finetune(args, rank, world, local_rank):
    """One compressed-state fine-tuning step of the whole model (config 3).

    PackedCausalLM over random packed stores of ``args.model``'s shapes (Qwen3-1.7B
    by default: q/k RMSNorm, tied lm_head, GQA): make_trainable(mode="both")
    promotes every store's scales and codebook to fp32 parameters, and a step is
    forward over ``--batch`` sequences of ``--seq`` tokens, next-token
    cross-entropy, backward (libepq.so's packed GEMM forward and fused dX /
    dscale / dcb backward; torch SDPA, RMSNorm, SiLU, the bf16 lm_head and the
    softmax around them), and one fused AdamW update.  The reference's loop is
    ScaleTuner.step (finetune.py:135-176) on the same model."""
    import torch
    import torch.distributed as dist
    from epure import synthetic
    from epure.finetune import make_trainable
    from epure.model import PackedCausalLM, PackedDecoder

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    model_name = args.model
    shapes = synthetic.SHAPES[model_name]
    B, T = args.batch or 8, args.seq
    dec = PackedDecoder(shapes, layers=args.layers, device=dev, seed=1000 * rank, max_len=T,
                        fused_glue=False)
    model = PackedCausalLM(dec, "ours")
    params = make_trainable(model, "both")
    opt = torch.optim.AdamW(params, lr=1e-5, fused=True)
    g = torch.Generator(device=dev).manual_seed(rank)
    ids = torch.randint(0, shapes.vocab, (B, T), generator=g, device=dev)

    def step(batch):
        loss = model(batch).loss
        loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=True)
        return loss

    L = dec.layers
    m = B * T
    lin = dec.stack.flops(m)                                  # 2 m sum(n k) over the packed linears
    qkv0 = sum(2 * m * st.out_features * st.in_features
               for n_, st in dec.stack.blocks[0].items() if n_ in ("q_proj", "k_proj", "v_proj"))
    # forward + dscale/dcb contraction everywhere, dX everywhere but layer 0's q/k/v
    # (its input, the frozen embedding, needs no gradient)
    flops = 3 * lin - qkv0
    flops += 4 * m * shapes.vocab * shapes.hidden             # lm_head forward + dX
    flops += 7 * B * shapes.heads * T * T * shapes.head_dim * L   # causal attention fwd (2) + bwd (5) halves
    launches = 7 * L + 7 * L + (7 * L - 3)                    # forward, dscale/dcb, dX kernels of libepq.so

    for _ in range(args.warmup):
        step(ids)
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        ev0.record(stream)
        for _ in range(args.steps):
            step(ids)
        ev1.record(stream)
        torch.cuda.synchronize(dev)
    ms = ev0.elapsed_time(ev1) / args.steps
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    # end to end: the token batch from pinned host memory, the step, the loss read back
    idh = torch.empty(ids.shape, dtype=ids.dtype, pin_memory=True)
    idh.copy_(ids.cpu())
    lh = torch.empty(1, dtype=torch.float32, pin_memory=True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        loss = step(idh.to(dev, non_blocking=True))
        lh.copy_(loss.detach().view(1), non_blocking=True)
        stream.synchronize()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    tf_peak, tf_kind = _tensor_peak()
    achieved = flops / (ms * 1e-3) / 1e12
    if rank == 0:
        line = {
            "metric": f"fine-tune tok/s @{model_name} (whole model: fwd + CE + bwd + AdamW, "
                      f"{B}x{T} tokens/step)",
            "value": round(world * m * 1000.0 / ms, 2), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random packed stores, random token ids)",
            "config": {"workload": f"{model_name} whole-model compressed-state fine-tune step "
                                   f"({L} layers, {7 * L} packed linears, fp32 scales and codebooks, "
                                   f"make_trainable mode=both, AdamW)",
                       "mode": "finetune", "global_batch": world * B, "seq_len": T,
                       "parallelism": f"data-parallel replicas x{world}" if world > 1 else "single GPU",
                       "flops_per_step": flops, "final_loss": round(float(lh.item()), 4)},
            "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": tf_peak,
                         "unit": "TFLOP/s", "frac": round(achieved / tf_peak, 4), "peak_kind": tf_kind,
                         "kernel": "whole step (packed gemm_tc + bwd_dx_tc + bwd_dw_tc, SDPA, lm_head)",
                         "traffic": None},
            "e2e": {"value": round(world * m * 1000.0 / e2e_ms, 2), "unit": UNIT,
                    "h2d_bytes_per_step": ids.numel() * ids.element_size(), "d2h_bytes_per_step": 4},
            "gpu_launches": launches * args.steps,
            "clocks": clocks.summary(),
        }
        if args.fallback:
            line["fallback"] = time_fallback_finetune(dec, ids, steps=max(1, min(args.steps, 2)))
        print(json.dumps(line), flush=True)
    return 0


def time_fallback_finetune(dec, ids, steps):
    """The reference's fine-tuning autograd on the same model and batch (GPU, torch ops).

    make_trainable (finetune.py:49-102) + PackedLinear.forward's fallback
    F.linear(x, materialize(bf16)) (runtime.py:78-89, 123-124): torch autograd
    differentiates the gather/scale expansion and the GEMM; fp32 parameters,
    the same AdamW update.
    """
    import torch
    from epure.model import PackedCausalLM
    model = PackedCausalLM(dec, "reference")
    params = [p for b in model.layers for mod in b.children() for p in (mod.store.scale, mod.store.cb)]
    opt = torch.optim.AdamW(params, lr=1e-5, fused=True)

    def step():
        model(ids).loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=True)

    step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    return {"what": "reference fine-tune autograd: F.linear(x, materialize(bf16)) per store, "
                    "fp32 scale/codebook parameters (torch ops), same model and AdamW",
            "ms_per_step": round(ms, 3), "value": round(ids.numel() * 1000.0 / ms, 2), "unit": UNIT,
            "steps": steps}


def run_embedding(args, rank, world, local_rank):
    """Packed embedding rows (PackedEmbedding.forward -> epq_embedding) for a batch of
    `--tokens` ids from a vector-codebook table of the model's vocab x hidden."""
    import torch
    from epure import synthetic
    from epure.runtime import PackedEmbedding

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    shapes = synthetic.SHAPES[args.model]
    st = synthetic.make_store(shapes.vocab, shapes.hidden, device=dev, seed=1000 * rank)
    emb = PackedEmbedding(st, dtype=torch.bfloat16)
    n = args.tokens
    g = torch.Generator(device=dev).manual_seed(rank)
    # rotate over 64 id batches so the gathered rows do not stay in L2
    batches = [torch.randint(0, shapes.vocab, (n,), generator=g, device=dev) for _ in range(64)]

    def reference(ids):                    # the reference's torch formulation (runtime.py:129-160)
        flat = ids.reshape(-1)
        idx = st.index_rows(flat).to(torch.long)
        w = st.cb.reshape(st.levels, 4)[idx].reshape(flat.numel(), st.in_features).to(torch.bfloat16)
        sc = st.scale[flat].to(torch.bfloat16)
        for gi, start in enumerate(range(0, st.in_features, st.group)):
            w[:, start:start + st.group] *= sc[:, gi:gi + 1]
        return w

    def timed(fn, steps):
        for i in range(max(args.warmup, 3)):
            fn(batches[i % 64])
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(steps):
            fn(batches[i % 64])
        e1.record()
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / steps

    with ClockSampler(local_rank) as clocks:
        ms = timed(emb, args.steps)
    ms_ref = timed(reference, max(3, min(args.steps, 20)))
    # bytes a batch must move: each id's index row (k / 4) and scales, the codebook, the output
    k = shapes.hidden
    step_bytes = n * (k // 4 + (k // st.group) * 2 + k * 2) + st.cb.numel() * 2
    hbm_peak, peak_kind = _peaks()
    achieved = step_bytes / (ms * 1e-3) / 1e9
    if rank == 0:
        print(json.dumps({
            "metric": f"packed embedding rows/s @{args.model} ({n} ids per batch)",
            "value": round(n * 1000.0 / ms, 1), "unit": "rows/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"{shapes.vocab} x {k} vector-codebook embedding, {n} random ids",
                       "mode": "embedding", "l2": "64 rotating id batches over a 0.3+ GB table",
                       "bytes_per_step": step_bytes},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(achieved / hbm_peak, 4), "peak_kind": peak_kind,
                         "kernel": "embedding_kernel", "traffic": None},
            "reference_torch_ms": round(ms_ref, 5),
            "gpu_launches": args.steps,
            "clocks": clocks.summary(),
        }), flush=True)


# ---------------------------------------------------------------------------
# our arm: the whole-model decode token (the headline)
# ---------------------------------------------------------------------------
def _max_over_ranks(vals, dev, world):
    if world == 1:
        return vals
    import torch
    import torch.distributed as dist
    t = torch.tensor(vals, dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t]


def _timed_replays(fn, steps, dev, stream, clocks_index=None, barrier=None):
    """CUDA-event time (ms) of ``steps`` calls of fn() on ``stream``, bracketed by syncs.
    ``barrier`` (multi-rank) lines the ranks up after the clock sampler has started,
    so that its start-up does not skew one rank against the others."""
    import torch
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(clocks_index) if clocks_index is not None else None
    if sampler:
        sampler.__enter__()
    if barrier is not None:
        barrier()
    torch.cuda.synchronize(dev)
    e0.record(stream)
    for _ in range(steps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    if sampler:
        sampler.__exit__()
    return e0.elapsed_time(e1), (sampler.summary() if sampler else None)


def run_model(args, rank, world, local_rank):
    """Greedy decode of the whole model (epure.model.PackedDecoder), one CUDA graph per token."""
    import torch
    import torch.distributed as dist
    from epure import synthetic
    from epure.decode import GraphedLinearStack
    from epure.model import PackedDecoder
    from epure.synthetic import store_bytes

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    shapes = synthetic.SHAPES[args.model]
    max_len = PROMPT + args.warmup + args.steps + 2
    dec = PackedDecoder(shapes, layers=args.layers, device=dev, seed=1000 * rank, max_len=max_len,
                        fp32_logits=False, gpu_layout=args.layout, program=args.program).capture()
    g = torch.Generator().manual_seed(rank)
    prompt = torch.randint(0, shapes.vocab, (PROMPT,), generator=g)
    stream = torch.cuda.current_stream(dev)

    def restart():
        first = int(torch.argmax(dec.prefill(prompt)))
        dec.tok.fill_(first)
        dec.pos.fill_(PROMPT)
        torch.cuda.synchronize(dev)

    # device-resident: K replays of the token graph; the next token stays on the device
    restart()
    for _ in range(args.warmup):
        dec._graph.replay()
    torch.cuda.synchronize(dev)
    ms, clocks = _timed_replays(dec._graph.replay, args.steps, dev, stream, local_rank,
                                barrier=dist.barrier if world > 1 else None)
    if world > 1:
        dist.barrier()

    # end to end through the public greedy step: the token in from pinned host
    # memory, the graph, the next token back to the host, every step
    th = torch.empty(1, dtype=torch.long, pin_memory=True)

    def e2e_step():
        dec.tok.copy_(th, non_blocking=True)
        dec._graph.replay()
        th.copy_(dec.tok, non_blocking=True)
        stream.synchronize()

    restart()
    th.copy_(dec.tok.cpu())
    for _ in range(args.warmup):
        e2e_step()
    restart()
    th.copy_(dec.tok.cpu())
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    e2e_ms, _ = _timed_replays(e2e_step, args.steps, dev, stream)
    e2e_ms = max(e2e_ms, (time.perf_counter() - t0) * 1e3)

    packed = sum(store_bytes(st) for b in dec.stack.blocks for st in b.values())
    lm = dec.lm_head.numel() * dec.lm_head.element_size()
    pos_avg = PROMPT + args.warmup + args.steps / 2
    kv = 2 * dec.layers * pos_avg * shapes.kv_heads * shapes.head_dim * 2
    token_bytes = int(packed + lm + shapes.hidden * 2 + kv)
    if dec.use_program:
        # the dominant kernel alone: the token's decode program (every packed
        # linear and the attention of every layer, one launch) replayed in a graph
        # at the position the timed tokens averaged
        dec._ppos.fill_(int(pos_avg))
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            dec._program.run()
        stream.wait_stream(side)
        torch.cuda.synchronize(dev)
        pg = torch.cuda.CUDAGraph()
        with torch.cuda.graph(pg):
            dec._program.run()
        for _ in range(args.warmup):
            pg.replay()
        lin_ms, _ = _timed_replays(pg.replay, args.steps, dev, stream)
        # packed stores + this position's K/V rows + the activations in and out of every step
        lin_bytes = int(dec.stack.algorithmic_bytes(m=1, act_bytes=2)
                        + 2 * dec.layers * (int(pos_avg) + 1) * shapes.kv_heads * shapes.head_dim * 2)
        kern = {"kernel": "decode_program_kernel (every layer's packed linears and attention, one launch)",
                "launches": 1, "launch_avg_us": None}
        n_launch = 1
    else:
        # the dominant kernel alone: the token's packed launches (gemv_mma_kernel) in one graph
        lin = GraphedLinearStack(dec.stack, m=1, dtype=torch.bfloat16, device=dev).capture()
        lin.x.copy_(torch.randn(lin.x.shape, generator=torch.Generator(device=dev).manual_seed(rank),
                                device=dev).to(torch.bfloat16))
        for _ in range(args.warmup):
            lin.replay()
        lin_ms, _ = _timed_replays(lin.replay, args.steps, dev, stream)
        lin_bytes = dec.stack.algorithmic_bytes(m=1, act_bytes=2)
        n_launch = 4 * dec.layers
        kern = {"kernel": "gemv_mma_kernel (the token's packed launches replayed alone)", "launches": n_launch}
    ms, e2e_ms, lin_ms = _max_over_ranks([ms / args.steps, e2e_ms / args.steps, lin_ms / args.steps],
                                         dev, world)
    kern["launch_avg_us"] = round(lin_ms * 1e3 / n_launch, 3)
    kern["bytes_per_launch_avg"] = int(lin_bytes / n_launch)
    hbm_peak, peak_kind = _peaks()
    lin_gbs = lin_bytes / (lin_ms * 1e-3) / 1e9
    tok_gbs = token_bytes / (ms * 1e-3) / 1e9
    full = args.model == "llama3-8b" and dec.layers == shapes.layers
    if rank == 0:
        # `config` is exactly the reference arm's (the driver compares the two);
        # what only this arm knows goes to config_detail
        name, cfg = workload(args, world)
        detail = {"layout": args.layout, "bytes_per_step": token_bytes,
                  "decode_path": ("one persistent decode program per token" if dec.use_program
                                  else "five fused launches per layer"),
                  "bytes_split": {"packed": packed, "lm_head": lm, "kv": int(kv),
                                  "embedding_row": shapes.hidden * 2}}
        line = {
            "metric": METRIC,
            "value": round(world * 1000.0 / ms, 2), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded random weights in the benchmark format; uniform random prompt ids)",
            "config": cfg,
            "config_detail": detail,
            "roofline": dict({"bound": "hbm", "achieved": round(lin_gbs, 1), "peak": hbm_peak, "unit": "GB/s",
                              "frac": round(lin_gbs / hbm_peak, 4), "peak_kind": peak_kind}, **kern,
                             **_traffic(NCU_TRAFFIC_RATIO["program" if dec.use_program else "per-linear"],
                                        lin_bytes, full)),
            "token_roofline": {"bound": "hbm", "bytes_per_token": token_bytes, "achieved": round(tok_gbs, 1),
                               "peak": hbm_peak, "unit": "GB/s", "frac": round(tok_gbs / hbm_peak, 4),
                               "roofline_tok_s": round(hbm_peak * 1e9 / token_bytes, 1)},
            "e2e": {"value": round(world * 1000.0 / e2e_ms, 2), "unit": UNIT,
                    "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 8},
            # ours per token: program (or 5 per layer) + final RMSNorm + argmax
            "gpu_launches": ((3 if dec.use_program else 5 * dec.layers + 2)) * args.steps,
            "clocks": clocks,
        }
        if world == 1 and not args.no_cpu_baseline:
            threads = host_threads()
            times, _ = cpu_reference(SHAPES[args.model], dec.layers, threads, seconds=args.cpu_seconds)
            per = sum(times) / len(times)
            line["cpu_baseline"] = {
                "value": round(1.0 / per, 4), "unit": UNIT, "cores": threads, "kind": "port",
                "sample": f"{len(times)} whole decode tokens ({dec.layers} layers: packed linears through the "
                          f"lib.rs restatement, the rest numpy) in ~{args.cpu_seconds:g} s"}
        print(json.dumps(line), flush=True)
    return 0


def tp_check(shapes, rank, world, dev, layers=2):
    """Max relative error of the tensor-parallel chain against the single-GPU chain
    on a ``layers``-layer, full-width slice of one seeded model (fp32 outputs)."""
    import torch
    import torch.distributed as dist
    from epure import _native, synthetic
    from epure.decode import ChainedLinearStack
    from epure.tp import TPChainedLinearStack, shard_blocks

    full = synthetic.LinearStack(shapes, layers=layers, device=dev, seed=4242, gpu_layout="tiled")
    shards = synthetic.LinearStack.from_blocks(shapes, shard_blocks(full.blocks, rank, world, device=dev), dev)
    runner = TPChainedLinearStack(shards, dtype=torch.bfloat16, device=dev)
    x = torch.randn(1, shapes.hidden, generator=torch.Generator(device=dev).manual_seed(7),
                    device=dev).to(torch.bfloat16)
    got = torch.zeros(1, shapes.hidden, dtype=torch.float32, device=dev)
    _native.chain_run(runner.ws, x, got)
    torch.cuda.synchronize(dev)
    err = torch.zeros(1, dtype=torch.float64, device=dev)
    if rank == 0:
        one = ChainedLinearStack(full, device=dev)
        want = torch.zeros_like(got)
        _native.chain_run(one.ws, x, want)
        torch.cuda.synchronize(dev)
        err[0] = float((got - want).abs().max() / want.abs().max())
    dist.broadcast(err, 0)
    dist.barrier()
    runner.release()
    return float(err[0])


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from epure import synthetic
    from epure.decode import ChainedLinearStack, GraphedLinearStack

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    shapes = synthetic.SHAPES[args.model]
    use_tp = args.tp and world > 1
    chain = args.mode == "chain"
    prefill = args.mode == "prefill"
    m = args.tokens if prefill else args.batch
    check = None
    if use_tp and chain:
        err = tp_check(shapes, rank, world, dev)
        check = {"what": "TP chain vs the single-GPU chain, 2 layers of the same seeded model at full width, "
                         "fp32 outputs", "max_rel_err": err, "bound": 1e-4, "ok": err <= 1e-4}
        if not check["ok"]:
            if rank == 0:
                print(json.dumps({"metric": METRIC, "error": "tp_check failed", "tp_check": check}), flush=True)
            return 1
    if use_tp:
        # every rank draws its own shards of one model (same seed on every rank)
        stack = synthetic.LinearStack(shapes, layers=args.layers, device=dev, seed=1000,
                                      gpu_layout="tiled" if chain else "mma16", tp=(rank, world))
    else:
        stack = synthetic.LinearStack(shapes, layers=args.layers, device=dev, seed=1000 * rank,
                                      gpu_layout="tiled" if chain else "mma16")
    if use_tp and chain:
        from epure.tp import TPChainedLinearStack
        runner = TPChainedLinearStack(stack, dtype=torch.bfloat16, device=dev).capture()
        kernel_name = (f"chain_kernel on 1/{world} shards, all-reduce of o and down inside the "
                       "kernel (peer NVLink loads)")
    elif use_tp:
        from epure.tp import TPLinearStack
        runner = TPLinearStack(stack.blocks, m=m, dtype=torch.bfloat16, device=dev).capture()
        kernel_name = (("gemm_tc_kernel" if m > 16 else "gemv_mma_kernel") +
                       f" on 1/{world} shards + NCCL all-reduce after o and down")
    elif chain:
        runner = ChainedLinearStack(stack, dtype=torch.bfloat16, device=dev).capture()
        kernel_name = "chain_kernel (one persistent launch per step)"
    elif prefill:
        runner = GraphedLinearStack(stack, m=m, dtype=torch.bfloat16, device=dev).capture()
        kernel_name = "gemm_tc_kernel (all launches of the step)"
    else:
        runner = GraphedLinearStack(stack, m=m, dtype=torch.bfloat16, device=dev).capture()
        kernel_name = ("gemv_mma_kernel" if m <= 16 else "gemm_tc_kernel") + " (all launches of the step)"
    g = torch.Generator(device=dev).manual_seed(rank)
    runner.x.copy_(torch.randn(runner.x.shape, generator=g, device=dev).to(torch.bfloat16))
    step_bytes = stack.algorithmic_bytes(m=m, act_bytes=2)
    step_flops = stack.flops(m=m)
    launches = runner.launches_per_step

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        runner.replay()
    torch.cuda.synchronize(dev)

    # device-resident: K graph replays between two events on the replay stream;
    # the clock sampler starts (NVML, first sample) before the ranks line up
    stream = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        barrier()
        torch.cuda.synchronize(dev)
        ev0.record(stream)
        for _ in range(args.steps):
            runner.replay()
        ev1.record(stream)
        torch.cuda.synchronize(dev)
    barrier()
    ms = max_over_ranks(ev0.elapsed_time(ev1)) / args.steps

    # end to end through the public runner with host buffers
    x_host = torch.empty(runner.x.shape, dtype=runner.x.dtype, pin_memory=True)
    x_host.copy_(runner.x.cpu())
    out_host = torch.empty(runner.out.shape, dtype=runner.out.dtype, pin_memory=True)
    for _ in range(args.warmup):
        runner(x_host, out_host)
    torch.cuda.synchronize(dev)
    barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record(stream)
    for _ in range(args.steps):
        runner(x_host, out_host)
        stream.synchronize()            # the host reads each token's output
    e1.record(stream)
    torch.cuda.synchronize(dev)
    wall_ms = (time.perf_counter() - t0) * 1e3 / args.steps
    barrier()
    e2e_ms = max_over_ranks(max(e0.elapsed_time(e1) / args.steps, wall_ms))

    hbm_peak, peak_kind = _peaks()
    achieved_gbs = step_bytes / (ms * 1e-3) / 1e9
    workload_name = f"{args.model} packed linears, batch-1 decode token ({7 * stack.layers} linears)"
    if prefill:
        workload_name = workload_name.replace("batch-1 decode token", f"{m}-token prefill")
    elif m > 1:
        workload_name = workload_name.replace("batch-1 decode token", f"batch-{m} decode step ({m} tokens)")
    if stack.layers != shapes.layers:
        workload_name += f" (first {stack.layers} of {shapes.layers} layers)"
    if prefill:
        tf_peak, tf_kind = _tensor_peak()
        achieved_tf = step_flops / (ms * 1e-3) / 1e12
        roofline = {"bound": "tensor", "achieved": round(achieved_tf, 1), "peak": tf_peak,
                    "unit": "TFLOP/s", "frac": round(achieved_tf / tf_peak, 4),
                    "peak_kind": tf_kind, "kernel": kernel_name,
                    "launch_avg_us": round(ms * 1e3 / launches, 3), "traffic": None}
    else:
        roofline = {"bound": "hbm", "achieved": round(achieved_gbs, 1),
                    "peak": hbm_peak, "unit": "GB/s",
                    "frac": round(achieved_gbs / hbm_peak, 4),
                    "peak_kind": peak_kind,
                    "kernel": kernel_name,
                    "launch_avg_us": round(ms * 1e3 / launches, 3),
                    "traffic": (int(step_bytes * NCU_TRAFFIC_RATIO[args.mode])
                                if NCU_TRAFFIC_RATIO.get(args.mode) and stack.layers == 32
                                and args.model == "llama3-8b" and m == 1 else None),
                    "traffic_note": ("per step, scaled from one ncu capture (profiles/): dram bytes / "
                                     "algorithmic bytes of the " + ("4-layer chain" if chain else "gate+up launch")
                                     if NCU_TRAFFIC_RATIO.get(args.mode) else None)}
    streams = 1 if use_tp else world          # independent token streams across the job
    if use_tp:
        # aggregate over the ranks: each streams its shard bytes in the same step time
        roofline["achieved"] = round(roofline["achieved"] * world, 1)
        roofline["peak"] = round(roofline["peak"] * world, 1)
        roofline["aggregate_over_gpus"] = world
        roofline["traffic"] = None
        roofline.pop("traffic_note", None)
    if rank == 0:
        metric = (f"prefill tok/s @{args.model} ({m}-token prompt, packed linears)"
                  if prefill else METRIC)
        if not prefill and m > 1:
            metric = f"decode tok/s bs{m} @{args.model} (packed linears)"
        if use_tp and not prefill:
            metric = (f"decode tok/s bs{m} @{args.model}, tensor-parallel over {world} GPUs "
                      "(packed linears)")
        line = {
            "metric": metric,
            "value": round(streams * m * 1000.0 / ms, 2),
            "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms, 5),
            "higher_is_better": True,
            "scaling": "strong" if use_tp else "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": workload_name,
                       "mode": ("tp-" + args.mode) if use_tp else args.mode,
                       "global_batch": streams * m,
                       "seq_len": m,
                       "parallelism": (f"tp{world}" if use_tp else
                                       f"replicas x{world}" if world > 1 else "single GPU"),
                       "l2": (f"inputs larger than L2 ({step_bytes / 1e9:.2f} GB moved per step)"
                              if step_bytes > 126e6 else "working set may fit in L2"),
                       "bytes_per_step": step_bytes, "flops_per_step": step_flops},
            "roofline": roofline,
            "e2e": {"value": round(streams * m * 1000.0 / e2e_ms, 2), "unit": UNIT,
                    "h2d_bytes_per_step": x_host.numel() * x_host.element_size(),
                    "d2h_bytes_per_step": out_host.numel() * out_host.element_size()},
            "gpu_launches": launches * args.steps,
            "clocks": clocks.summary(),
        }
        if check is not None:
            line["tp_check"] = check
            # `config` is exactly the reference arm's; the rest goes to config_detail
            detail = dict(line["config"])
            _, line["config"] = workload(args, world)
            line["config_detail"] = {k: v for k, v in detail.items() if k not in line["config"]}
            # the driver's multi-GPU run: BASELINE's metric, as the reference arm prints
            # it; the workload (70B shapes, tensor parallel) is named in config
            line["metric"] = METRIC
        if args.fallback:
            line["fallback"] = time_fallback(stack, runner.x, steps=max(1, min(args.steps, 3)))
        if world == 1 and not args.no_cpu_baseline and args.mode != "prefill" and m == 1:
            threads = host_threads()
            times, _ = cpu_reference(SHAPES[args.model], stack.layers, threads, seconds=args.cpu_seconds,
                                     linears_only=True)
            per = sum(times) / len(times)
            line["cpu_baseline"] = {
                "value": round(1.0 / per, 4), "unit": UNIT, "cores": threads, "kind": "port",
                "sample": f"{len(times)} tokens of the {7 * stack.layers} packed linears through the lib.rs "
                          f"restatement in ~{args.cpu_seconds:g} s"}
        print(json.dumps(line), flush=True)
    if use_tp:
        runner.release()        # the graph holds NCCL work: drop it before the group goes
        torch.cuda.synchronize(dev)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--mode", choices=["model", "chain", "per-linear", "prefill", "finetune", "embedding"],
                    default=None, help="default: model at N = 1 (and with --replicas), tensor-parallel chain at N > 1")
    ap.add_argument("--model", choices=sorted(SHAPES), default=None)
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--tokens", type=int, default=None)
    ap.add_argument("--seq", type=int, default=2048, help="--mode finetune: tokens per sequence")
    ap.add_argument("--batch", type=int, default=None,
                    help="decode batch (tokens per step) for --mode per-linear: M rows through "
                         "every linear (tensor-core GEMV up to 16, the tcgen05 GEMM above)")
    ap.add_argument("--layout", choices=["mma16", "tiled"], default="mma16",
                    help="--mode model: index layout of the packed stores (tensor-core GEMV or LUT GEMV "
                         "at batch 1)")
    ap.add_argument("--tp", action="store_true",
                    help="at N > 1 with --mode chain / per-linear: one model tensor-parallel over the N GPUs")
    ap.add_argument("--replicas", action="store_true",
                    help="at N > 1: N independent copies of the N = 1 workload instead of tensor parallelism")
    ap.add_argument("--program", action="store_true",
                    help="--mode model: run each token's layers as one persistent decode program")
    ap.add_argument("--fallback", action="store_true",
                    help="also time the reference's bf16 fallback path on the same step (GPU)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.mode is None:
        if world > 1 and not args.replicas:
            args.mode, args.tp = "chain", True
        else:
            args.mode = "model"
    if args.model is None:
        args.model = ("qwen3-1.7b" if args.mode == "finetune" else
                      "llama3-70b" if (args.tp and world > 1) else "llama3-8b")
    if args.tokens is None:
        args.tokens = 8 * 2048 if args.mode == "finetune" else 2048
    if args.batch is not None and args.mode not in ("per-linear", "finetune"):
        ap.error("--batch applies to --mode per-linear and --mode finetune")
    if args.batch is None and args.mode != "finetune":
        args.batch = 1

    if args.impl == "reference":
        return run_reference(args, rank, world)

    import torch
    import torch.distributed as dist
    if world > 1:
        from datetime import timedelta
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.mode == "finetune":
            return run_finetune(args, rank, world, local_rank)
        if args.mode == "model":
            return run_model(args, rank, world, local_rank)
        if args.mode == "embedding":
            return run_embedding(args, rank, world, local_rank)
        return run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())

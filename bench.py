"""Benchmark: batch-1 decode through every packed linear of a Llama-3-8B-shaped model.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step is one decode token: all 32 x 7 codebook-quantized linears of the
Llama-3-8B shapes (indices u8 per 4-weight vector, 256x4 fp16 codebook, fp16
scale per row per 128 weights; 1.85 GB of indices), visited in layer order
with each launch reading the previous one's output.  The packed weights
(1.9 GB) are far larger than the 126 MB L2, so every step streams them from
HBM; no L2 flush is needed.  Attention, norms and the bf16 lm_head are not
part of the packed-linear path and are not in the step.

Our arm runs the step as ONE persistent launch of libepq.so's chain kernel
(epq_chain_run: every packed linear of the token, weights streamed through a
TMA ring per SM, each linear's input polled from the tagged split-k partial sums
of the previous one, no grid barrier), replayed from a CUDA
graph (value), and separately through the public runner with host buffers
(e2e: pinned H2D copy of the token input, replay, D2H copy of the output, every
step).  `--mode per-linear` instead replays 128 launches of the single-linear
tensor-core GEMV (one per fused q/k/v, o, gate/up, down).  At N > 1
each rank runs an independent replica on its own GPU (weak scaling; the 8B
model fits one GPU, so there is no collective on the data path); the time is
the max over ranks.

Other workloads (not the headline; each prints its own metric):
  --mode finetune [--tokens 16384]: one compressed-state fine-tuning step (the
      config-3 batch of 8 x 2048 tokens, Qwen3-1.7B shapes by default) through
      every packed linear: forward, dX, dscale/dcb (epure.train.PackedTrainStep);
  --mode prefill [--tokens 2048]: a prompt of `tokens` rows through every packed
      linear (the tensor-core dequant-GEMM, one launch per fused group), metric
      prefill tok/s, roofline against the sustained bf16 tensor peak;
  --mode model: greedy decode of the whole model (epure.model.PackedDecoder:
      packed linears through libepq.so, attention / norms / lm_head in torch, one
      CUDA graph per token after a 128-token prompt), metric tok/s;
  --mode embedding [--tokens N]: packed embedding rows for N ids (epq_embedding), with
      the reference's torch formulation timed beside it;
  --mode per-linear --batch B: a B-token decode step through the per-linear launches
      (the tensor-core GEMV up to 16 rows, the tcgen05 GEMM above), metric tok/s;
  --model qwen3-1.7b|llama3-8b|llama3-70b picks the decoder shapes;
  --layers L keeps the first L layers (small cases for profiling);
  --tp (with N > 1): one model tensor-parallel over the N GPUs (column-parallel
      q/k/v and gate/up, row-parallel o and down), one token stream, strong
      scaling; in the default chain mode the all-reduce of o and down happens
      inside the persistent kernel over NVLink, with --mode per-linear it is an
      NCCL all-reduce after each row-parallel launch;
  --fallback also times the reference's bf16 fallback path on the GPU
      (F.linear(x, materialize(bf16)) store by store, torch ops) on the same step.

The reference arm (--impl reference) runs the reference's fused CPU kernel
(kernel/src/lib.rs, restated in C under oracle/) on the host cores: each step
is one layer's 7 linears with f32 activations, and tokens/s is scaled by the
32 layers.  Rank 0 alone runs it.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "epure-runtime_b200"))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s bs1 @8B; dequant-GEMV HBM GB/s as % of B200 peak"
UNIT = "tok/s"
WORKLOAD = "llama3-8b packed linears, batch-1 decode token (224 linears)"

# DRAM traffic / algorithmic bytes per mode, from one ncu capture each.  Traffic
# grows with the bytes streamed, so a step's traffic is reported as the ratio
# times the step's algorithmic bytes.
#   per-linear: gemv_mma_kernel on a Llama-3-8B gate+up launch
#     (profiles/gemv_mma_kernel_llama3-8b_gateup_b1.md): 31,236,096 B of
#     dram__bytes_read.sum + dram__bytes_write.sum against 31,264,768 B.
#   chain: chain_kernel on a 4-layer Llama-3-8B chain
#     (profiles/chain_kernel_llama3-8b_decode_b1.md): 232,937,728 B read +
#     24,145,664 B written against 232,349,696 algorithmic bytes.
NCU_TRAFFIC_RATIO = {"per-linear": 31236096 / 31264768,
                     "chain": (232937728 + 24145664) / 232349696}
TRAFFIC_NOTE = {"per-linear": "per step, scaled from one ncu capture of the gate+up launch "
                              "(traffic/algorithmic = 0.999)",
                "chain": "per step, scaled from one ncu capture of a 4-layer chain "
                         "(traffic/algorithmic = 1.106; the extra bytes are the tagged split-k "
                         "partial sums written back to DRAM)"}


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
    """nvidia-smi clock/throttle samples for one GPU during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
# CPU reference arm / CPU baseline
# ---------------------------------------------------------------------------
def cpu_reference_sample(seconds=10.0, threads=0, steps=None, warmup=1, model="llama3-8b"):
    """Time the lib.rs restatement on one layer of `model`; returns (tok/s, info)."""
    import numpy as np
    from oracle import oracle as O
    from epure import synthetic

    shapes = synthetic.SHAPES[model]
    O.build_c_oracle()
    rng = np.random.default_rng(0)
    layer = []
    for name, n, k in shapes.linears():
        idx = rng.integers(0, 256, (n, k // 4), dtype=np.uint8)
        cb = rng.standard_normal((256, 4)).astype(np.float16).astype(np.float32)
        sc = np.abs(rng.normal(0, 0.02, (n, k // 128))).astype(np.float16).astype(np.float32)
        x = rng.standard_normal((1, k)).astype(np.float32)
        layer.append((x, idx, sc, cb, n, k))

    def one_layer():
        for x, idx, sc, cb, n, k in layer:
            O.c_dequant_matmul(x, idx, sc, cb, n, k, 4, 128, 256, threads=threads)

    for _ in range(warmup):
        one_layer()
    times = []
    t_total = time.perf_counter()
    while True:
        t0 = time.perf_counter()
        one_layer()
        times.append(time.perf_counter() - t0)
        if steps is not None:
            if len(times) >= steps:
                break
        elif time.perf_counter() - t_total >= seconds:
            break
    per_layer = statistics.median(times)
    tok_s = 1.0 / (per_layer * shapes.layers)
    used = threads if threads > 0 else O.c_threads()
    info = {"cores": used, "kind": "port",
            "sample": f"1 of {shapes.layers} {model} layers (7 linears, f32 activations), "
                      f"{len(times)} timed repetitions, median {per_layer*1e3:.1f} ms/layer; "
                      f"tok/s = 1/({shapes.layers} x layer)"}
    return tok_s, info


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    tok_s, info = cpu_reference_sample(steps=args.steps, warmup=args.warmup, model=args.model)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(tok_s, 4), "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1000.0 / tok_s, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "global_batch": 1, "parallelism": "host threads",
                   "l2": "n/a (CPU)"},
        "cpu_baseline": {"value": round(tok_s, 4), "unit": UNIT, **info},
        "e2e": {"value": round(tok_s, 4), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# our arm
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
    """One compressed-state fine-tuning step over every packed linear (config 3)."""
    import torch
    import torch.distributed as dist
    from epure import synthetic
    from epure.train import PackedTrainStep

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    model = args.model
    shapes = synthetic.SHAPES[model]
    m = args.tokens
    # make_trainable(mode="both") keeps scales and codebooks as fp32 parameters
    stack = synthetic.LinearStack(shapes, layers=args.layers, device=dev, seed=1000 * rank,
                                  gpu_layout="mma16", scale_dtype=torch.float32,
                                  cb_dtype=torch.float32)
    trainer = PackedTrainStep(stack, m, device=dev, seed=rank)
    g = torch.Generator(device=dev).manual_seed(rank)
    x = torch.randn(m, shapes.hidden, generator=g, device=dev).to(torch.bfloat16)
    flops = trainer.flops()
    for _ in range(args.warmup):
        trainer.step(x)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        ev0.record(stream)
        for _ in range(args.steps):
            trainer.step(x)
        ev1.record(stream)
        torch.cuda.synchronize(dev)
    ms = ev0.elapsed_time(ev1) / args.steps
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    # end to end: the token batch from pinned host memory, the step, one gradient read back
    xh = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
    xh.copy_(x.cpu())
    gh = torch.empty(1, dtype=torch.float32, pin_memory=True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        xd = xh.to(dev, non_blocking=True)
        trainer.step(xd)
        gh.copy_(trainer.grads[0]["q_proj"][1][:1], non_blocking=True)
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
            "metric": f"fine-tune tok/s @{model} (packed linears fwd + dX + dscale/dcb, {m} tokens/step)",
            "value": round(world * m * 1000.0 / ms, 2), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": f"{model} packed linears, compressed-state fine-tune step "
                                   f"({7 * stack.layers} linears, fp32 scales and codebooks)",
                       "mode": "finetune", "global_batch": world * m, "seq_len": m,
                       "parallelism": f"data-parallel replicas x{world}" if world > 1 else "single GPU",
                       "flops_per_step": flops},
            "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": tf_peak,
                         "unit": "TFLOP/s", "frac": round(achieved / tf_peak, 4), "peak_kind": tf_kind,
                         "kernel": "gemm_tc_kernel + bwd_dx_tc_kernel + bwd_dw_tc_kernel",
                         "traffic": None},
            "e2e": {"value": round(world * m * 1000.0 / e2e_ms, 2), "unit": UNIT,
                    "h2d_bytes_per_step": x.numel() * x.element_size(), "d2h_bytes_per_step": 4},
            "gpu_launches": (4 + 7) * stack.layers * args.steps,
            "clocks": clocks.summary(),
        }
        if args.fallback:
            line["fallback"] = time_fallback_finetune(stack, x, steps=max(1, min(args.steps, 2)))
        print(json.dumps(line), flush=True)
    return 0


def time_fallback_finetune(stack, x, steps):
    """The reference's fine-tuning autograd on the same step (GPU, torch ops).

    make_trainable (finetune.py:49-102) + PackedLinear.forward's fallback
    F.linear(x, materialize(bf16)) (runtime.py:78-89, 123-124): torch autograd
    differentiates the gather/scale expansion and the GEMM; fp32 parameters.
    """
    import torch
    import torch.nn.functional as F
    params = []
    for b in stack.blocks:
        pb = {}
        for name, st in b.items():
            pb[name] = (st.index_rows().long(), st.cb.float().clone().requires_grad_(True),
                        st.scale.float().clone().requires_grad_(True), st)
        params.append(pb)

    def weight(p):
        idx, cb, sc, st = p
        w = cb.to(torch.bfloat16)[idx].reshape(st.out_features, -1)[:, :st.in_features]
        return w * sc.to(torch.bfloat16).repeat_interleave(st.group, dim=1)[:, :st.in_features]

    def step():
        h = x.detach().requires_grad_(True)
        outs = []
        for pb in params:
            q = F.linear(h, weight(pb["q_proj"]))
            k = F.linear(h, weight(pb["k_proj"]))
            v = F.linear(h, weight(pb["v_proj"]))
            o = F.linear(q, weight(pb["o_proj"]))
            gt = F.linear(o, weight(pb["gate_proj"]))
            u = F.linear(o, weight(pb["up_proj"]))
            h = F.linear(u, weight(pb["down_proj"]))
            outs += [k, v, gt]
        loss = h.float().square().mean() + sum(t.float().mean() for t in outs)
        loss.backward()

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
                    "fp32 scale/codebook parameters (torch ops)",
            "ms_per_step": round(ms, 3), "value": round(x.shape[0] * 1000.0 / ms, 2), "unit": UNIT,
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


def run_model(args, rank, world, local_rank):
    """Greedy decode of the whole model (epure.model.PackedDecoder): packed linears
    through libepq.so, attention / norms / RoPE / SwiGLU / lm_head in torch, one
    CUDA graph per token (argmax and position update included)."""
    import torch
    import torch.distributed as dist
    from epure import synthetic
    from epure.model import PackedDecoder
    from epure.synthetic import store_bytes

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    shapes = synthetic.SHAPES[args.model]
    prompt_len = 128
    max_len = prompt_len + args.warmup + args.steps + 2
    dec = PackedDecoder(shapes, layers=args.layers, device=dev, seed=1000 * rank, max_len=max_len,
                        fp32_logits=False, gpu_layout=args.layout).capture()
    g = torch.Generator().manual_seed(rank)
    prompt = torch.randint(0, shapes.vocab, (prompt_len,), generator=g)

    def restart():
        first = int(torch.argmax(dec.prefill(prompt)))
        dec.tok.fill_(first)
        dec.pos.fill_(prompt_len)
        torch.cuda.synchronize(dev)

    restart()
    for _ in range(args.warmup):
        dec._graph.replay()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    stream = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        ev0.record(stream)
        for _ in range(args.steps):
            dec._graph.replay()
        ev1.record(stream)
        torch.cuda.synchronize(dev)
    ms = ev0.elapsed_time(ev1) / args.steps
    # end to end: each token goes from pinned host memory into the graph's input
    # and the next token is read back to the host, every step
    restart()
    th = torch.empty(1, dtype=torch.long, pin_memory=True)
    th.copy_(dec.tok.cpu())
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        dec.tok.copy_(th, non_blocking=True)
        dec._graph.replay()
        th.copy_(dec.tok, non_blocking=True)
        stream.synchronize()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([ms, e2e_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms = float(t[0]), float(t[1])
    # algorithmic bytes of one token: packed stores, lm_head, one embedding row, and
    # the K/V of the positions attended (averaged over the timed steps)
    packed = sum(store_bytes(st) for b in dec.stack.blocks for st in b.values())
    lm = dec.lm_head.numel() * dec.lm_head.element_size()
    pos_avg = prompt_len + args.warmup + args.steps / 2
    kv = 2 * dec.layers * pos_avg * shapes.kv_heads * shapes.head_dim * 2
    step_bytes = int(packed + lm + shapes.hidden * 2 + kv)
    hbm_peak, peak_kind = _peaks()
    achieved = step_bytes / (ms * 1e-3) / 1e9
    if rank == 0:
        layers_note = (f" (first {dec.layers} of {shapes.layers} layers)"
                       if dec.layers != shapes.layers else "")
        line = {
            "metric": f"greedy decode tok/s bs1 @{args.model} (whole model: packed linears + "
                      "attention, norms, lm_head)",
            "value": round(world * 1000.0 / ms, 2), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": f"{args.model} greedy decode after a {prompt_len}-token prompt"
                                   + layers_note, "layout": args.layout,
                       "mode": "model", "global_batch": world, "seq_len": max_len,
                       "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                       "l2": f"inputs larger than L2 ({step_bytes / 1e9:.2f} GB moved per step)",
                       "bytes_per_step": step_bytes,
                       "bytes_split": {"packed": packed, "lm_head": lm, "kv": int(kv)}},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak,
                         "unit": "GB/s", "frac": round(achieved / hbm_peak, 4),
                         "peak_kind": peak_kind,
                         "kernel": ("whole token graph: " + ("gemv_mma_kernel" if args.layout == "mma16"
                                                              else "gemv_lut_kernel") +
                                    " (packed) + decode glue kernels + cuBLAS lm_head"),
                         "traffic": None},
            "e2e": {"value": round(world * 1000.0 / e2e_ms, 2), "unit": UNIT,
                    "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 8},
            "gpu_launches": 4 * dec.layers * args.steps,
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)


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

    # device-resident: K graph replays between two events on the replay stream
    barrier()
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
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
    workload = WORKLOAD.replace("llama3-8b", args.model).replace(
        "224 linears", f"{7 * stack.layers} linears")
    if prefill:
        workload = workload.replace("batch-1 decode token", f"{m}-token prefill")
    elif m > 1:
        workload = workload.replace("batch-1 decode token", f"batch-{m} decode step ({m} tokens)")
    if stack.layers != shapes.layers:
        workload += f" (first {stack.layers} of {shapes.layers} layers)"
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
                    "traffic_note": TRAFFIC_NOTE.get(args.mode)}
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
            "config": {"workload": workload,
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
        if args.fallback:
            line["fallback"] = time_fallback(stack, runner.x, steps=max(1, min(args.steps, 3)))
        if world == 1 and not args.no_cpu_baseline and args.mode != "prefill":
            tok_s, info = cpu_reference_sample(seconds=args.cpu_seconds, model=args.model)
            line["cpu_baseline"] = {"value": round(tok_s, 4), "unit": UNIT, **info}
        print(json.dumps(line), flush=True)
    if use_tp:
        runner.release()        # the graph holds NCCL work: drop it before the group goes
        torch.cuda.synchronize(dev)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--mode", choices=["chain", "per-linear", "prefill", "finetune", "model", "embedding"],
                    default="chain")
    ap.add_argument("--model", choices=["qwen3-1.7b", "llama3-8b", "llama3-70b"], default=None)
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--tokens", type=int, default=None)
    ap.add_argument("--batch", type=int, default=1,
                    help="decode batch (tokens per step) for --mode per-linear: M rows through "
                         "every linear (tensor-core GEMV up to 16, the tcgen05 GEMM above)")
    ap.add_argument("--layout", choices=["mma16", "tiled"], default="mma16",
                    help="--mode model: index layout of the packed stores (tensor-core GEMV or LUT GEMV "
                         "at batch 1)")
    ap.add_argument("--tp", action="store_true",
                    help="at N > 1: one model tensor-parallel over the N GPUs instead of N replicas")
    ap.add_argument("--fallback", action="store_true",
                    help="also time the reference's bf16 fallback path on the same step (GPU)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    args.model_set = args.model is not None
    if args.model is None:
        args.model = "qwen3-1.7b" if args.mode == "finetune" else "llama3-8b"
    if args.tokens is None:
        args.tokens = 8 * 2048 if args.mode == "finetune" else 2048
    if args.batch != 1 and args.mode != "per-linear":
        ap.error("--batch applies to --mode per-linear (the chain kernel is batch-1)")

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

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

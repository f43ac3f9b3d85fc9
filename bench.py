"""Benchmark of the AGILLM4.1 MoE block forward on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one MoE block forward (router -> top-2 -> dispatch -> expert FFNs
-> combine) over the whole batch. Workload at one GPU: B=48, L=1536 tokens
(73,728), d_model=1280, 14 experts with hidden 3200, top-2, bf16, random-init
weights N(0, 0.02^2), x ~ N(0, 1), seed 1. Inputs (x: 189 MB, expert
weights: 229 MB) are larger than the 126 MB L2, so no flush is needed between
steps.

With N > 1 (one process per GPU under torchrun) every rank holds the same
B x L workload of its own tokens (weak scaling) and the block runs expert
parallel: the static expert ownership plus at most 2 hot-expert replicas per
rank, rows moved over NVLink peer memory inside the kernels; tokens/s is the
sum over ranks and the time is the max over ranks.

The JSON line carries the whole-job tokens/s (device-timed, inputs resident
in HBM), the end-to-end tokens/s through the public module API with host
buffers (pinned host -> device copy of x and device -> host copy of the
output inside the timed region), the per-stage kernel times measured live
with CUDA events around each kernel stage, the roofline of the dominant
kernel (the tcgen05 grouped GEMM), the CPU baseline (the oracle, i.e. the
reference's torch op sequence, on the host cores) and the SM clocks seen
during the timed region.

``--impl reference`` times the reference's CPU implementation of the path
(the oracle) on the host cores instead, on the same workload shapes.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

D, HIDDEN, EXPERTS, TOP_K, BATCH, SEQ, SEED = 1280, 3200, 14, 2, 48, 1536, 1
METRIC = "MoE tokens/s (d1280, 14 exp, top-2) at 1/2/4/8 B200; % of roofline"
UNIT = "tokens/s"
FLOP_PER_TOKEN = 4 * D * HIDDEN * TOP_K          # 32,768,000 (FC1 + FC2, k rows per token)
# Algorithmic HBM bytes per token of the memory-bound stages (bf16):
ROUTER_BYTES = 2 * D + 4 * TOP_K + 2 * TOP_K      # read x row; write idx (int32) + gates (bf16)
PERMUTE_BYTES = 2 * D + 4 * TOP_K + 2 * D * TOP_K + 4 * TOP_K + 4 * TOP_K  # x, idx -> k rows, row_of, token_of
COMBINE_BYTES = 2 * D * TOP_K + 4 * TOP_K + 2 * TOP_K + 2 * D             # k rows, row_of, gates -> out row
STAGES = ["router", "plan", "permute", "fc1", "fc2", "shared", "combine"]
KERNELS_PER_STEP = 6   # router, plan, permute, fc1, fc2, combine
DECODE_KERNELS_PER_LAYER = 4   # at most 128 tokens: decode front (router + plan + permute), fc1, fc2, combine
TILE_ROWS = 128
# Multi-GPU workload: each rank holds B x L tokens; router logits carry a
# per-expert bias log(p_e) * ZIPF_SCALE with p Zipf(1.2) over a seeded
# permutation of the experts (seed 3), which gives a ~5:1 max/mean expert load.
EP_SEED, ZIPF_S, ZIPF_SCALE = 3, 1.2, 0.63
EP_STAGES = ["route", "counts_plan", "dispatch_a2a", "expert_ffn", "return_a2a", "combine"]
P2P_STAGES = ["route", "counts_exchange_plan", "dispatch_to_peers", "signal", "fc1", "fc2_to_owners", "barrier2",
              "combine"]


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return dict(hbm=float(j["hbm_gbs"]), tf=float(j["bf16_tflops"]),
                    tf_sus=float(j.get("bf16_tflops_sustained", j["bf16_tflops"])), src="measured")
    return dict(hbm=6650.0, tf=1590.0, tf_sus=1400.0, src="fallback")


def load_traffic():
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f)
    return {}


class ClockSampler:
    """nvidia-smi clock/throttle sampling (every 20 ms) around a timed region.

    The sampler is started before the warm-up (nvidia-smi takes ~0.1 s to
    produce its first sample) and stopped after the last pass over the same
    workload. ``mark_start()`` / ``mark_stop()`` bracket the timed region on
    the host clock; ``summary()`` reports the samples whose timestamps fall in
    that window, and when the window holds fewer than 5 (a short timed
    region), the samples of the whole loaded period (warm-up, timed region and
    the per-stage pass, all the same forward) instead, saying which.
    """

    QUERY = ("timestamp,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    PERIOD_MS = 20

    def __init__(self, device):
        # nvidia-smi numbers GPUs differently from CUDA under CUDA_VISIBLE_DEVICES: use the UUID.
        try:
            self.gpu = "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
        except Exception:
            self.gpu = str(device.index if isinstance(device, torch.device) else device)
        self.proc = None
        self.path = None
        self.t0 = self.t1 = None

    def __enter__(self):
        try:
            import tempfile
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", str(self.PERIOD_MS)],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            time.sleep(0.3)               # let nvidia-smi start sampling before the load begins
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def mark_start(self):
        self.t0 = time.time()

    def mark_stop(self):
        self.t1 = time.time()

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    @staticmethod
    def _ts(text):
        import datetime
        for fmt in ("%Y/%m/%d %H:%M:%S.%f", "%Y/%m/%d %H:%M:%S"):
            try:
                return datetime.datetime.strptime(text.strip(), fmt).timestamp()
            except ValueError:
                continue
        return None

    def summary(self):
        if self.proc is None or not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        window = "whole loaded period (warm-up, timed region, per-stage pass)"
        if self.t0 is not None and self.t1 is not None:
            # nvidia-smi prints local time; allow one period of slack at each end
            slack = self.PERIOD_MS / 1000.0
            inside = []
            for r in rows:
                t = self._ts(r[0])
                if t is not None and self.t0 - slack <= t <= self.t1 + slack:
                    inside.append(r)
            if len(inside) >= 5:
                rows, window = inside, "timed region"
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        loaded = [s for s in sm if mx and s > 0.3 * max(mx)] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows), "window": window, "period_ms": self.PERIOD_MS,
                "power_w_max": max((float(r[3]) for r in rows if r[3].replace(".", "").isdigit()), default=None)}


def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(v, world):
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def cpu_oracle_rate(n_tokens, budget_s=12.0, min_reps=2, threads=None):
    """Tokens/s of the reference's torch op sequence on the host CPU (fp32)."""
    from oracle import reference_moe
    threads = threads or (os.cpu_count() or 1)
    torch.set_num_threads(threads)
    sd = reference_moe.make_state(D, HIDDEN, EXPERTS, SEED, dtype=torch.float32)
    x = reference_moe.make_input(n_tokens, D, SEED)
    with torch.no_grad():
        reference_moe.moe_forward(x[: min(256, n_tokens)], sd, TOP_K)   # warm-up
        reps, t0 = 0, time.perf_counter()
        while reps < min_reps or time.perf_counter() - t0 < budget_s:
            reference_moe.moe_forward(x, sd, TOP_K)
            reps += 1
        dt = time.perf_counter() - t0
    return n_tokens * reps / dt, threads, reps, dt


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_reference(args, world, rank):
    """--impl reference: the reference's CPU path (the oracle, i.e. the
    reference's torch op sequence) on the host cores, on a 2,048-token sample
    of the workload per step. Also reported (key ``gpu``): the same op
    sequence in bf16 on this B200 over the whole 73,728-token workload, the
    reference's own GPU forward (a library GEMM per linear, 28 host syncs per
    block) for like-for-like context."""
    if rank != 0:
        return
    from oracle import reference_moe
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    sample = 2048
    sd = reference_moe.make_state(D, HIDDEN, EXPERTS, SEED, dtype=torch.float32)
    x = reference_moe.make_input(sample, D, SEED)
    times = []
    with torch.no_grad():
        for i in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            reference_moe.moe_forward(x, sd, TOP_K)
            if i >= args.warmup:
                times.append(time.perf_counter() - t0)
    total = sum(times)
    value = sample * len(times) / total
    cfg = workload_config(world)
    cfg["sample"] = f"{sample} tokens of the B{BATCH} L{SEQ} workload per step (fp32, host cores)"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * total / len(times),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1) input, N(0,0.02^2) weights)",
        "config": cfg,
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{sample} tokens of the workload per step, fp32, torch.set_num_threads({threads}), "
                                   f"CPU {cpu_model()}"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if torch.cuda.is_available() and not args.skip_reference_gpu:
        line["gpu"] = reference_gpu_rate(args)
    print(json.dumps(line), flush=True)


def reference_gpu_rate(args):
    """The reference's op sequence (oracle/reference_moe.py restates
    MoEFFN.forward, agillm41.py:4389-4431) in bf16 on one GPU over the whole
    B48 x L1536 workload, CUDA-event timed; inputs resident in HBM."""
    from oracle import reference_moe

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    N = BATCH * SEQ
    sd = reference_moe.make_state(D, HIDDEN, EXPERTS, SEED, dtype=torch.bfloat16, device=dev)
    x = reference_moe.make_input(N, D, SEED, dtype=torch.bfloat16, device=dev)
    with torch.no_grad():
        for _ in range(3):
            reference_moe.moe_forward(x, sd, TOP_K)
        torch.cuda.synchronize(dev)
        steps = 10
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            reference_moe.moe_forward(x, sd, TOP_K)
        e1.record()
        torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / steps
    return {"value": N / (ms / 1000.0), "unit": UNIT, "ms_per_step": round(ms, 3), "steps": steps,
            "workload": f"B{BATCH} L{SEQ} ({N} tokens) d{D} E{EXPERTS} H{HIDDEN} top{TOP_K} bf16, seed {SEED}",
            "what": "the reference's torch op sequence (router Linear, topk, softmax, per-(rank, expert) nonzero, "
                    "index_select, expert Linear-ReLU-Linear, index_add_) on one B200, library kernels"}


def workload_config(world, tokens=BATCH * SEQ):
    shape = f"B{BATCH} L{SEQ}" if tokens == BATCH * SEQ else f"{tokens} tokens"
    return {"workload": f"MoE block forward {shape} d{D} E{EXPERTS} H{HIDDEN} top{TOP_K} bf16 seed{SEED}",
            "global_batch": BATCH * world, "seq_len": SEQ, "tokens_per_gpu": tokens, "d_model": D,
            "experts": EXPERTS, "expert_hidden": HIDDEN, "top_k": TOP_K,
            "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
            "l2": "inputs larger than L2 (x 189 MB + expert weights 229 MB > 126 MB); no flush"}


def run_ours(args, world, rank, local):
    import agillm41_b200
    from agillm41_b200 import ops, synthetic

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    N = args.tokens
    sd = synthetic.make_state(D, HIDDEN, EXPERTS, SEED, dtype=torch.bfloat16, device=dev)
    x = synthetic.make_input(N, D, SEED + rank * 1000, dtype=torch.bfloat16, device=dev)
    w1, b1, w2, b2, wr = pack_weights(sd)
    out = torch.empty_like(x)
    stream = torch.cuda.current_stream(dev)

    def step(events=None):
        ops.moe_forward(x, wr, w1, b1, w2, b2, TOP_K, out=out, stage_events=events)

    with ClockSampler(dev) as clk:
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize()
        from agillm41_b200._lib import read_device_error
        err = read_device_error(ops.Workspace.get(dev, 0)[:4].view(torch.int32))
        if err:
            raise RuntimeError(f"device error word 0x{err:x} after warm-up")

        # ---- timed region (device time) ----
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier(world)
        torch.cuda.synchronize()
        clk.mark_start()
        start.record(stream)
        for i in range(args.steps):
            step()
        stop.record(stream)
        torch.cuda.synchronize()
        clk.mark_stop()
        barrier(world)
        ms_total = start.elapsed_time(stop)
        ms_total = max_over_ranks(ms_total, world)
        # ---- per-stage breakdown: a second pass with CUDA events between the
        # kernels (not part of the headline number; events between kernels keep
        # the next kernel from starting early) ----
        n_ev = max(3, min(args.steps, 50))
        evs = [[torch.cuda.Event(enable_timing=True) for _ in range(8)] for _ in range(n_ev)]
        for i in range(n_ev):
            step(evs[i])
        torch.cuda.synchronize()
    stage_ms = {s: 0.0 for s in STAGES}
    for e in evs:
        for j, s in enumerate(STAGES):
            stage_ms[s] += e[j].elapsed_time(e[j + 1])
    stage_ms = {s: v / n_ev for s, v in stage_ms.items()}
    alone = stages_alone(x, wr) if rank == 0 else None
    clocks = clk.summary()
    value = N * world * args.steps / (ms_total / 1000.0)
    parity = None if args.skip_parity else parity_check(x, wr, w1, b1, w2, b2, out)

    if args.skip_e2e:
        e2e_value = None
    else:
        e2e_value = run_e2e(args, world, dev, sd, x, out, N, stream)
        e2e_value["copy_roofline"] = copy_roofline(dev, x.numel() * 2, e2e_value["value"], N)
    decode = None if args.skip_decode else run_decode(args, dev, stream)
    train = None
    if not args.skip_train:
        train = run_train(args, dev, stream)
        # The reference's production MoE (agillm41.py:8590-8594: --moe_experts 2 --moe_top_k 1
        # --moe_mlp_mult 4 --moe_shared_experts 1 --moe_shared_mlp_mult 2 --amp, batch 22 x 1536)
        train["production"] = run_train(args, dev, stream, experts=2, hidden=4 * D, top_k=1, shared=1,
                                        shared_hidden=2 * D, batch=22, seq=1536,
                                        label="production MoE block training step")
        train["production"]["forward"] = run_forward_production(args, dev, stream)
    if not args.skip_aux:
        aux = run_aux(args, dev, stream)
        if train is None:
            train = {"aux_loss": aux}
        else:
            train["aux_loss"] = aux
    codec_leg = None if args.skip_codec else run_codec(args, dev, stream, world == 1 and not args.skip_cpu)
    skewed = None if args.skip_skewed else run_skewed_single(args, dev, stream)
    block_ffn = None if args.skip_block else run_block_ffn(args, dev, stream, x, (w1, b1, w2, b2, wr))
    expert_stream = None
    if not args.skip_expert_stream:
        try:
            expert_stream = run_expert_stream(args, dev)
        except Exception as exc:  # a side leg must not take the headline line down with it
            expert_stream = {"error": f"{type(exc).__name__}: {exc}"}
    report(args, world, rank, N, ms_total, stage_ms, clocks, value, e2e_value, x, decode, train, codec_leg,
           parity=parity, skewed=skewed, block_ffn=block_ffn, alone=alone, expert_stream=expert_stream)


def run_block_ffn(args, dev, stream, x, weights):
    """The FFN half of the reference Block at this workload (agillm41.py:4547,
    `x + self.ff(self.ln2(x))`): torch's LayerNorm (ln2, d = 1280, seeded
    affine parameters) then agm_moe_forward_residual (the MoE block with the
    residual add fused into its combine). Reports the LayerNorm's share of
    that half, i.e. what a LayerNorm fused into the router and permute could
    save at most (its read of x and write of the normalised rows)."""
    import torch.nn.functional as F

    from agillm41_b200 import ops

    w1, b1, w2, b2, wr = weights
    g = torch.Generator(device="cpu").manual_seed(SEED + 11)
    ln_w = (1.0 + 0.1 * torch.randn(D, generator=g)).to(dev, torch.bfloat16)
    ln_b = (0.1 * torch.randn(D, generator=g)).to(dev, torch.bfloat16)

    def ln():
        return F.layer_norm(x, (D,), ln_w, ln_b, 1e-5)

    def block():
        return ops.moe_forward_residual(ln(), x, wr, w1, b1, w2, b2, TOP_K)

    def fused():
        return ops.moe_block_forward(x, ln_w, ln_b, 1e-5, wr, w1, b1, w2, b2, TOP_K)

    def our_ln():
        return ops.layernorm(x, ln_w, ln_b, 1e-5)

    def timed(fn, steps):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    steps = max(10, min(args.steps, 50))
    ln_ms = timed(ln, steps)
    block_ms = timed(block, steps)
    our_ln_ms = timed(our_ln, steps)
    fused_ms = timed(fused, steps)
    peaks = load_peaks()
    nbytes = 2 * x.numel() * 2
    return {"workload": f"x + MoEFFN(LayerNorm(x)), B{BATCH} L{SEQ} d{D} bf16",
            "ms_per_step": round(fused_ms, 4), "tokens_per_s": x.shape[0] / (fused_ms / 1000.0),
            "api": "agm_moe_block_forward (LayerNorm kernel + forward with the residual in the combine)",
            "layernorm_ms": round(our_ln_ms, 4),
            "layernorm_hbm_frac": round(nbytes / (our_ln_ms / 1000.0) / 1e9 / peaks["hbm"], 3),
            "with_torch_layernorm": {"ms_per_step": round(block_ms, 4), "layernorm_ms": round(ln_ms, 4),
                                     "layernorm_hbm_frac": round(nbytes / (ln_ms / 1000.0) / 1e9 / peaks["hbm"], 3)},
            "note": "LayerNorm roofline: it reads x and writes the normalised rows (2 x 189 MB)"}


def pack_weights(sd, experts=EXPERTS):
    """[E, ...] expert weight stacks and the router weight of a state dict."""
    w1 = torch.stack([sd[f"experts.{e}.0.weight"] for e in range(experts)]).contiguous()
    b1 = torch.stack([sd[f"experts.{e}.0.bias"] for e in range(experts)]).contiguous()
    w2 = torch.stack([sd[f"experts.{e}.2.weight"] for e in range(experts)]).contiguous()
    b2 = torch.stack([sd[f"experts.{e}.2.bias"] for e in range(experts)]).contiguous()
    return w1, b1, w2, b2, sd["router.weight"].contiguous()


def parity_check(x, wr, w1, b1, w2, b2, out, slice_tokens=4096):
    """Parity of the timed forward's output (run after the timed region).

    Routing: the reference computes its router logits with torch's library
    GEMM (``F.linear(x, W_r).float()``, agillm41.py:4399) and picks
    ``topk`` of them (4418). The kernel's routing is compared with that over
    the whole workload: tokens routed differently, and how many of those are
    explained (the kernel's logit differs from the library's, whose bf16
    rounding of split-K partial sums is not the correctly rounded value, or
    the library's top k+1 logits hold an exact tie).
    Output: on the first ``slice_tokens`` tokens whose routing matches, the
    largest error of the timed output against an fp32 evaluation of the
    block's formula (gate-weighted FC2(ReLU(FC1 x)) over the chosen experts,
    from the same bf16 weights and gates), and the fraction of elements
    outside the bf16 parity bound 1e-2 + 2e-2 |ref|.
    """
    import torch.nn.functional as F
    from agillm41_b200 import ops

    with torch.no_grad():
        lib_logits = F.linear(x, wr).float()
        ref_idx = torch.topk(lib_logits, TOP_K, dim=-1).indices
        _, ex = ops.moe_forward(x, wr, w1, b1, w2, b2, TOP_K, want=("idx", "gates", "logits"))
        idx = ex["idx"].long()
        diff = (idx != ref_idx).any(dim=1)
        n_diff = int(diff.sum())
        logit_differs = (ex["logits"] != lib_logits).any(dim=1)
        top = torch.topk(lib_logits, TOP_K + 1, dim=-1).values
        tie = (top[:, 1:] == top[:, :-1]).any(dim=1)
        explained = int((diff & (logit_differs | tie)).sum())
        n = min(slice_tokens, x.shape[0])
        ok = ~diff[:n]
        xs = x[:n].float()
        gates = ex["gates"][:n].float()
        ref = torch.zeros(n, D, dtype=torch.float32, device=x.device)
        for r in range(TOP_K):
            for e in range(EXPERTS):
                rows = (idx[:n, r] == e).nonzero().flatten()
                if rows.numel() == 0:
                    continue
                h = torch.relu(xs[rows] @ w1[e].float().t() + b1[e].float())
                h = h.to(torch.bfloat16).float()            # the reference rounds the hidden to the dtype
                y = h @ w2[e].float().t() + b2[e].float()
                ref.index_add_(0, rows, y * gates[rows, r:r + 1])
        o = out[:n].float()
        err = (o - ref).abs()[ok]
        bound = 1e-2 + 2e-2 * ref.abs()[ok]
    return {"tokens": int(x.shape[0]), "routed_differently": n_diff, "explained": explained,
            "unexplained": n_diff - explained,
            "routing_reference": "torch F.linear(x, W_r).float() then topk (the reference's library GEMM)",
            "output_slice_tokens": n, "output_rows_compared": int(ok.sum()),
            "max_abs_err": float(err.max()) if err.numel() else 0.0,
            "frac_outside_bf16_bound": float((err > bound).float().mean()) if err.numel() else 0.0,
            "output_reference": "fp32 evaluation of sum_r g_r FC2_e(ReLU(FC1_e x)) from the bf16 weights and "
                                "the kernel's gates, hidden rounded to bf16"}


def copy_roofline(dev, nbytes, e2e_tokens_per_s, n_tokens, reps=10):
    """Pinned host<->device copy rates on this box, the ceiling of the
    end-to-end leg: H2D alone, D2H alone, and both at once on two streams
    (what the host pipeline overlaps), each of ``nbytes`` per step. The e2e
    fraction is the bidirectional copy time of one step's input and output
    over the e2e step time."""
    h_in = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    h_out = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    d_in = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    d_out = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    s1, s2 = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def run(h2d, d2h, n):
        for _ in range(n):
            if h2d:
                with torch.cuda.stream(s1):
                    d_in.copy_(h_in, non_blocking=True)
            if d2h:
                with torch.cuda.stream(s2):
                    h_out.copy_(d_out, non_blocking=True)

    def timed(h2d, d2h):
        run(h2d, d2h, 2)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        run(h2d, d2h, reps)
        torch.cuda.synchronize()
        return (time.perf_counter() - t0) / reps

    t_h2d, t_d2h, t_bi = timed(True, False), timed(False, True), timed(True, True)
    e2e_step = n_tokens / e2e_tokens_per_s
    return {"bytes_each_way": nbytes, "h2d_gbs": round(nbytes / t_h2d / 1e9, 2),
            "d2h_gbs": round(nbytes / t_d2h / 1e9, 2), "bidirectional_gbs_each_way": round(nbytes / t_bi / 1e9, 2),
            "bidirectional_ms": round(1000 * t_bi, 3), "e2e_ms_per_step": round(1000 * e2e_step, 3),
            "frac": round(t_bi / e2e_step, 3),
            "note": "pinned buffers, host wall clock over 10 copies; frac = bidirectional copy time of one step's "
                    "input and output / e2e step time"}


def run_expert_stream(args, dev, n_tokens=64, steps=10):
    """Host-resident experts (the module's set_expert_stream(True); the
    reference's _run_expert, agillm41.py:4367-4379, and its block streaming,
    7656-7668): a decode batch of 64 tokens through MoEFFN.forward with the
    routed experts on the host. The forward routes on the GPU, reads the
    per-expert row counts, copies each active expert's weights once from a
    page-locked pack while the rows are permuted, and runs the same kernels.
    Bound: the pinned host-to-device copy of the active experts' weights,
    timed on this box for the same bytes. The reference instead moves an
    expert to the GPU and back for every (rank, expert) call with rows
    (pageable copies, then empty_cache); its bytes are reported, not timed.
    Host wall clock per forward (the forward holds one host read)."""
    import agillm41_b200
    from agillm41_b200 import ops, synthetic

    m = agillm41_b200.MoEFFN(D, mlp_mult=4, experts=EXPERTS, top_k=TOP_K)
    m.experts = torch.nn.ModuleList([torch.nn.Sequential(torch.nn.Linear(D, HIDDEN), torch.nn.ReLU(),
                                                         torch.nn.Linear(HIDDEN, D)) for _ in range(EXPERTS)])
    m.load_state_dict(synthetic.make_state(D, HIDDEN, EXPERTS, SEED + 7))
    m = m.to(device=dev, dtype=torch.bfloat16).eval()
    x = synthetic.make_input(n_tokens, D, SEED + 7, dtype=torch.bfloat16, device=dev)
    with torch.no_grad():
        idx, _, _, _ = ops.router_topk(x, m.router.weight.detach().contiguous(), TOP_K)
    per_rank = torch.stack([torch.bincount(idx[:, r].long(), minlength=EXPERTS) for r in range(TOP_K)]).cpu()
    active = int((per_rank.sum(0) > 0).sum())
    calls = int((per_rank > 0).sum())
    for ex in m.experts:
        ex.to("cpu")

    def timed(empty_cache):
        m.set_expert_stream(True, empty_cache=empty_cache)
        with torch.no_grad():
            for _ in range(3):
                m(x)
            torch.cuda.synchronize(dev)
            t0 = time.perf_counter()
            for _ in range(steps):
                m(x)
            torch.cuda.synchronize(dev)
        return (time.perf_counter() - t0) / steps

    dt_keep = timed(False)
    dt = timed(True)
    per_expert = 2 * (2 * D * HIDDEN + HIDDEN + D)  # bf16 W1, b1, W2, b2
    h2d = active * per_expert
    h_buf = torch.empty(h2d, dtype=torch.uint8).pin_memory()
    d_buf = torch.empty(h2d, dtype=torch.uint8, device=dev)
    d_buf.copy_(h_buf, non_blocking=True)
    torch.cuda.synchronize(dev)
    t1 = time.perf_counter()
    for _ in range(5):
        d_buf.copy_(h_buf, non_blocking=True)
    torch.cuda.synchronize(dev)
    h2d_gbs = h2d / ((time.perf_counter() - t1) / 5) / 1e9
    achieved = h2d / dt / 1e9
    return {
        "workload": f"MoE block forward with host-resident experts (expert streaming), {n_tokens} tokens, d{D} "
                    f"E{EXPERTS} H{HIDDEN} top{TOP_K} bf16, seed {SEED + 7}",
        "ms_per_step": round(1000 * dt, 3), "tokens_per_s": n_tokens / dt, "steps": steps,
        "active_experts": active, "h2d_bytes_per_step": h2d,
        "timing": "host wall clock per forward (one host read of the counts inside), after 3 warm-up forwards",
        "roofline": {"bound": "pcie", "achieved": round(achieved, 2), "peak": round(h2d_gbs, 2), "unit": "GB/s",
                     "frac": round(achieved / h2d_gbs, 3),
                     "peak_source": "pinned host-to-device copy of the same bytes on this box, one stream"},
        "empty_cache_false": {"ms_per_step": round(1000 * dt_keep, 3),
                              "achieved_gbs": round(h2d / dt_keep / 1e9, 2),
                              "frac": round(h2d / dt_keep / 1e9 / h2d_gbs, 3),
                              "note": "set_expert_stream(True, empty_cache=False): the device copies stay in the "
                                      "allocator's cache between forwards; the headline figures above use the "
                                      "default (empty_cache=True, as the reference), which returns them to the "
                                      "driver after every forward"},
        "reference_loop_bytes_per_step": 2 * calls * per_expert,
        "reference_loop_note": f"{calls} (rank, expert) calls with rows, each moving its expert to the GPU and "
                               "back (pageable), then torch.cuda.empty_cache()",
    }


def skewed_workload(dev, rank, n_tokens):
    """The expert-parallel configuration's per-rank workload: B x L tokens of
    this rank (input seed 3 + 1000 * rank), weights seed 3 whose router
    carries the Zipf(1.2) per-expert logit bias (~5:1 max/mean expert load)."""
    from agillm41_b200 import synthetic

    bias = synthetic.zipf_logit_bias(EXPERTS, EP_SEED, s=ZIPF_S, scale=ZIPF_SCALE)
    sd = synthetic.make_state(D, HIDDEN, EXPERTS, EP_SEED, dtype=torch.bfloat16, device=dev,
                              router_logit_bias=bias)
    x = synthetic.make_input(n_tokens, D, EP_SEED + 1000 * rank, dtype=torch.bfloat16, device=dev,
                             pin_feature0=True)
    return x, pack_weights(sd)


def run_skewed_single(args, dev, stream):
    """The skewed (Zipf) routing workload of the expert-parallel runs on one
    GPU: the same per-rank work as ``skewed`` at N > 1, so that its scaling
    compares like with like."""
    from agillm41_b200 import ops

    x, (w1, b1, w2, b2, wr) = skewed_workload(dev, 0, args.tokens)
    out = torch.empty_like(x)
    for _ in range(max(3, args.warmup)):
        ops.moe_forward(x, wr, w1, b1, w2, b2, TOP_K, out=out)
    torch.cuda.synchronize()
    steps = max(10, min(args.steps, 100))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        ops.moe_forward(x, wr, w1, b1, w2, b2, TOP_K, out=out)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    _, ex = ops.moe_forward(x, wr, w1, b1, w2, b2, TOP_K, want=("counts",))
    c = ex["counts"].float()
    return {"workload": f"MoE block forward, {args.tokens} tokens d{D} E{EXPERTS} H{HIDDEN} top{TOP_K} bf16, "
                        f"Zipf({ZIPF_S}) router logit bias x{ZIPF_SCALE} (seed {EP_SEED})",
            "value": args.tokens / (ms / 1000.0), "unit": UNIT, "ms_per_step": round(ms, 4), "steps": steps,
            "expert_load_max_over_mean": round(float(c.max() / c.mean()), 3),
            "placement": "single GPU (all experts)"}


def run_forward_production(args, dev, stream):
    """Inference forward of the reference's production MoE (2 experts, top-1,
    H = 4d, one shared expert of 2d, agillm41.py:8590-8594) in bf16 over
    22 x 1536 tokens: tokens/s and the expert GEMMs' rate over the whole
    forward (router, permute and combine included)."""
    from agillm41_b200 import ops, synthetic

    E, H, k, Hs, N = 2, 4 * D, 1, 2 * D, 22 * 1536
    sd = synthetic.make_state(D, H, E, SEED, dtype=torch.bfloat16, device=dev, shared=1, shared_hidden=Hs)
    w = [torch.stack([sd[f"experts.{e}.{i}.{p}"] for e in range(E)]).contiguous()
         for i, p in ((0, "weight"), (0, "bias"), (2, "weight"), (2, "bias"))]
    sh = tuple(sd[f"shared.0.{i}.{p}"].unsqueeze(0).contiguous()
               for i, p in ((0, "weight"), (0, "bias"), (2, "weight"), (2, "bias")))
    wr = sd["router.weight"].contiguous()
    x = synthetic.make_input(N, D, SEED, dtype=torch.bfloat16, device=dev)
    out = torch.empty_like(x)

    def step():
        ops.moe_forward(x, wr, *w, k, shared=sh, out=out)

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    steps = max(10, min(args.steps, 100))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    peaks = load_peaks()
    flop = 4 * D * (k * H + Hs) * N
    tf = flop / (ms / 1000.0) / 1e12
    return {"workload": f"production MoE block forward, B22 L1536 ({N} tokens) d{D} E{E} H{H} top{k} + 1 shared "
                        f"H{Hs}, bf16, seed {SEED}",
            "ms_per_step": round(ms, 4), "tokens_per_s": N / (ms / 1000.0), "steps": steps,
            "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": peaks["tf_sus"], "unit": "TFLOP/s",
                         "frac": round(tf / peaks["tf_sus"], 3),
                         "note": "expert and shared GEMM FLOPs over the whole forward"},
            "gpu_launches_per_step": 6,   # router, plan, permute, FC1 (+ shared FC1), FC2 (+ shared FC2), combine
            "shared_folded": True}


def run_train(args, dev, stream, *, experts=EXPERTS, hidden=HIDDEN, top_k=TOP_K, shared=0, shared_hidden=0,
              batch=BATCH, seq=SEQ, label="MoE block training step"):
    """Training step of the MoE block as the reference trains it with --amp
    (torch.autocast bf16 over fp32 master weights, agillm41.py:3054-3066 and
    6793): the 16-bit casts of the fp32 weights (an optimiser step changes
    them every step), the forward that keeps its intermediates and the
    backward to dx, the router weight and every expert (and shared-expert)
    weight and bias, on a B x L token workload (fp32 x and upstream gradient,
    seeded). GEMM work per step: the forward projections plus their dgrad and
    wgrad, 3 x 4 x d x (k H + S Hs) FLOP per token.
    """
    from agillm41_b200 import ops, synthetic

    N = batch * seq if args.tokens == BATCH * SEQ else args.tokens
    sd = synthetic.make_state(D, hidden, experts, SEED, dtype=torch.float32, device=dev, shared=shared,
                              shared_hidden=shared_hidden or None)
    master = (sd["router.weight"].contiguous(),
              torch.stack([sd[f"experts.{e}.0.weight"] for e in range(experts)]).contiguous(),
              torch.stack([sd[f"experts.{e}.0.bias"] for e in range(experts)]).contiguous(),
              torch.stack([sd[f"experts.{e}.2.weight"] for e in range(experts)]).contiguous(),
              torch.stack([sd[f"experts.{e}.2.bias"] for e in range(experts)]).contiguous())
    smaster = None
    if shared:
        smaster = tuple(torch.stack([sd[f"shared.{s}.{i}.{p}"] for s in range(shared)]).contiguous()
                        for i, p in ((0, "weight"), (0, "bias"), (2, "weight"), (2, "bias")))
    del sd
    x = synthetic.make_input(N, D, SEED, dtype=torch.float32, device=dev)
    g = torch.Generator(device="cpu").manual_seed(SEED + 7)
    dout = torch.randn(N, D, generator=g).to(dev)

    def step(check=False):
        wc = [ops.cast_f32(t, torch.bfloat16) for t in master]
        sc = None if smaster is None else tuple(ops.cast_f32(t, torch.bfloat16) for t in smaster)
        out, saved = ops.moe_forward_train(x, *wc, top_k, shared=sc, check_errors=check)
        return ops.moe_backward(dout, saved, wc[0], wc[1], wc[3], top_k, shared=sc, check_errors=check)

    for i in range(max(3, args.warmup)):
        step(check=(i == 0))
    torch.cuda.synchronize()
    steps = max(3, min(args.steps, 30))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    peaks = load_peaks()
    flop = 3 * 4 * D * (top_k * hidden + shared * shared_hidden) * N
    tf = flop / (ms / 1000.0) / 1e12
    shared_txt = f" + {shared} shared H{shared_hidden}" if shared else ""
    # launches: 5 (+4) weight casts; forward: x cast, router, plan, permute, FC1, FC2, 2 per shared
    # expert, combine; backward: combine/routing, FC2 wgrad + dgrad, 2 x (column sums + reduce), FC1
    # wgrad + dgrad, router wgrad + reduce, dx, and per shared expert 4 GEMMs + bias reduce (+ db2 once)
    launches = 24 + (4 + 2 + 2 + 5 * shared if shared else 0)
    return {"workload": f"{label} (forward + backward), B{batch} L{seq} ({N} tokens) d{D} E{experts} "
                        f"H{hidden} top{top_k}{shared_txt}, autocast bf16 over fp32 master weights, seed {SEED}",
            "ms_per_step": round(ms, 4), "tokens_per_s": N / (ms / 1000.0), "steps": steps,
            "gemm_flop_per_step": flop,
            "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": peaks["tf_sus"], "unit": "TFLOP/s",
                         "frac": round(tf / peaks["tf_sus"], 3),
                         "note": "all expert GEMMs' FLOPs over the whole step time (casts, router, permute, "
                                 "combine and their backward included), so a lower bound on the GEMMs' own rate"},
            "gpu_launches_per_step": launches}


def run_aux(args, dev, stream):
    """Auxiliary router losses (_collect_moe_aux, agillm41.py:4463-4492) as the
    autocast trainer calls them after its forward: the fp32 stashed router
    input of B x L tokens and the fp32 router weight, load-balance 0.01 and
    router-z 0.001 (the production run's coefficients, agillm41.py:8591); one
    step = agm_moe_aux_forward + agm_moe_aux_backward. Each reads the input
    once: 2 x N x d x 4 bytes of algorithmic traffic (plus the [N, E] logits,
    written once and read twice)."""
    from agillm41_b200 import ops, synthetic

    N = BATCH * SEQ if args.tokens == BATCH * SEQ else args.tokens
    w = synthetic.make_state(D, D, EXPERTS, SEED, dtype=torch.float32, device=dev)["router.weight"].contiguous()
    x = synthetic.make_input(N, D, SEED, dtype=torch.float32, device=dev)
    g = torch.ones((), device=dev)

    def step():
        loss, saved = ops.moe_aux_forward(x, w, 0.01, 0.001)
        return loss, ops.moe_aux_backward(g, x, w, saved)

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    steps = max(10, min(args.steps, 100))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    peaks = load_peaks()
    nbytes = 2 * N * D * 4 + 3 * N * EXPERTS * 4
    gbs = nbytes / (ms / 1000.0) / 1e9
    return {"workload": f"MoE auxiliary losses forward + backward, {N} tokens d{D} E{EXPERTS}, fp32 stash and "
                        f"router weight, aux 0.01 z 0.001, seed {SEED}",
            "ms_per_step": round(ms, 4), "steps": steps,
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm"], "unit": "GB/s",
                         "frac": round(gbs / peaks["hbm"], 3),
                         "note": "the input read once by each pass plus the logits, over both passes' time"},
            "gpu_launches_per_step": 6}


def _codec_layer_state():
    """A codec state (the reference's tensor codec, agillm41.py:4858-5074)
    holding one production MoE layer's expert tensors (2 experts, d = 1280,
    H = 4d; 26.2 M values): seeded Gaussian weights quantised row-wise to int8
    with fp16 row scales, biases to int8 with one scale, zlib level 1 behind
    the "ZLIB" tag (the reference's compressor without zstandard)."""
    import zlib

    import numpy as np

    rng = np.random.default_rng(SEED)
    H = 4 * D
    shapes = {}
    for e in range(2):
        shapes[f"experts.{e}.0.weight"] = (H, D)
        shapes[f"experts.{e}.0.bias"] = (H,)
        shapes[f"experts.{e}.2.weight"] = (D, H)
        shapes[f"experts.{e}.2.bias"] = (D,)
    tensors = {}
    for key, shape in shapes.items():
        w = rng.standard_normal(shape, dtype=np.float32) * 0.02
        item = {"shape": list(shape), "orig_dtype": "float32", "packed_dtype": "int8", "codec": "zstd"}
        if len(shape) == 2:
            s = np.maximum(np.abs(w).max(axis=1) / 127.0, 1e-12).astype(np.float16)
            q = np.clip(np.rint(w / s.astype(np.float32)[:, None]), -127, 127).astype(np.int8)
            item.update(pack_kind="int8_rowwise", rows=shape[0], cols=shape[1], scales_dtype="float16",
                        scales_codec="raw", scales_data=torch.from_numpy(s.view(np.uint8).copy()))
        else:
            scale = max(float(np.abs(w).max()) / 127.0, 1e-12)
            q = np.clip(np.rint(w / scale), -127, 127).astype(np.int8)
            item.update(pack_kind="int8_symmetric", scale=scale)
        item["data"] = torch.frombuffer(bytearray(b"ZLIB" + zlib.compress(q.tobytes(), 1)), dtype=torch.uint8)
        tensors[key] = item
    return {"__agillm43_tensor_state_codec__": "agillm43_tensor_state_v3_rowq8c", "mode": "rowq8-zstd",
            "plain": {}, "tensors": tensors}, shapes


def run_codec(args, dev, stream, cpu_leg):
    """Tensor-codec decode of one production MoE layer's experts into fp32
    device parameters (the side-update consumer's copy, agillm41.py:6029-6046):

    * kernel: agm_codec_decode over the int8 payloads already in device memory,
      algorithmic bytes = 1 B read + 4 B written per value (+ row scales);
    * e2e: agillm41_b200.codec.apply_tensor_state from the compressed host
      state (threaded decompression, pinned H2D of the packed bytes, decode);
    * cpu_baseline: the reference's path (decode_tensor_state on the host's
      cores, then value.to(device) and copy_), restated by the oracle.
    """
    from agillm41_b200 import _lib, codec
    from agillm41_b200._lib import load, ptr, stream_handle

    state, shapes = _codec_layer_state()
    targets = {k: torch.empty(v, dtype=torch.float32, device=dev) for k, v in shapes.items()}
    n_total = sum(v[0] * (v[1] if len(v) > 1 else 1) for v in shapes.values())
    # kernel leg: payloads resident on the device
    staged = [codec._Payload(k, it) for k, it in state["tensors"].items()]
    dev_q = [(p, p.packed.to(dev), None if p.scales is None else p.scales.to(dev)) for p in staged]
    lib = load()

    import ctypes

    table = (_lib.AgmCodecTensor * len(dev_q))(*[p.entry(q, sc, targets[p.key]) for p, q, sc in dev_q])

    def kernels():
        # agm_codec_decode_batch: the four weight tensors in one launch, the
        # four biases in another
        rc = lib.agm_codec_decode_batch(ctypes.cast(table, ctypes.c_void_p), len(dev_q), _lib.AGM_APPLY_COPY, 1.0,
                                        stream_handle(dev))
        _lib.check(rc, "agm_codec_decode_batch")

    for _ in range(3):
        kernels()
    torch.cuda.synchronize()
    # The decode replayed as a CUDA graph, so that the device time is not
    # bounded by the host's launch rate.
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        kernels()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    steps = max(10, min(args.steps, 50))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    cur = torch.cuda.current_stream(dev)
    e0.record(cur)
    for _ in range(steps):
        graph.replay()
    e1.record(cur)
    torch.cuda.synchronize()
    k_ms = e0.elapsed_time(e1) / steps
    del graph
    scale_bytes = sum(p.scales.numel() for p in staged if p.scales is not None)
    nbytes = n_total * (1 + 4) + scale_bytes
    gbs = nbytes / (k_ms / 1000.0) / 1e9
    peaks = load_peaks()
    # e2e leg: compressed host state -> applied device parameters
    for _ in range(2):
        codec.apply_tensor_state(state, targets)
    torch.cuda.synchronize()
    e2e_steps = 5
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        codec.apply_tensor_state(state, targets)
    torch.cuda.synchronize()
    e2e_ms = (time.perf_counter() - t0) * 1000.0 / e2e_steps
    h2d = sum(p.packed.numel() for p in staged) + scale_bytes
    out = {"workload": f"tensor-codec decode of one production MoE layer's experts (2 experts, d{D}, H{4 * D}: "
                       f"{n_total} values, row-wise int8 weights, int8 biases) into fp32 device parameters",
           "kernel_ms": round(k_ms, 4), "values_per_s": n_total / (k_ms / 1000.0), "steps": steps,
           "timing": "CUDA events around graph replays of the layer's decode (two launches), payloads resident in HBM",
           "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm"], "unit": "GB/s",
                        "frac": round(gbs / peaks["hbm"], 3),
                        "note": "1 B of int8 read and 4 B of fp32 written per value, plus the row scales"},
           "e2e": {"ms": round(e2e_ms, 3), "values_per_s": n_total / (e2e_ms / 1000.0),
                   "h2d_bytes": int(h2d), "note": "host wall clock from the compressed state to applied "
                                                  "parameters: threaded zlib, pinned H2D, decode"},
           "gpu_launches_per_step": 2}
    if cpu_leg:
        from oracle import codec_oracle

        for _ in range(1):
            for k, v in codec_oracle.decode_tensor_state(state).items():
                codec_oracle.apply_value(targets[k], v)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        reps = 3
        for _ in range(reps):
            for k, v in codec_oracle.decode_tensor_state(state).items():
                codec_oracle.apply_value(targets[k], v)
            torch.cuda.synchronize()
        c_ms = (time.perf_counter() - t0) * 1000.0 / reps
        out["cpu_baseline"] = {"ms": round(c_ms, 3), "values_per_s": n_total / (c_ms / 1000.0),
                               "cores": torch.get_num_threads(), "kind": "port",
                               "sample": "the whole layer: the reference's decode on the host (zlib, int8 x scale "
                                         "in fp32) then value.to(device) and copy_ per tensor"}
    return out


def _ep_variant(args, world, rank, dev, stream, x, weights, ref, counts_all, kind, placement, replicas=None,
                chunks=1, reserve_sms=20):
    """Time one expert-parallel variant on this rank's tokens x; the max over
    ranks of the device time of exactly args.steps forwards."""
    import torch.distributed as dist

    from agillm41_b200 import ep

    w1, b1, w2, b2, wr = weights
    N = x.shape[0]
    mine = ep.ExpertParallelMoE.shard_weights(w1, b1, w2, b2, rank, world, placement, replicas=replicas)
    if kind == "p2p":
        moe = ep.P2PExpertParallelMoE((wr,) + tuple(mine), TOP_K, EXPERTS, max_tokens=N, placement=placement,
                                      chunks=chunks, replicas=replicas, reserve_sms=reserve_sms)
    else:
        moe = ep.ExpertParallelMoE((wr,) + tuple(mine), TOP_K, EXPERTS, placement=placement)
    for _ in range(args.warmup):
        out = moe.forward(x)
    torch.cuda.synchronize()
    same = bool(torch.equal(out, ref))
    names = P2P_STAGES if kind == "p2p" else EP_STAGES
    evs = None if chunks > 1 else [[torch.cuda.Event(enable_timing=True) for _ in range(len(names) + 1)]
                                   for _ in range(args.steps)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(dev) as clk:
        barrier(world)
        clk.mark_start()
        start.record(stream)
        for i in range(args.steps):
            moe.forward(x)
        stop.record(stream)
        torch.cuda.synchronize()
        clk.mark_stop()
        barrier(world)
        # per-phase pass (events between the phases; not the headline number)
        if evs is not None:
            for i in range(args.steps):
                moe.forward(x, events=evs[i])
            torch.cuda.synchronize()
    ms = max_over_ranks(start.elapsed_time(stop), world)
    st = None
    if evs is not None:
        st = {s_: 0.0 for s_ in names}
        for e in evs:
            for j, s_ in enumerate(names):
                st[s_] += e[j].elapsed_time(e[j + 1])
        st = {s_: round(max_over_ranks(v / args.steps, world), 4) for s_, v in st.items()}
    if kind == "p2p":
        same = same and moe.device_error() == 0
        moe.close()
    if kind == "p2p":
        masks = ep.holder_masks(EXPERTS, world, placement, replicas)
        units = ep.rank_loads(counts_all, placement, masks)
        works = [int(2 * u) for u in units]                     # 128-row tiles (units of 256 rows)
    else:
        works = [ep.plan_dispatch(counts_all, r, placement).recv_tile_expert.size for r in range(world)]
    ok = torch.tensor([1.0 if same else 0.0], device=dev)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    mean = sum(works) / world
    res = dict(value=N * world * args.steps / (ms / 1000.0), ms_per_step=ms / args.steps, stages_ms=st,
               tiles_per_rank=works, max_over_mean_tiles=round(max(works) / mean, 3) if mean else None,
               placement_bound_efficiency=round(mean / max(works), 3) if max(works) else None,
               bit_identical_to_single_gpu=bool(ok.item() > 0), clocks=clk.summary())
    if replicas is not None:
        res["replicas"] = replicas
    return res


def _gathered_counts(x, weights, world):
    import torch.distributed as dist

    from agillm41_b200 import ops

    w1, b1, w2, b2, wr = weights
    counts = ops.moe_forward(x, wr, w1, b1, w2, b2, TOP_K, want=("counts",))[1]["counts"].to(torch.int32)
    counts_all = torch.empty(world * EXPERTS, dtype=torch.int32, device=x.device)
    dist.all_gather_into_tensor(counts_all, counts.contiguous())
    return counts_all.cpu().numpy().reshape(world, EXPERTS)


EP_DECLARED = "replicated"     # the placement of the N > 1 headline
EP_BUDGET = 2                  # replicas per rank on top of the static ownership


def run_ep(args, world, rank, local):
    """Expert-parallel forward over `world` GPUs (one process each).

    Headline (``value``): the same per-rank workload as the one-GPU line (B x
    L = 73,728 tokens of this rank, weights seed 1, input seed 1 + 1000 x
    rank), so value(N) / (N x value(1)) compares like with like, on ONE
    declared placement: "replicated" = the static ownership the configuration
    names (14 experts over 2/4/8 ranks: 7/7, 4/4/3/3, 2x6+1x2) plus replicas
    of the experts that make a rank busiest, at most 2 extra experts per rank,
    chosen at set-up from the all-gathered counts of one calibration forward
    (ep.choose_replicas); each forward splits a replicated expert's rows among
    its holders on the device. Rows move inside the permute kernel and the
    FC2 epilogue over NVLink peer memory.
    Extra keys: ``placements`` (the same workload under static, balanced and
    local placements) and ``skewed`` (the expert-parallel configuration's
    Zipf(1.2)-skewed routing, weights seed 3, input seed 3 + 1000 x rank:
    replicated, static, local and the NCCL all-to-all static path), each with
    per-phase times, tiles per rank and the placement-implied efficiency bound.
    """
    from agillm41_b200 import ep, ops, synthetic

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    N = args.tokens
    stream = torch.cuda.current_stream(dev)
    sd = synthetic.make_state(D, HIDDEN, EXPERTS, SEED, dtype=torch.bfloat16, device=dev)
    x = synthetic.make_input(N, D, SEED + rank * 1000, dtype=torch.bfloat16, device=dev)
    weights = pack_weights(sd)
    w1, b1, w2, b2, wr = weights
    ref = ops.moe_forward(x, wr, w1, b1, w2, b2, TOP_K)          # single-GPU forward of this rank's tokens
    counts_all = _gathered_counts(x, weights, world)
    replicas = ep.choose_replicas(counts_all, budget=EP_BUDGET)
    head = _ep_variant(args, world, rank, dev, stream, x, weights, ref, counts_all, "p2p", EP_DECLARED, replicas)
    others = {}
    if not args.skip_ep_variants:
        for placement in ("static", "balanced", "local"):
            others[f"p2p_{placement}"] = _ep_variant(args, world, rank, dev, stream, x, weights, ref, counts_all,
                                                     "p2p", placement)

    skewed = {}
    if not args.skip_skewed:
        xs, wsk = skewed_workload(dev, rank, N)
        ref_s = ops.moe_forward(xs, wsk[4], *wsk[:4], TOP_K)
        counts_s = _gathered_counts(xs, wsk, world)
        reps_s = ep.choose_replicas(counts_s, budget=EP_BUDGET)
        skewed["p2p_replicated"] = _ep_variant(args, world, rank, dev, stream, xs, wsk, ref_s, counts_s, "p2p",
                                               "replicated", reps_s)
        if not args.skip_ep_variants:
            for kind, placement in (("p2p", "static"), ("p2p", "local"), ("nccl", "static")):
                skewed[f"{kind}_{placement}"] = _ep_variant(args, world, rank, dev, stream, xs, wsk, ref_s,
                                                            counts_s, kind, placement)
        c = counts_s.sum(axis=0).astype(float)
        skewed["expert_load_max_over_mean"] = round(float(c.max() / c.mean()), 3)
        skewed["workload"] = (f"expert-parallel MoE block forward, {N} tokens/rank d{D} E{EXPERTS} H{HIDDEN} "
                              f"top{TOP_K} bf16, Zipf({ZIPF_S}) logit bias x{ZIPF_SCALE} (seed {EP_SEED})")
        del xs, wsk, ref_s

    # End to end through the public API with host buffers (copy in, forward, copy out).
    mine = ep.ExpertParallelMoE.shard_weights(w1, b1, w2, b2, rank, world, EP_DECLARED, replicas=replicas)
    moe = ep.P2PExpertParallelMoE((wr,) + tuple(mine), TOP_K, EXPERTS, max_tokens=N, placement=EP_DECLARED,
                                  replicas=replicas)
    x_host = x.cpu().pin_memory()
    y_host = torch.empty_like(x_host).pin_memory()
    x_dev = torch.empty_like(x)

    def e2e_step():
        x_dev.copy_(x_host, non_blocking=True)
        y = moe.forward(x_dev)
        y_host.copy_(y, non_blocking=True)

    for _ in range(args.warmup):
        e2e_step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world)
    e2e_same = bool(torch.equal(y_host.to(dev), ref))
    moe.close()
    if rank != 0:
        return
    peaks = load_peaks()
    stages = head["stages_ms"]
    ffn_ms = stages["fc1"] + stages["fc2_to_owners"]
    # Grouped GEMM roofline: FLOPs of the busiest rank's FC1+FC2 launches / their event-timed duration.
    flop = 2 * 2 * TILE_ROWS * max(head["tiles_per_rank"]) * D * HIDDEN
    achieved = flop / (ffn_ms / 1000.0) / 1e12
    line = {
        "metric": METRIC, "value": head["value"], "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) input, N(0,0.02^2) random-init expert weights)",
        "config": {"workload": f"MoE block forward B{BATCH} L{SEQ} d{D} E{EXPERTS} H{HIDDEN} top{TOP_K} bf16 "
                               f"seed{SEED} per rank (the one-GPU workload on every rank)",
                   "global_batch": BATCH * world, "seq_len": SEQ, "tokens_per_gpu": N,
                   "parallelism": f"expert parallel x{world}, placement '{EP_DECLARED}': static ownership "
                                  f"{[len(r) for r in ep.static_owner_ranges(EXPERTS, world)]} + at most "
                                  f"{EP_BUDGET} hot-expert replicas per rank {replicas}; rows moved by the permute "
                                  f"kernel and the FC2 epilogue over NVLink peer memory",
                   "l2": "inputs larger than L2; no flush"},
        "e2e": {"value": N * world * args.steps / (e2e_ms / 1000.0), "unit": UNIT,
                "h2d_bytes_per_step": x_host.numel() * 2, "d2h_bytes_per_step": y_host.numel() * 2,
                "api": "P2PExpertParallelMoE.forward with host copies", "output_matches": e2e_same},
        "gpu_launches": 10 * args.steps,   # router, plan, counts exchange, EP plan, permute, barrier, FC1, FC2, barrier, combine
        "roofline": {"kernel": "grouped_gemm_pair_kernel (FC1+FC2, busiest rank)", "bound": "tensor",
                     "achieved": round(achieved, 1), "peak": peaks["tf"], "unit": "TFLOP/s",
                     "frac": round(achieved / peaks["tf"], 3),
                     "peak_source": f"{peaks['src']} bf16 burst", "traffic": None},
        "placement": head,
        "placements": others,
        "skewed": skewed,
        "cpu_baseline": None,
        "clocks": head["clocks"],
    }
    print(json.dumps(line), flush=True)


def run_e2e(args, world, dev, sd, x, out, N, stream):
    """Same metric through the public module API on host buffers, copies timed.

    Headline: MoEFFN.forward_host (C ABI agm_moe_forward_host), which overlaps
    the host->device copy, the forward and the device->host copy chunk by
    chunk. Also reported: the plain sequence copy-in, MoEFFN.forward, copy-out.
    """
    import agillm41_b200

    m = agillm41_b200.MoEFFN(D, mlp_mult=4, experts=EXPERTS, top_k=TOP_K)
    m.experts = torch.nn.ModuleList([torch.nn.Sequential(torch.nn.Linear(D, HIDDEN), torch.nn.ReLU(),
                                                         torch.nn.Linear(HIDDEN, D)) for _ in range(EXPERTS)])
    m = m.to(device=dev, dtype=torch.bfloat16).eval()
    m.load_state_dict(sd)
    x_host = x.reshape(1, N, D).cpu().pin_memory()
    y_host = torch.empty_like(x_host).pin_memory()
    x_dev = torch.empty(1, N, D, dtype=torch.bfloat16, device=dev)

    def pipelined_step():
        with torch.no_grad():
            m.forward_host(x_host, out_host=y_host)

    def sequential_step():
        x_dev.copy_(x_host, non_blocking=True)
        with torch.no_grad():
            y = m(x_dev)
        y_host.copy_(y, non_blocking=True)

    def timed(step):
        for _ in range(max(1, args.warmup)):
            step()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier(world)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        ms = max_over_ranks(e0.elapsed_time(e1), world)
        return N * world * args.steps / (ms / 1000.0)

    seq = timed(sequential_step)
    assert torch.equal(y_host.reshape(N, D).to(dev), out), "module output differs from the timed forward"
    y_host.zero_()
    pipe = timed(pipelined_step)
    assert torch.equal(y_host.reshape(N, D).to(dev), out), "host-pipelined output differs from the timed forward"
    return {"value": pipe, "unit": UNIT, "h2d_bytes_per_step": x_host.numel() * 2,
            "d2h_bytes_per_step": y_host.numel() * 2, "api": "MoEFFN.forward_host (agm_moe_forward_host)",
            "sequential_copy_forward_copy": seq}


DECODE_LAYERS, DECODE_BATCH, DECODE_SEED = 28, 64, 2


def run_decode(args, dev, stream):
    """AR decode shape: 28 MoE layers (independent random-init weights,
    N(0, 0.02^2), seeds 1000 + layer) over 64 sequences x 1 new token; the
    input of layer l is the output of layer l-1 plus an N(0, 1) perturbation
    (seed 2). One step = all 28 layers. Timed eagerly and as one CUDA graph
    replay (the forward has no host synchronisation, so the 28 layers
    capture into a single graph). Roofline: the step must stream every
    active expert's weights once (Sum over layers and active experts of
    W1 + b1 + W2 + b2 bytes); 28 x 229.5 MB > L2, so no flush is needed.
    """
    from agillm41_b200 import ops, synthetic

    E, k, B = EXPERTS, TOP_K, DECODE_BATCH
    layers = []
    for layer in range(DECODE_LAYERS):
        sd = synthetic.make_state(D, HIDDEN, E, 1000 + layer, dtype=torch.bfloat16, device=dev)
        layers.append((sd["router.weight"].contiguous(),
                       torch.stack([sd[f"experts.{e}.0.weight"] for e in range(E)]).contiguous(),
                       torch.stack([sd[f"experts.{e}.0.bias"] for e in range(E)]).contiguous(),
                       torch.stack([sd[f"experts.{e}.2.weight"] for e in range(E)]).contiguous(),
                       torch.stack([sd[f"experts.{e}.2.bias"] for e in range(E)]).contiguous()))
        del sd
    g = torch.Generator(device="cpu").manual_seed(DECODE_SEED)
    x0 = torch.randn(B, D, generator=g).to(torch.bfloat16).to(dev)
    noise = [torch.randn(B, D, generator=g).to(torch.bfloat16).to(dev) for _ in range(DECODE_LAYERS)]
    xs = [torch.empty(B, D, dtype=torch.bfloat16, device=dev) for _ in range(DECODE_LAYERS + 1)]
    outs = [torch.empty(B, D, dtype=torch.bfloat16, device=dev) for _ in range(DECODE_LAYERS)]
    counts = [torch.empty(E, dtype=torch.int32, device=dev) for _ in range(DECODE_LAYERS)]
    ws = torch.empty(ops.workspace_bytes(B, D, E, k, HIDDEN, 0, 1, torch.bfloat16), dtype=torch.uint8, device=dev)
    lib = ops.load()

    keep = ops._lib.AGM_FLAG_KEEP_ERROR
    # the same weights in the decode tile layout (each 128 x 64 tile one contiguous 16 KB block)
    tiled = [(ops.decode_tile_layout(w1), ops.decode_tile_layout(w2)) for (_, w1, _, w2, _) in layers]
    use_tiles = [False]

    def step():
        ws[:4].zero_()                   # one clear of the error word per decode step
        xs[0].copy_(x0)
        flags = keep | (ops._lib.AGM_FLAG_DECODE_TILES if use_tiles[0] else 0)
        for layer, (wr, w1, b1, w2, b2) in enumerate(layers):
            if use_tiles[0]:
                w1, w2 = tiled[layer]
            # x_{l+1} = noise_l + MoE(x_l): the perturbation is added inside the combine kernel
            # (agm_moe_forward_residual; the same bits as a separate add)
            rc = lib.agm_moe_forward_residual(
                ops.ptr(xs[layer]), ops.ptr(noise[layer]), ops.dtype_code(torch.bfloat16), B, D, E, k, HIDDEN,
                ops.ptr(wr), ops.ptr(w1), ops.ptr(b1), ops.ptr(w2), ops.ptr(b2), 0, 1, None, None, None, None,
                ops.ptr(xs[layer + 1]), ops.ptr(ws), ws.numel(), flags, torch.cuda.current_stream(dev).cuda_stream)
            ops.check(rc, "agm_moe_forward_residual")

    def counts_pass():
        # one untimed pass that also writes the per-expert counts (the active experts per layer)
        for layer, (wr, w1, b1, w2, b2) in enumerate(layers):
            rc = lib.agm_moe_forward(
                ops.ptr(xs[layer]), ops.dtype_code(torch.bfloat16), B, D, E, k, HIDDEN, ops.ptr(wr), ops.ptr(w1),
                ops.ptr(b1), ops.ptr(w2), ops.ptr(b2), 0, 1, None, None, None, None, ops.ptr(outs[layer]),
                ops.ptr(ws), ws.numel(), keep, None, None, ops.ptr(counts[layer]), None, None, None,
                torch.cuda.current_stream(dev).cuda_stream)
            ops.check(rc, "agm_moe_forward")
            torch.add(outs[layer], noise[layer], out=chk)
            if not torch.equal(chk, xs[layer + 1]):
                raise RuntimeError("fused residual add differs from the separate add in the decode chain")

    def timed(fn, steps):
        for _ in range(max(3, args.warmup)):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(torch.cuda.current_stream(dev))
        for _ in range(steps):
            fn()
        e1.record(torch.cuda.current_stream(dev))
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    steps = max(10, min(args.steps, 50))
    eager_ms = timed(step, steps)
    err = ops._lib.read_device_error(ws[:4].view(torch.int32))
    if err:
        raise RuntimeError(f"device error word 0x{err:x} in the decode leg")
    ref_out = xs[-1].clone()
    chk = torch.empty(B, D, dtype=torch.bfloat16, device=dev)
    counts_pass()
    torch.cuda.synchronize()
    graph_ms = graph_tiles_ms = None
    try:
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            step()                       # one call on the capture stream before capturing
        torch.cuda.current_stream(dev).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        graph_ms = timed(graph.replay, steps)
        if not torch.equal(xs[-1], ref_out):
            raise RuntimeError("graph replay output differs from the eager decode step")
        del graph
        # the decode tile layout, captured the same way
        use_tiles[0] = True
        with torch.cuda.stream(side):
            step()
        torch.cuda.current_stream(dev).wait_stream(side)
        graph_t = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph_t):
            step()
        graph_tiles_ms = timed(graph_t.replay, steps)
        if not torch.equal(xs[-1], ref_out):
            raise RuntimeError("decode tile layout output differs from the nn.Linear layout")
        del graph_t
        use_tiles[0] = False
    except RuntimeError as exc:
        if "differs" in str(exc):
            raise
        graph_ms = graph_tiles_ms = None
        print(f"decode: CUDA graph capture unavailable: {exc}", file=sys.stderr)
    active = sum(int((c > 0).sum()) for c in counts)
    expert_bytes = 2 * (2 * D * HIDDEN + HIDDEN + D)
    wbytes = active * expert_bytes
    peaks = load_peaks()
    best = min(v for v in (eager_ms, graph_ms, graph_tiles_ms) if v is not None)
    layout = "decode tiles" if best == graph_tiles_ms else "nn.Linear"
    gbs = wbytes / (best / 1000.0) / 1e9
    return {"workload": f"AR decode: {DECODE_LAYERS} MoE layers x {B} tokens, d{D} E{E} H{HIDDEN} top{k} bf16, "
                        f"seed {DECODE_SEED}",
            "ms_per_step_eager": round(eager_ms, 4), "ms_per_step_graph": None if graph_ms is None else round(graph_ms, 4),
            "ms_per_step_graph_decode_tiles": None if graph_tiles_ms is None else round(graph_tiles_ms, 4),
            "weight_layout_of_best": layout,
            "us_per_layer": round(1000 * best / DECODE_LAYERS, 2), "tokens_per_s": B / (best / 1000.0),
            "steps": steps, "active_experts": active, "weight_bytes_per_step": wbytes,
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm"], "unit": "GB/s",
                         "frac": round(gbs / peaks["hbm"], 3), "peak_source": f"{peaks['src']} HBM copy"},
            # per layer: the decode front (router + plan + permute in one cluster launch), FC1, FC2, combine
            "gpu_launches_per_step": DECODE_KERNELS_PER_LAYER * DECODE_LAYERS,
            "residual": "perturbation added inside each layer's combine kernel (agm_moe_forward_residual)"}


PAIR_MIN_ROWS = 16384   # AGM_PAIR_MIN_ROWS: agm_moe_forward runs its expert GEMMs on CTA pairs from k*N rows up


def gemm_kernel_name(n_tokens):
    if TOP_K * n_tokens >= PAIR_MIN_ROWS:
        return "grouped_gemm_pair_kernel (FC1+FC2, tcgen05 cta_group::2, 256x256 tiles)"
    return "grouped_gemm_tc_kernel (FC1+FC2, tcgen05, one CTA per tile)"


def stages_alone(x, wr, reps=20):
    """Each memory-bound stage kernel launched `reps` times back to back
    through its own C-ABI entry point (router: agm_router_topk; permute:
    agm_permute; combine: agm_combine) on preallocated outputs, CUDA events
    around the loop on the launching stream: the kernel's own duration plus
    the gap between two launches. The per-stage pass of the forward puts an
    event between kernels, so each of its stage times also holds a launch
    latency and the kernel's prologue, which the forward itself hides by
    letting each kernel start while the previous one finishes."""
    from agillm41_b200 import _lib, ops

    lib = ops.load()
    dev = x.device
    n, d = x.shape
    st = torch.cuda.current_stream(dev).cuda_stream
    idx, gates, hist, _ = ops.router_topk(x, wr, TOP_K)
    plan = ops.dispatch_plan(hist, n, TOP_K)
    x_perm, row_of = ops.permute(x, idx, plan, EXPERTS)
    out = torch.empty_like(x)
    bf16 = _lib.AGM_BF16
    P = _lib.ptr

    def router():
        return lib.agm_router_topk(P(x), P(wr), bf16, n, d, EXPERTS, TOP_K, 0, None, None, P(idx), P(gates),
                                   P(hist), None, st)

    def permute():
        return lib.agm_permute(P(x), bf16, n, d, EXPERTS, TOP_K, P(idx), P(plan["block_off"]), P(plan["seg_start"]),
                               P(plan["counts"]), P(x_perm), P(row_of), P(plan["token_of"]), None, st)

    def combine():
        return lib.agm_combine(P(x_perm), P(row_of), P(gates), bf16, n, d, TOP_K, None, 0, 0, P(out), st)

    res = {}
    for name, fn in (("router", router), ("permute", permute), ("combine", combine)):
        for _ in range(3):
            assert fn() == 0, name
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        res[name] = e0.elapsed_time(e1) / reps
    return res


def report(args, world, rank, N, ms_total, stage_ms, clocks, value, e2e, x, decode=None, train=None, codec=None,
           parity=None, skewed=None, block_ffn=None, alone=None, expert_stream=None):
    if rank != 0:
        return
    peaks = load_peaks()
    gemm_ms = (stage_ms["fc1"] + stage_ms["fc2"]) / 2.0          # average launch of the grouped GEMM
    gemm_flop_per_launch = FLOP_PER_TOKEN * N / 2.0
    achieved_tf = gemm_flop_per_launch / (gemm_ms / 1000.0) / 1e12
    traffic_rec = load_traffic()
    traffic = traffic_rec.get("grouped_gemm_fc1_fc2_avg_bytes_per_launch")

    alone = alone or {}

    def hbm(stage, per_tok):
        gbs = per_tok * N / (stage_ms[stage] / 1000.0) / 1e9
        rec = {"ms": round(stage_ms[stage], 4), "achieved_gbs": round(gbs, 1), "frac": round(gbs / peaks["hbm"], 3),
               "algorithmic_bytes": per_tok * N}
        if stage in alone:
            g2 = per_tok * N / (alone[stage] / 1000.0) / 1e9
            rec["alone"] = {"ms": round(alone[stage], 4), "achieved_gbs": round(g2, 1),
                            "frac": round(g2 / peaks["hbm"], 3)}
        return rec

    cpu = None
    if world == 1 and not args.skip_cpu:
        rate, threads, reps, dt = cpu_oracle_rate(2048)
        cpu = {"value": rate, "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"2048 tokens of the workload x {reps} forwards ({dt:.1f} s), fp32, "
                         f"torch.set_num_threads({threads}), CPU {cpu_model()}"}
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_total / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) input, N(0,0.02^2) random-init expert weights)",
        "config": workload_config(world, N),
        "e2e": e2e,
        "gpu_launches": KERNELS_PER_STEP * args.steps,
        "roofline": {"kernel": gemm_kernel_name(N), "bound": "tensor",
                     "achieved": round(achieved_tf, 1), "peak": peaks["tf"], "unit": "TFLOP/s",
                     "frac": round(achieved_tf / peaks["tf"], 3),
                     "frac_of_sustained_peak": round(achieved_tf / peaks["tf_sus"], 3),
                     "peak_source": f"{peaks['src']} bf16 burst (the GEMM launches are timed inside a "
                                    f"{ms_total:.0f} ms region, not a seconds-long loop; sustained "
                                    f"{peaks['tf_sus']})",
                     "traffic": traffic,
                     "traffic_source": traffic_rec.get("source", "not measured in this run") if traffic else None,
                     "flop_per_launch": gemm_flop_per_launch},
        "stages": {
            "router": hbm("router", ROUTER_BYTES), "permute": hbm("permute", PERMUTE_BYTES),
            "combine": hbm("combine", COMBINE_BYTES),
            "plan_ms": round(stage_ms["plan"], 4), "fc1_ms": round(stage_ms["fc1"], 4),
            "fc2_ms": round(stage_ms["fc2"], 4), "hbm_peak_gbs": peaks["hbm"],
        },
        "cpu_baseline": cpu,
        "clocks": clocks,
    }
    if parity is not None:
        line["parity"] = parity
    if skewed is not None:
        line["skewed"] = skewed
    if block_ffn is not None:
        line["block_ffn"] = block_ffn
    if decode is not None:
        line["decode"] = decode
    if train is not None:
        line["train"] = train
    if codec is not None:
        line["codec"] = codec
    if expert_stream is not None:
        line["expert_stream"] = expert_stream
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--tokens", type=int, default=BATCH * SEQ,
                    help="tokens per GPU (default: the 48 x 1536 workload; smaller for profiling)")
    ap.add_argument("--skip-e2e", action="store_true", help="skip the host-buffer end-to-end leg")
    ap.add_argument("--skip-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--skip-decode", action="store_true", help="skip the 28-layer decode leg")
    ap.add_argument("--skip-train", action="store_true", help="skip the training-step (forward + backward) leg")
    ap.add_argument("--skip-codec", action="store_true", help="skip the tensor-codec decode leg")
    ap.add_argument("--skip-aux", action="store_true", help="skip the auxiliary router-loss leg")
    ap.add_argument("--skip-parity", action="store_true", help="skip the routing/output parity check")
    ap.add_argument("--skip-skewed", action="store_true", help="skip the skewed-routing legs")
    ap.add_argument("--skip-block", action="store_true", help="skip the Block FFN-half (LayerNorm share) leg")
    ap.add_argument("--skip-expert-stream", action="store_true",
                    help="skip the host-resident-experts (expert streaming) leg")
    ap.add_argument("--skip-ep-variants", action="store_true",
                    help="N > 1: time only the declared expert-parallel placement")
    ap.add_argument("--skip-reference-gpu", action="store_true",
                    help="--impl reference: skip the reference's op sequence timed on the GPU")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, world, rank)
        return
    world, rank, local = dist_setup(args.gpus)
    try:
        if world > 1:
            run_ep(args, world, rank, local)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()

"""Benchmark of the FPA operator: forward and forward+backward at the README shape (B4 H12 T2048 D64 fp16).

    python bench.py [--gpus N --steps K --warmup W] [--impl native|reference] [--scaling strong|weak]

One process per GPU (torchrun for N > 1). A step is one forward+backward pass of the operator through its public
API over one batch. With strong scaling (the default, as configuration 2 asks) the 48 (b, h) heads of the one
configuration-2 batch are split over the ranks (48/24/12/6 heads per GPU at N = 1/2/4/8); with --scaling weak every
rank runs a full configuration-2 batch of its own. The heads are independent, so there is no collective on the data
path; the only collectives are the barriers and the max-over-ranks of the timings.

Prints ONE JSON line (rank 0). `value` is the whole-job fwd+bwd throughput in TFLOP/s (causal FlashAttention FLOP
count 7*B*H*T^2*D) with inputs resident in HBM: the device step replayed from a CUDA graph, median over the timed
steps. Beside it: the reference benchmark's own protocol (eager calls, 3 warm-up, median of 15; reference
bench.py:11-23, 46-48) as `eager_*`; `e2e` through the public API from pinned host buffers with o and all six
gradients copied back, host<->device copies inside the timed region; configuration 4 (B1 H16 T16383 D128) split
the same way; the dominant kernel's roofline; the reference's PyTorch CPU path on the host cores.

`--impl reference` times the reference's CPU implementation of the operator (the dense PyTorch definition behind
impl="reference", fp32 arithmetic for fp16 inputs as kernel.py:23-24 and 57-64 compute it) on the host cores,
over a sample of the configuration's heads per step.
"""
import argparse
import json
import os
import statistics
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "fwd / fwd+bwd ms & TFLOP/s at 4x12x2048x64 fp16 (% tensor peak), 1-8 GPU"
PUBLISHED_FWD_BWD_TFLOPS = 20.6   # README.md:57 of the reference: 4.38 ms fwd+bwd on sm_75 = 90.19 GFLOP / 4.38 ms
FALLBACK_PEAK_TFLOPS = 1590.0
L2_FLUSH_BYTES = 256 << 20
CONFIG4 = (1, 16, 16383, 128)
# DRAM bytes (read + write) per launch of each tensor-core kernel at configuration 2 on one GPU, from an ncu
# capture (dram__bytes_read.sum + dram__bytes_write.sum); reported as roofline.traffic for the dominant kernel.
NCU_TRAFFIC_C2 = {"bwd_kv_tc": (54.38 + 2.17) * 1e6, "bwd_q_tc": (54.85 + 1.57) * 1e6, "fwd_tc": (39.42 + 0.09) * 1e6}


def parse(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["native", "reference"], default="native")
    ap.add_argument("--scaling", choices=["strong", "weak"], default="strong")
    ap.add_argument("--shape", default="4,12,2048,64", help="B,H,T,D in total (strong) or per rank (weak)")
    ap.add_argument("--dtype", choices=["fp16", "fp32"], default="fp16")
    ap.add_argument("--no-cpu-baseline", action="store_true", help="skip the CPU reference sample")
    ap.add_argument("--e2e-pieces", type=int, default=4,
                    help="at least this many pieces in the pipelined end-to-end step (several sequences per GPU)")
    ap.add_argument("--no-config4", action="store_true", help="skip the configuration-4 measurement")
    ap.add_argument("--no-triton-reference", action="store_true",
                    help="skip timing the reference's own Triton kernels (installed under baseline/_ref)")
    ap.add_argument("--workload", choices=["operator", "lm"], default="operator",
                    help="operator: configuration 2 (the BASELINE metric); lm: configuration 5, the LM training step")
    ap.add_argument("--lm-layers", type=int, default=12, help="blocks of the LM (configuration 5: 12)")
    ap.add_argument("--lm-batch", type=int, default=8, help="sequences per GPU (configuration 5: 8)")
    return ap.parse_args(argv)


# Named configurations of the reference's benchmarks (B, H, T, D); the published number applies to 2 only.
NAMED_SHAPES = {(4, 12, 2048, 64): "configuration 2", CONFIG4: "configuration 4"}


def shape_label(B, H, T, D):
    return NAMED_SHAPES.get((B, H, T, D), "custom shape")


def metric_for(B, H, T, D, dtype="fp16"):
    if (B, H, T, D) == (4, 12, 2048, 64) and dtype == "fp16":
        return METRIC
    return f"fwd / fwd+bwd ms & TFLOP/s at {B}x{H}x{T}x{D} {dtype} (% tensor peak), 1-8 GPU"


def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


LM_METRIC = "LM training step tokens/s (GPT-2-small-shaped FPA decoder, T=2048, batch 8/GPU, fp16 autocast)"


def lm_main(args, rank, world, local):
    """Configuration 5: one data-parallel training step of the FPA language model per step (forward, loss,
    backward with the DDP gradient all-reduce over NCCL, AdamW), tokens/s over all ranks."""
    import torch.distributed as dist
    from datetime import timedelta
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    from first_passage_attention_b200 import LaunchStats
    from first_passage_attention_b200.lm import FPALanguageModel, LMConfig, LMTrainer, make_tokens
    cfg = LMConfig(n_layers=args.lm_layers)
    T, Bt = 2048, args.lm_batch
    torch.manual_seed(0)  # the same initial weights on every rank
    model = FPALanguageModel(cfg).to(device)
    trainer = LMTrainer(model)
    host_tok = make_tokens(Bt, T, cfg.vocab, seed=1000 + rank, device="cpu").pin_memory()
    host_loss = torch.empty((), dtype=torch.float32, pin_memory=True)

    def step():
        tok = host_tok.to(device, non_blocking=True)  # the step's inputs from pinned host memory
        loss = trainer.step(tok)
        host_loss.copy_(loss, non_blocking=True)      # and its result back

    def sync_all():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step()
    sync_all()
    LaunchStats.reset()
    sampler = ClockSampler(local)
    evs = []
    with sampler:
        for _ in range(args.steps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            step()
            b.record()
            evs.append((a, b))
        torch.cuda.synchronize()
    ms = statistics.median(a.elapsed_time(b) for a, b in evs)
    launches = LaunchStats.kernels
    if world > 1:
        t = torch.tensor([ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    tokens = Bt * T * world
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        # The same model and step on the host cores with the reference (dense PyTorch) attention, one sequence of
        # T=256 (bounded sample), reported in tokens/s.
        torch.set_num_threads(cpu_threads())
        torch.manual_seed(0)
        cpu_model = FPALanguageModel(cfg, impl="reference")
        cpu_tr = LMTrainer(cpu_model, ddp=False)
        tok = make_tokens(1, 256, cfg.vocab, seed=7, device="cpu")
        cpu_tr.step(tok)
        t0 = time.time()
        cpu_tr.step(tok)
        dt = time.time() - t0
        cpu = {"value": 256 / dt, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
               "sample": f"one sequence of T=256 through the same {cfg.n_layers}-block model with the reference "
                         f"(dense PyTorch) attention, fp32, one training step, {dt:.1f} s"}
    if rank == 0:
        line = {"metric": LM_METRIC, "value": tokens / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f16 (autocast), f32 master weights",
                "data": "synthetic token ids, random-init weights",
                "config": {"workload": f"configuration 5: {cfg.n_layers} blocks, d_model {cfg.d_model}, "
                                       f"{cfg.n_heads} heads, vocab {cfg.vocab}, T {T}, batch {Bt} per GPU",
                           "params": model.n_params(), "parallelism": f"DDP over {world} GPU(s), NCCL all-reduce",
                           "l2": "working set (weights, optimizer state, activations) far above L2"},
                "e2e": {"value": tokens / (ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": host_tok.numel() * 8,
                        "d2h_bytes_per_step": 4},
                "gpu_launches": launches, "clocks": sampler.summary(), "cpu_baseline": cpu,
                "loss": float(host_loss)}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def flops(B, H, T, D, which):
    f = 2.0 * B * H * T * T * D
    return f if which == "fwd" else 3.5 * f


def head_shard(B, H, rank, world):
    """Contiguous block of the flattened (b, h) heads owned by `rank` when B*H heads are split over `world` ranks:
    returns (z0, z1). Heads are independent in the forward and the backward, so the shards need no exchange."""
    n = B * H
    if n % world:
        raise ValueError(f"{n} heads cannot be split evenly over {world} ranks")
    per = n // world
    return rank * per, (rank + 1) * per


def shard_block(H, z0, z1):
    """The flattened heads z0..z1 as a rectangle of (b, h): (b0, b1, h0, h1), or None if they are not one (a range
    of whole batches, or a range of heads inside one batch)."""
    if z0 % H == 0 and z1 % H == 0:
        return z0 // H, z1 // H, 0, H
    if z0 // H == (z1 - 1) // H:
        return z0 // H, z0 // H + 1, z0 % H, (z1 - 1) % H + 1
    return None


def take_heads(x, z0, z1, H):
    """The heads z0..z1 of a [B, H, ...] tensor; beta (H,) gives the entries of those heads. A rectangular block of
    (b, h) keeps its [b1 - b0, h1 - h0, ...] shape (so dbeta sums over its batches, as the operator's does);
    otherwise the heads come as [1, z1 - z0, ...] with beta[z % H]."""
    blk = shard_block(H, z0, z1)
    if x.dim() == 1:
        if blk is not None:
            return x[blk[2]:blk[3]]
        return x[torch.arange(z0, z1, device=x.device) % H]
    if blk is not None:
        b0, b1, h0, h1 = blk
        return x[b0:b1, h0:h1]
    flat = x.reshape(-1, *x.shape[2:])
    return flat[z0:z1].unsqueeze(0)


def load_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            m = json.load(f)
        return float(m["bf16_tflops"]), "measured (MEASURED_PEAKS.json bf16_tflops, burst)"
    except (OSError, KeyError, ValueError):
        return FALLBACK_PEAK_TFLOPS, "fallback"


def make_inputs(B, H, T, D, seed, device, dtype=torch.float16):
    """Configuration 2: q, k, v ~ N(0,1) in fp16; phi = fp32 cumsum of N(0,1) steps; psi = phi + N(0,1);
    beta = ones(H); grad_o = ones."""
    g = torch.Generator(device=device).manual_seed(seed)
    q, k, v = (torch.randn(B, H, T, D, generator=g, device=device).to(dtype) for _ in range(3))
    phi = torch.randn(B, H, T, generator=g, device=device).cumsum(-1)
    psi = phi + torch.randn(B, H, T, generator=g, device=device)
    beta = torch.ones(H, device=device)
    do = torch.ones(B, H, T, D, device=device, dtype=dtype)
    return q, k, v, phi, psi, beta, do


def make_config4_inputs(B, H, T, D, seed, device):
    """Configuration 4: q, k, v ~ N(0, 0.5) in fp16; phi = cumsum of N(0,1) steps; psi = phi + N(0, 2);
    beta = 2 * ones(H); grad_o ~ N(0,1)."""
    g = torch.Generator(device=device).manual_seed(seed)
    q, k, v = ((0.5 * torch.randn(B, H, T, D, generator=g, device=device)).half() for _ in range(3))
    phi = torch.randn(B, H, T, generator=g, device=device).cumsum(-1)
    psi = phi + 2 * torch.randn(B, H, T, generator=g, device=device)
    beta = 2 * torch.ones(H, device=device)
    do = torch.randn(B, H, T, D, generator=g, device=device).half()
    return q, k, v, phi, psi, beta, do


class ClockSampler:
    """Samples SM clock and throttle reasons with NVML in a background thread while the timed region runs."""

    REASONS = {0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x4: "sw_power_cap", 0x1: "gpu_idle"}

    def __init__(self, index, period=0.002):
        self.index, self.period = index, period
        self.samples, self.reasons = [], set()
        self._stop = threading.Event()
        self.max_mhz = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:  # NVML unavailable: report no clocks rather than fail the benchmark
            self._nvml = None

    def sample(self):
        """One reading (also called from the timing loop while queued GPU work runs)."""
        if not self._nvml:
            return
        try:
            self.samples.append(self._nvml.nvmlDeviceGetClockInfo(self._h, self._nvml.NVML_CLOCK_SM))
            r = self._nvml.nvmlDeviceGetCurrentClocksEventReasons(self._h)
            self.reasons.update(n for bit, n in self.REASONS.items() if r & bit)
        except Exception:
            pass

    def _run(self):
        while not self._stop.is_set():
            self.sample()
            time.sleep(self.period)

    def __enter__(self):
        if self._nvml:
            self._stop.clear()
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        if self._nvml:
            self._stop.set()
            self._t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons - {"gpu_idle"}), "samples": len(self.samples)}


def step_times(fn, steps, warmup, flush, during=None):
    """Runs fn warmup times, then `steps` times with an L2 flush (a 256 MiB write, outside the events) before each;
    each step is bracketed by CUDA events on the current stream. `during` is called while the enqueued steps run on
    the GPU (clock sampling). Returns the per-step device times in ms."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    evs = []
    for _ in range(steps):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        evs.append((a, b))
    if during is not None:
        during()
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in evs]


def reference_protocol(fn, flush, warm=3, n=15):
    """The reference benchmark's timing (its bench.py:11-23): `warm` eager calls, then `n` calls each bracketed by
    CUDA events and followed by a synchronize; the median in ms. An L2 flush precedes every timed call."""
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(n):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    return statistics.median(ts)


def capture(fn, device):
    """fn captured in a CUDA graph after two warm-up runs on a side stream; None (and a note on stderr) if capture
    fails, in which case the caller times fn eagerly."""
    try:
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(2):
                fn()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        torch.cuda.synchronize()
        return g
    except Exception as exc:
        print(f"# CUDA graph capture failed ({exc}); timing eagerly", file=sys.stderr, flush=True)
        return None


# ------------------------------------------------------------------------------------- reference CPU path ----
def reference_cpu_inputs(n_heads, T, D, seed=0):
    """n_heads heads drawn as configuration 2 draws them (fp16 q, k, v ~ N(0,1); phi = cumsum N(0,1); psi = phi +
    N(0,1); beta = 1; grad_o = ones), on the host."""
    g = torch.Generator().manual_seed(seed)
    q, k, v = (torch.randn(1, n_heads, T, D, generator=g).half() for _ in range(3))
    phi = torch.randn(1, n_heads, T, generator=g).cumsum(-1)
    psi = phi + torch.randn(1, n_heads, T, generator=g)
    beta = torch.ones(n_heads)
    do = torch.ones(1, n_heads, T, D, dtype=torch.float16)
    return q, k, v, phi, psi, beta, do


_REF_MODULE = []


def reference_module():
    """The unmodified reference module (its kernel.py, installed under baseline/_ref), or None when it is not there
    or does not import. Loaded once."""
    if not _REF_MODULE:
        import importlib.util
        path = os.path.join(ROOT, "baseline", "_ref", "kernel.py")
        mod = None
        if os.path.exists(path):
            try:
                spec = importlib.util.spec_from_file_location("fpa_reference_module", path)
                mod = importlib.util.module_from_spec(spec)
                spec.loader.exec_module(mod)
            except Exception as exc:  # reported by the callers' "kind"
                print(f"# reference module under baseline/_ref does not import: {exc}", file=sys.stderr)
                mod = None
        _REF_MODULE.append(mod)
    return _REF_MODULE[0]


def reference_cpu_kind():
    """"reference" when the CPU leg runs the unmodified reference's own impl="reference" path, else "port" (this
    repository's restatement of the same definition, reference.py)."""
    return "reference" if reference_module() is not None else "port"


def reference_cpu_step(inputs):
    """One forward + backward of the reference's CPU path (the dense PyTorch definition, impl="reference"; fp32
    arithmetic for fp16 inputs) on the host; returns the elapsed seconds. Runs the unmodified reference module when
    it is installed under baseline/_ref, else this repository's restatement of it."""
    mod = reference_module()
    if mod is not None:
        fpa = mod.first_passage_attention
    else:
        from first_passage_attention_b200 import first_passage_attention as fpa
    leaves = [t.clone().requires_grad_() for t in inputs[:6]]
    t0 = time.perf_counter()
    o = fpa(*leaves, impl="reference")
    o.backward(inputs[6])
    return time.perf_counter() - t0


def reference_cpu_heads(T, D, budget_s, max_heads):
    """Number of heads one step of the reference CPU path can take within budget_s seconds, from a timed one-head
    call (after one untimed call); also returns that one-head time."""
    one = reference_cpu_inputs(1, T, D, seed=99)
    reference_cpu_step(one)
    t1 = reference_cpu_step(one)
    return max(1, min(max_heads, int(budget_s / max(t1, 1e-6)))), t1


def reference_arm(args, B, H, T, D, rank, world):
    """The reference's CPU implementation of the operator on the host cores (rank 0 only), on this arm's
    configuration: each step is one forward + backward over a sample of the configuration's heads sized so the
    whole run stays within about three minutes."""
    if rank != 0:
        return
    torch.set_num_threads(cpu_threads())
    steps, warmup = args.steps, args.warmup
    per_step_budget = min(8.0, 150.0 / max(1, steps + warmup))
    heads, _ = reference_cpu_heads(T, D, per_step_budget, B * H)
    inputs = reference_cpu_inputs(heads, T, D, seed=0)
    for _ in range(warmup):
        reference_cpu_step(inputs)
    times = [reference_cpu_step(inputs) for _ in range(steps)]
    sec = statistics.median(times)
    val = flops(1, heads, T, D, "fwd_bwd") / sec / 1e12
    src = ("the unmodified reference kernel.py under baseline/_ref" if reference_cpu_kind() == "reference"
           else "this repository's restatement of it")
    sample = (f"{heads} of the {B * H} heads of B{B} H{H} T{T} D{D} per step (heads are independent; full T), "
              f"forward + backward of the dense PyTorch definition (impl='reference', {src}), fp16 inputs computed "
              f"in fp32, median of {steps} steps")
    line = {"impl": "reference", "metric": metric_for(B, H, T, D), "value": val, "unit": "TFLOP/s",
            "n_gpus": world, "steps": steps, "warmup": warmup, "ms_per_step": 1e3 * sec, "higher_is_better": True,
            "scaling": args.scaling, "vs_baseline": None, "dtype": "f32 (fp16 inputs)", "data": "synthetic",
            "config": {"workload": f"{shape_label(B, H, T, D)} (B{B} H{H} T{T} D{D} fp16) fwd+bwd, sampled heads",
                       "B": B, "H": H, "T": T, "D": D, "heads_per_step": heads, "same_config": True},
            "cpu_baseline": {"value": val, "unit": "TFLOP/s", "cores": torch.get_num_threads(),
                             "kind": reference_cpu_kind(), "sample": sample},
            "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def triton_reference(inputs, flush):
    """The reference's own GPU path (its Triton kernels, impl="triton", from the unmodified reference module installed
    under baseline/_ref) timed with the reference benchmark's protocol (3 warm-up, median of 15, its bench.py:11-23,
    46-52) on the same inputs, when that module imports here; otherwise the reason it is unavailable."""
    mod = reference_module()
    if mod is None:
        return {"unavailable": "the reference module is not installed (or does not import) under baseline/_ref"}
    try:
        q, k, v, phi, psi, beta, do = inputs
        args = (q, k, v, phi, psi, beta)

        def fwd():
            with torch.no_grad():
                mod.first_passage_attention(*args, impl="triton")

        def fwd_bwd():
            x = [t.clone().requires_grad_() for t in args]
            mod.first_passage_attention(*x, impl="triton").backward(do)
        f_ms = reference_protocol(fwd, flush)
        fb_ms = reference_protocol(fwd_bwd, flush)
    except Exception as exc:  # a reference that cannot run here is reported, not fatal
        return {"unavailable": f"{type(exc).__name__}: {str(exc).splitlines()[0][:200] if str(exc) else ''}"}
    B, H, T, D = inputs[0].shape
    return {"fwd_ms": f_ms, "fwd_bwd_ms": fb_ms, "fwd_tflops": flops(B, H, T, D, "fwd") / (f_ms * 1e-3) / 1e12,
            "fwd_bwd_tflops": flops(B, H, T, D, "fwd_bwd") / (fb_ms * 1e-3) / 1e12,
            "protocol": "reference bench.py: eager impl='triton', 3 warm-up, median of 15, L2 flushed before each",
            "source": "unmodified reference kernel.py installed under baseline/_ref"}


# ------------------------------------------------------------------------------------------------ native ----
def e2e_chunks(Bs, Hs, want=4):
    """Pieces of a [Bs, Hs] shard the end-to-end step pipelines. Several sequences: each sequence, cut into equal
    groups of heads until there are at least `want` pieces; one sequence: up to four groups of heads (a piece of one
    or two heads is latency-bound on the GPU). At configuration 2, 4 and 8 pieces measured the same within the
    run-to-run spread of the host copies (1.57-1.76 ms per step on one B200). Returns [(b, h0, h1)]."""
    if Bs > 1:
        g = next((c for c in range(1, Hs + 1) if Hs % c == 0 and Bs * c >= want), Hs)
        per = Hs // g
        return [(b, c * per, (c + 1) * per) for b in range(Bs) for c in range(g)]
    n = max(c for c in range(1, 5) if Hs % c == 0)
    per = Hs // n
    return [(0, c * per, (c + 1) * per) for c in range(n)]


def main(argv=None):
    args = parse(argv)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    B, H, T, D = (int(x) for x in args.shape.split(","))
    dtype = torch.float16 if args.dtype == "fp16" else torch.float32
    if args.workload == "lm":
        lm_main(args, rank, world, local)
        return
    if args.impl == "reference":
        reference_arm(args, B, H, T, D, rank, world)
        return

    import torch.distributed as dist
    from datetime import timedelta
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)

    from first_passage_attention_b200 import LaunchStats, first_passage_attention

    def sync_all():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(ms):
        if world == 1:
            return ms
        t = torch.tensor([ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    def shard(shape, maker, seed):
        """This rank's inputs: strong scaling keeps its block of the heads of the one batch every rank draws;
        weak scaling draws a full batch of its own."""
        b_, h_, t_, d_ = shape
        if args.scaling == "strong":
            z0, z1 = head_shard(b_, h_, rank, world)
            full = maker(b_, h_, t_, d_, seed, device)
            out = [take_heads(x, z0, z1, h_).contiguous() for x in full]
            del full
            return out
        return list(maker(b_, h_, t_, d_, seed + rank, device))

    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    q, k, v, phi, psi, beta, do = shard((B, H, T, D), lambda *a: make_inputs(*a, dtype=dtype), 1000)
    Bs, Hs = q.shape[:2]

    def fwd():
        with torch.no_grad():
            first_passage_attention(q, k, v, phi, psi, beta, impl="cuda")

    leaves = [t.detach().clone().requires_grad_() for t in (q, k, v, phi, psi, beta)]

    def fwd_bwd():
        for x in leaves:
            x.grad = None
        first_passage_attention(*leaves, impl="cuda").backward(do)

    def fwd_bwd_reference_style():
        """The reference benchmark's fwd+bwd (its bench.py:50-52): fresh leaves by clone, forward, backward."""
        x = [t.clone().requires_grad_() for t in (q, k, v, phi, psi, beta)]
        first_passage_attention(*x, impl="cuda").backward(do)

    # 1. Device step, inputs resident in HBM: the forward + backward captured once in a CUDA graph and replayed.
    sync_all()
    fwd_graph = capture(fwd, device)
    fwd_ms = max_over_ranks(statistics.median(step_times(fwd_graph.replay if fwd_graph else fwd, args.steps,
                                                         args.warmup, flush)))
    sync_all()
    for _ in range(args.warmup):
        fwd_bwd()
    sync_all()
    LaunchStats.reset()
    graph = capture(fwd_bwd, device)
    launches_per_step = LaunchStats.kernels // 3 if graph is not None else None  # two warm-up runs + the capture
    step_fn = graph.replay if graph is not None else fwd_bwd
    sampler = ClockSampler(local)

    def clock_samples():  # the GPU is busy with the queued steps while these run
        for _ in range(4):
            sampler.sample()
            time.sleep(0.001)

    sync_all()
    LaunchStats.reset()
    with sampler:
        step_ms = max_over_ranks(statistics.median(step_times(step_fn, args.steps, args.warmup, flush,
                                                              during=clock_samples)))
    launches = LaunchStats.kernels if graph is None else launches_per_step * args.steps
    sync_all()

    # 2. The reference benchmark's protocol: eager calls, median of 15 after 3 warm-up.
    eager_fwd_ms = max_over_ranks(reference_protocol(fwd, flush))
    eager_step_ms = max_over_ranks(reference_protocol(fwd_bwd_reference_style, flush))
    sync_all()

    # 3. Weak-scaling companion at N > 1: every rank runs the full configuration batch at once.
    weak = None
    if world > 1 and args.scaling == "strong":
        wq = make_inputs(B, H, T, D, 2000 + rank, device, dtype=dtype)
        wl = [t.clone().requires_grad_() for t in wq[:6]]

        def weak_step():
            for x in wl:
                x.grad = None
            first_passage_attention(*wl, impl="cuda").backward(wq[6])
        wg = capture(weak_step, device)
        wms = max_over_ranks(statistics.median(step_times(wg.replay if wg else weak_step, args.steps, args.warmup,
                                                          flush)))
        weak = {"ms_per_step": wms, "value": world * flops(B, H, T, D, "fwd_bwd") / (wms * 1e-3) / 1e12,
                "unit": "TFLOP/s", "heads_per_gpu": B * H}
        del wg, wl, wq
        sync_all()

    # 4. End to end through the public API: each step copies its inputs in from pinned host memory and o and all
    # six gradients back out. The host keeps each piece's inputs packed in one pinned block [q | k | v | do | phi |
    # psi | beta]; the step is pipelined over the pieces (each sequence, or groups of heads of one sequence) on a
    # copy-in stream, two compute streams and a copy-out stream, so the copies of one piece overlap the compute of
    # the others (PCIe is full duplex). Captured in a CUDA graph like the device step (the pipelined step is
    # host-bound when enqueued eagerly).
    chunks = e2e_chunks(Bs, Hs, args.e2e_pieces)
    esz = q.element_size()
    host_pack, layouts = [], []
    for (bi, h0, h1) in chunks:
        nh = h1 - h0
        parts = [(q, esz), (k, esz), (v, esz), (do, esz), (phi, 4), (psi, 4)]
        nbytes = [nh * T * D * esz] * 4 + [nh * T * 4] * 2 + [nh * 4]
        buf = torch.empty(sum(nbytes), dtype=torch.uint8, pin_memory=True)
        off = 0
        for (t_, _), nb in zip(parts, nbytes[:6]):
            buf[off:off + nb].copy_(t_[bi, h0:h1].detach().contiguous().cpu().view(torch.uint8).reshape(-1))
            off += nb
        buf[off:off + nh * 4].copy_(beta[h0:h1].detach().float().cpu().view(torch.uint8))
        host_pack.append(buf)
        layouts.append((nh, nbytes))
    host_out = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in (q, q, q, q, phi, psi)]
    host_dbeta = torch.empty(Hs, dtype=torch.float32, pin_memory=True)
    h2d = sum(b.numel() for b in host_pack)
    d2h = sum(t.numel() * t.element_size() for t in host_out) + host_dbeta.numel() * 4
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    s_comp = [torch.cuda.Stream(device), torch.cuda.Stream(device)]
    dt_big = q.dtype

    def unpack(buf, nh, nbytes):
        views, off = [], 0
        shapes = [(1, nh, T, D)] * 4 + [(1, nh, T)] * 2 + [(nh,)]
        dts = [dt_big] * 4 + [torch.float32] * 3
        for nb, shp, dt_ in zip(nbytes, shapes, dts):
            views.append(buf[off:off + nb].view(dt_).view(shp))
            off += nb
        qd, kd, vd, dod, phid, psid, betad = views
        return [qd, kd, vd, phid, psid, betad], dod

    def e2e():
        main_s = torch.cuda.current_stream()
        for st_ in [s_in, s_out] + s_comp:
            st_.wait_stream(main_s)
        dbetas = []
        for ci, ((bi, h0, h1), buf_h, (nh, nbytes)) in enumerate(zip(chunks, host_pack, layouts)):
            cs = s_comp[ci % 2]
            with torch.cuda.stream(s_in):
                buf = buf_h.to(device, non_blocking=True)
                ev_in = torch.cuda.Event()
                ev_in.record()
            cs.wait_event(ev_in)
            with torch.cuda.stream(cs):
                buf.record_stream(cs)
                xs, dod = unpack(buf, nh, nbytes)
                xs = [t.requires_grad_() for t in xs]
                o = first_passage_attention(*xs, impl="cuda")
                o.backward(dod)
                outs = [o.detach()] + [x.grad for x in xs[:5]]
                dbetas.append((h0, h1, xs[5].grad))
                ev_c = torch.cuda.Event()
                ev_c.record(cs)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_c)
                for hst, d in zip(host_out, outs):
                    d.record_stream(s_out)
                    hst[bi:bi + 1, h0:h1].copy_(d, non_blocking=True)
        for cs in s_comp:
            main_s.wait_stream(cs)
        # dbeta of the shard: each group of heads summed over the sequences, in piece order.
        dbeta_dev = torch.zeros(Hs, dtype=torch.float32, device=device)
        for h0, h1, g_ in dbetas:
            dbeta_dev[h0:h1] += g_
        ev_b = torch.cuda.Event()
        ev_b.record(main_s)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_b)
            dbeta_dev.record_stream(s_out)
            host_dbeta.copy_(dbeta_dev, non_blocking=True)
        main_s.wait_stream(s_out)

    sync_all()
    e2e_graph = capture(e2e, device)
    e2e_ms = max_over_ranks(statistics.median(step_times(e2e_graph.replay if e2e_graph else e2e, args.steps,
                                                         args.warmup, flush)))
    e2e_graphed = e2e_graph is not None
    del e2e_graph
    # The pipelined pieces compute what the device step does: their gradients read back to the host against the
    # device step's (fp16 rounding of a different key-range split and summation order at most).
    torch.cuda.synchronize(device)

    def rel_diff(host_t, dev_t):
        ref = dev_t.detach().float().cpu()
        return float((host_t.float() - ref).abs().max() / ref.abs().max().clamp_min(1e-30))
    e2e_check = max(rel_diff(h_, l_.grad) for h_, l_ in zip(host_out[1:] + [host_dbeta], leaves))
    sync_all()

    # 5. Configuration 4 (B1 H16 T16383 D128 fp16), its heads split the same way.
    cfg4 = None
    if not args.no_config4 and (B, H, T, D) == (4, 12, 2048, 64) and dtype == torch.float16 and 16 % world == 0:
        c4 = shard(CONFIG4, make_config4_inputs, 4000)
        c4l = [t.clone().requires_grad_() for t in c4[:6]]

        def c4_fwd():
            with torch.no_grad():
                first_passage_attention(*c4[:6], impl="cuda")

        def c4_step():
            for x in c4l:
                x.grad = None
            first_passage_attention(*c4l, impl="cuda").backward(c4[6])
        n4 = max(3, min(args.steps, 10))
        g4f = capture(c4_fwd, device)
        f4 = max_over_ranks(statistics.median(step_times(g4f.replay if g4f else c4_fwd, n4, args.warmup, flush)))
        g4 = capture(c4_step, device)
        s4 = max_over_ranks(statistics.median(step_times(g4.replay if g4 else c4_step, n4, args.warmup, flush)))
        Bc, Hc, Tc, Dc = CONFIG4
        peak4, _ = load_peak()
        cfg4 = {"workload": f"configuration 4: B{Bc} H{Hc} T{Tc} D{Dc} fp16, {Hc // world} heads per GPU",
                "fwd_ms": f4, "fwd_tflops": flops(Bc, Hc, Tc, Dc, "fwd") / (f4 * 1e-3) / 1e12,
                "fwd_bwd_ms": s4, "fwd_bwd_tflops": flops(Bc, Hc, Tc, Dc, "fwd_bwd") / (s4 * 1e-3) / 1e12,
                "fwd_bwd_pct_peak_per_gpu": 100 * flops(Bc, Hc, Tc, Dc, "fwd_bwd") / world / (s4 * 1e-3) / 1e12
                / peak4, "steps": n4}
        del g4f, g4, c4, c4l
        sync_all()

    # 6. The reference's own Triton kernels on this GPU, same inputs and protocol (one GPU only).
    triton_ref = None
    if world == 1 and not args.no_triton_reference:
        triton_ref = triton_reference((q, k, v, phi, psi, beta, do), flush)
        torch.cuda.synchronize()

    # 7. Per-kernel device times of the library's launches (CUDA events around each launch, on the call's stream),
    # in a separate pass so the event records stay out of the timed regions above.
    from first_passage_attention_b200 import _lib
    lib = _lib.load()
    _lib.profile_report()
    lib.fpa_profile(1)
    for _ in range(args.steps):
        flush.zero_()
        fwd_bwd()
    torch.cuda.synchronize()
    lib.fpa_profile(0)
    kernels = _lib.profile_report()

    K = args.steps
    f_fwd, f_step = flops(Bs, Hs, T, D, "fwd"), flops(Bs, Hs, T, D, "fwd_bwd")
    peak, peak_src = load_peak()
    job_step = f_step * world / (step_ms * 1e-3) / 1e12
    job_fwd = f_fwd * world / (fwd_ms * 1e-3) / 1e12
    per_gpu_fwd = f_fwd / (fwd_ms * 1e-3) / 1e12
    per_gpu_step = f_step / (step_ms * 1e-3) / 1e12

    # Algorithmic FLOPs per launch (causal FlashAttention convention, unit G = B*H*T^2*D): the forward kernel does
    # the forward's 2G; the kv-pass does 4 of the backward's 5 G-sized products (S^T, dP^T, dV, dK); the q-pass does
    # dQ (its S and dP are the recomputation the convention does not count); the FFMA backward for D <= 128 runs
    # both passes in one launch (5G).
    G = float(Bs) * Hs * T * T * D
    algo = {"fwd_tc": 2 * G, "fwd_simt": 2 * G, "bwd_kv_tc": 4 * G, "bwd_kv_simt": 4 * G, "bwd_q_tc": G,
            "bwd_q_simt": G, "bwd_simt": 5 * G}
    per_launch_us = {k_: 1e3 * ms / n for k_, (n, ms) in kernels.items()}
    dom = max(kernels, key=lambda k_: kernels[k_][1]) if kernels else None
    if dom in algo:
        ach = algo[dom] / (per_launch_us[dom] * 1e-6) / 1e12
        roof = {"bound": "tensor", "kernel": dom, "achieved": ach, "peak": peak, "unit": "TFLOP/s",
                "frac": ach / peak, "peak_source": peak_src,
                "traffic": NCU_TRAFFIC_C2.get(dom) if (Bs * Hs, T, D) == (48, 2048, 64) else None,
                "traffic_unit": "bytes per launch (ncu dram__bytes_read.sum + dram__bytes_write.sum)",
                "share_of_step": kernels[dom][1] / max(1e-9, sum(ms for (n, ms) in kernels.values()))}
    else:
        roof = {"bound": "tensor", "kernel": "forward pass (field statistics + attention forward)",
                "achieved": per_gpu_fwd, "peak": peak, "unit": "TFLOP/s", "frac": per_gpu_fwd / peak,
                "peak_source": peak_src, "traffic": None}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        torch.set_num_threads(cpu_threads())
        heads, _ = reference_cpu_heads(T, D, 15.0, B * H)
        sec = reference_cpu_step(reference_cpu_inputs(heads, T, D, seed=0))
        src = ("the unmodified reference kernel.py under baseline/_ref" if reference_cpu_kind() == "reference"
               else "this repository's restatement of it")
        cpu = {"value": flops(1, heads, T, D, "fwd_bwd") / sec / 1e12, "unit": "TFLOP/s",
               "cores": torch.get_num_threads(), "kind": reference_cpu_kind(),
               "sample": f"{heads} of the {B * H} heads at T={T} D={D} in one call, forward + backward of the dense "
                         f"PyTorch definition (impl='reference', {src}), fp16 inputs computed in fp32, {sec:.1f} s"}

    if rank == 0:
        wl_ = f"B{Bs} H{Hs}" if args.scaling == "strong" else f"B{B} H{H}"
        line = {
            "metric": metric_for(B, H, T, D, args.dtype), "value": job_step, "unit": "TFLOP/s", "n_gpus": world,
            "steps": K, "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True,
            "scaling": args.scaling,
            "vs_baseline": (job_step / PUBLISHED_FWD_BWD_TFLOPS
                            if shape_label(B, H, T, D) == "configuration 2" and args.dtype == "fp16" else None),
            "dtype": "f16" if args.dtype == "fp16" else "f32", "data": "synthetic",
            "config": {"workload": f"{shape_label(B, H, T, D)}: B{B} H{H} T{T} D{D} {args.dtype} fwd+bwd, "
                                   f"{wl_} per GPU ({args.scaling} scaling)",
                       "global_heads": B * H * (world if args.scaling == "weak" else 1), "heads_per_gpu": Bs * Hs,
                       "T": T, "D": D, "accumulate": "f32", "same_config": True,
                       "parallelism": f"heads split over {world} GPU(s), no collective",
                       "timing": "device step replayed from a CUDA graph; median of the timed steps; max over ranks",
                       "l2": "flushed before every timed step (256 MiB write, outside the events)"},
            "fwd_ms": fwd_ms, "fwd_tflops": job_fwd, "fwd_pct_peak": 100 * per_gpu_fwd / peak,
            "fwd_bwd_ms": step_ms, "fwd_bwd_tflops": job_step, "fwd_bwd_pct_peak": 100 * per_gpu_step / peak,
            "eager_fwd_ms": eager_fwd_ms, "eager_ms": eager_step_ms,
            "eager_fwd_bwd_tflops": f_step * world / (eager_step_ms * 1e-3) / 1e12,
            "eager_protocol": "reference bench.py:11-23: eager calls (clone + forward + backward for fwd+bwd), "
                              "3 warm-up, median of 15, L2 flushed before each",
            "roofline": roof,
            "kernels_us_per_launch": {k_: round(v_, 2) for k_, v_ in sorted(per_launch_us.items())},
            "e2e": {"value": f_step * world / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "graph": e2e_graphed,
                    "result_read_back": "o and all six gradients (dq, dk, dv, dphi, dpsi, dbeta) into pinned host "
                                        "buffers",
                    "pipeline": f"{len(chunks)} pieces, one packed pinned block each; copy-in / 2 compute / copy-out "
                                "streams",
                    "grads_rel_diff_vs_device_step": e2e_check},
            "weak_scaling": weak,
            "config4": cfg4,
            "triton_reference": triton_ref,
            "gpu_launches": launches,
            "step_graph": graph is not None,
            "clocks": sampler.summary(),
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    del graph, fwd_graph
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

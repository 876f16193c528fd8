"""Benchmark of the FPA operator: forward and forward+backward at the README shape (B4 H12 T2048 D64 fp16).

    python bench.py [--gpus N --steps K --warmup W] [--impl native|reference] [--scaling weak|strong]

One process per GPU (torchrun for N > 1). A step is one forward+backward pass of the operator through its public
API over one batch: with weak scaling (default) every rank runs the full configuration-2 batch (B4 H12 T2048 D64,
its own shard of a global batch of 4N sequences); with --scaling strong the 48 heads of one batch are split across
the ranks. The heads are independent, so there is no collective on the data path; the only collectives are the
barrier and the max-over-ranks of the timings.

Prints ONE JSON line (rank 0). `value` is the whole-job fwd+bwd throughput in TFLOP/s (causal FlashAttention
FLOP count 7*B*H*T^2*D) with inputs resident in HBM; `e2e` is the same through the public API from pinned host
buffers with the host<->device copies in the timed region. `--impl reference` times the CPU restatement of the
reference's path (the oracle) on the host cores instead.
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
# DRAM bytes (read + write) per launch at configuration 2 per GPU from one ncu capture of this build
# (profiles/tc_kernels_config2_full.md); reported as roofline.traffic for the dominant kernel.
NCU_TRAFFIC_C2 = {"bwd_kv_tc": (54.38 + 3.12) * 1e6, "bwd_q_tc": (54.85 + 1.50) * 1e6, "fwd_tc": (39.42 + 0.03) * 1e6}


def parse():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["native", "reference"], default="native")
    ap.add_argument("--scaling", choices=["weak", "strong"], default="weak")
    ap.add_argument("--shape", default="4,12,2048,64", help="B,H,T,D per rank (weak) or in total (strong)")
    ap.add_argument("--no-cpu-baseline", action="store_true", help="skip the CPU oracle sample")
    ap.add_argument("--workload", choices=["operator", "lm"], default="operator",
                    help="operator: configuration 2 (the BASELINE metric); lm: configuration 5, the LM training step")
    ap.add_argument("--lm-layers", type=int, default=12, help="blocks of the LM (configuration 5: 12)")
    ap.add_argument("--lm-batch", type=int, default=8, help="sequences per GPU (configuration 5: 8)")
    return ap.parse_args()


# Named configurations of the reference's benchmarks, per GPU (B, H, T, D); the published number applies to 2 only.
NAMED_SHAPES = {(4, 12, 2048, 64): "configuration 2", (1, 16, 16383, 128): "configuration 4"}


def shape_label(B, H, T, D):
    return NAMED_SHAPES.get((B, H, T, D), "custom shape")


def metric_for(B, H, T, D):
    if (B, H, T, D) == (4, 12, 2048, 64):
        return METRIC
    return f"fwd / fwd+bwd ms & TFLOP/s at {B}x{H}x{T}x{D} fp16 (% tensor peak), 1-8 GPU"


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
    ms = sum(a.elapsed_time(b) for a, b in evs) / args.steps
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
        torch.set_num_threads(os.cpu_count())
        torch.manual_seed(0)
        cpu_model = FPALanguageModel(cfg, impl="reference")
        cpu_tr = LMTrainer(cpu_model, ddp=False)
        tok = make_tokens(1, 256, cfg.vocab, seed=7, device="cpu")
        cpu_tr.step(tok)
        t0 = time.time()
        cpu_tr.step(tok)
        dt = time.time() - t0
        cpu = {"value": 256 / dt, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
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


def take_heads(x, z0, z1, H):
    """The heads z0..z1 of a [B, H, ...] tensor as a [1, z1 - z0, ...] tensor; beta (H,) maps to beta[z % H]."""
    if x.dim() == 1:
        return x[torch.arange(z0, z1, device=x.device) % H]
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


def make_inputs(B, H, T, D, seed, device):
    """Configuration 2: q, k, v ~ N(0,1) in fp16; phi = fp32 cumsum of N(0,1) steps; psi = phi + N(0,1);
    beta = ones(H); grad_o = ones."""
    g = torch.Generator(device=device).manual_seed(seed)
    q, k, v = (torch.randn(B, H, T, D, generator=g, device=device).half() for _ in range(3))
    phi = torch.randn(B, H, T, generator=g, device=device).cumsum(-1)
    psi = phi + torch.randn(B, H, T, generator=g, device=device)
    beta = torch.ones(H, device=device)
    do = torch.ones(B, H, T, D, device=device, dtype=torch.float16)
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


def timed(fn, steps, warmup, flush, during=None):
    """Runs fn warmup times, then `steps` times with an L2 flush (a 256 MiB write) before each; each step is
    bracketed by CUDA events on the current stream. `during` is called while the enqueued steps run on the GPU
    (clock sampling). Returns the summed device time in ms."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    total = 0.0
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
    for a, b in evs:
        total += a.elapsed_time(b)
    return total


def cpu_oracle_sample(D, T, seconds_budget=30.0, heads=1):
    """Times the CPU oracle (float64 NumPy restatement of the reference path) on `heads` heads of the workload."""
    import numpy as np
    from oracle import fpa_oracle as O
    try:
        import threadpoolctl
        cores = max(i.get("num_threads", 1) for i in threadpoolctl.threadpool_info()) or 1
    except Exception:
        cores = os.cpu_count() or 1
    rng = np.random.default_rng(0)
    q, k, v = (rng.standard_normal((1, heads, T, D)).astype(np.float16).astype(np.float64) for _ in range(3))
    phi = rng.standard_normal((1, heads, T)).cumsum(-1)
    psi = phi + rng.standard_normal((1, heads, T))
    beta = np.ones(heads)
    do = np.ones((1, heads, T, D))
    t0 = time.perf_counter()
    O.forward(q, k, v, phi, psi, beta)
    O.backward(q, k, v, phi, psi, beta, do)
    dt = time.perf_counter() - t0
    return dt, cores


def reference_arm(args, B, H, T, D, rank, world):
    if rank != 0:
        return
    steps, warmup = args.steps, args.warmup
    # Each step is one head of the configuration at a prefix length chosen so the whole run stays near 3 minutes.
    per_step_budget = 180.0 / max(1, steps + warmup)
    Ts = T
    est = 3.2 * (T / 2048.0) ** 2          # seconds per head at length T on an 8-core host (measured: ~3 s at 2048)
    while est > per_step_budget and Ts > 256:
        Ts //= 2
        est = 3.2 * (Ts / 2048.0) ** 2
    for _ in range(warmup):
        cpu_oracle_sample(D, Ts)
    times = []
    cores = 1
    for _ in range(steps):
        dt, cores = cpu_oracle_sample(D, Ts)
        times.append(dt)
    ms = 1e3 * sum(times) / len(times)
    val = flops(1, 1, Ts, D, "fwd_bwd") / (ms * 1e-3) / 1e12
    sample = f"one (b,h) head of B{B} H{H} T{T} D{D}, prefix T={Ts}, fwd+bwd, float64 NumPy oracle"
    line = {"impl": "reference", "metric": metric_for(B, H, T, D), "value": val, "unit": "TFLOP/s", "n_gpus": world,
            "steps": steps, "warmup": warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": args.scaling,
            "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": {"workload": f"{shape_label(B, H, T, D)} (B{B} H{H} T{T} D{D} fp16) fwd+bwd, sampled",
                       "B": B, "H": H,
                       "T": T, "D": D},
            "cpu_baseline": {"value": val, "unit": "TFLOP/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    B, H, T, D = (int(x) for x in args.shape.split(","))
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

    # Shard of this rank: weak scaling runs a full per-GPU batch of its own; strong splits the B*H heads of one
    # batch across the ranks (every rank draws the same batch and keeps its heads).
    if args.scaling == "strong":
        z0, z1 = head_shard(B, H, rank, world)
        full = make_inputs(B, H, T, D, seed=1000, device=device)
        q, k, v, phi, psi, beta, do = (take_heads(t, z0, z1, H).contiguous() for t in full)
        del full
        Br, Hr = 1, z1 - z0
    else:
        Br, Hr = B, H
        q, k, v, phi, psi, beta, do = make_inputs(Br, Hr, T, D, seed=1000 + rank, device=device)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)

    def fwd():
        with torch.no_grad():
            first_passage_attention(q, k, v, phi, psi, beta, impl="cuda")

    leaves = [t.detach().clone().requires_grad_() for t in (q, k, v, phi, psi, beta)]

    def fwd_bwd():
        for x in leaves:
            x.grad = None
        first_passage_attention(*leaves, impl="cuda").backward(do)

    # End-to-end: pinned host inputs copied in and the step's result copied out every step, through the public API.
    # The host keeps each sequence's inputs packed in one pinned block [q | k | v | do | phi | psi] (one copy per
    # sequence: six separate copies ran 7 % slower). The step is pipelined over the batch: sequence b's host->device
    # copy, its forward + backward and its device->host copy run on separate streams, so the copies of one sequence
    # overlap the compute of the others (PCIe is full duplex). dbeta sums the per-sequence parts on the device.
    half_b = Hr * T * D * 2
    f_b = Hr * T * 4
    seq_b = 4 * half_b + 2 * f_b
    host_pack = torch.empty(Br, seq_b, dtype=torch.uint8, pin_memory=True)
    for bi in range(Br):
        off = 0
        for t_, nb in ((q, half_b), (k, half_b), (v, half_b), (do, half_b), (phi, f_b), (psi, f_b)):
            host_pack[bi, off:off + nb].copy_(t_[bi].detach().contiguous().cpu().view(torch.uint8).reshape(-1))
            off += nb
    host_beta = beta.detach().cpu().pin_memory()
    host_out = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in (q, q, q, q, phi, psi, beta)]
    h2d = host_pack.numel() + host_beta.numel() * host_beta.element_size()
    d2h = sum(t.numel() * t.element_size() for t in host_out)
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    # Two compute streams take the sequences in turn, so one sequence's kernels (a quarter of the batch fills the
    # GPU poorly) overlap the next one's.
    s_comp = [torch.cuda.Stream(device), torch.cuda.Stream(device)]

    host_loss = torch.empty(Br, dtype=torch.float32, pin_memory=True)

    def unpack(buf):
        """Views of one sequence's packed device block, in argument order: q, k, v, phi, psi, do."""
        views, off = [], 0
        for dt, nb, shape in ((torch.float16, half_b, (1, Hr, T, D)),) * 4 + ((torch.float32, f_b, (1, Hr, T)),) * 2:
            views.append(buf[off:off + nb].view(dt).view(shape))
            off += nb
        qd, kd, vd, dod, phid, psid = views
        return [qd, kd, vd, phid, psid, dod]

    def e2e(copy_all=False):
        """copy_all=False: the step's result read back is its loss, sum(o * do) per sequence (the configuration's
        grad_o = ones is the gradient of sum(o)); the gradients stay on the device as in a training step.
        copy_all=True: o and all six gradients are copied back as well."""
        main = torch.cuda.current_stream()
        for st_ in [s_in, s_out] + s_comp:
            st_.wait_stream(main)
        with torch.cuda.stream(s_in):
            beta_d = host_beta.to(device, non_blocking=True)
        dbetas = []
        for bi in range(Br):
            cs = s_comp[bi % 2]
            with torch.cuda.stream(s_in):
                buf = host_pack[bi].to(device, non_blocking=True)
                ev_in = torch.cuda.Event()
                ev_in.record()
            cs.wait_event(ev_in)
            with torch.cuda.stream(cs):
                buf.record_stream(cs)
                beta_d.record_stream(cs)
                dev = unpack(buf)
                xs = [t.requires_grad_() for t in dev[:5]] + [beta_d.detach().requires_grad_()]
                o = first_passage_attention(*xs, impl="cuda")
                o.backward(dev[5])
                dbetas.append(xs[5].grad)
                loss = (o.detach().float() * dev[5].float()).sum()
                outs = [o.detach()] + [x.grad for x in xs[:5]]
                ev_c = torch.cuda.Event()
                ev_c.record(cs)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_c)
                loss.record_stream(s_out)
                host_loss[bi:bi + 1].copy_(loss.reshape(1), non_blocking=True)
                if copy_all:
                    for hst, d in zip(host_out[:6], outs):
                        d.record_stream(s_out)
                        hst[bi:bi + 1].copy_(d, non_blocking=True)
        for cs in s_comp:
            main.wait_stream(cs)
        dbeta_dev = dbetas[0]
        for g_ in dbetas[1:]:
            dbeta_dev = dbeta_dev + g_
        if copy_all:
            ev_b = torch.cuda.Event()
            ev_b.record(main)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_b)
                dbeta_dev.record_stream(s_out)
                host_out[6].copy_(dbeta_dev, non_blocking=True)
        main.wait_stream(s_out)

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

    sync_all()
    fwd_total = max_over_ranks(timed(fwd, args.steps, args.warmup, flush))
    sync_all()
    LaunchStats.reset()
    sampler = ClockSampler(local)
    for _ in range(args.warmup):
        fwd_bwd()
    sync_all()
    # The device-side step is replayed from a CUDA graph (the library's launches captured once), so the host-side
    # cost of the Python autograd call does not leave the GPU idle between kernels; eager timing if capture fails.
    graph, launches_per_step = None, None
    try:
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(2):
                fwd_bwd()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        LaunchStats.reset()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fwd_bwd()
        launches_per_step = LaunchStats.kernels
        torch.cuda.synchronize()
    except Exception as exc:  # keep the benchmark alive with eager timing
        print(f"# CUDA graph capture failed ({exc}); timing eagerly", file=sys.stderr, flush=True)
        graph = None
    step_fn = graph.replay if graph is not None else fwd_bwd
    for _ in range(args.warmup):
        step_fn()
    sync_all()
    LaunchStats.reset()
    def clock_samples():  # the GPU is busy with the queued steps (about 10 ms) while these run
        for _ in range(4):
            sampler.sample()
            time.sleep(0.001)

    with sampler:
        step_total = max_over_ranks(timed(step_fn, args.steps, 0, flush, during=clock_samples))
    launches = LaunchStats.kernels if graph is None else launches_per_step * args.steps
    sync_all()
    # The pipelined end-to-end step is host-bound when enqueued eagerly (four API calls per step), so it is also
    # replayed from a CUDA graph that holds the copies from and to the pinned host buffers, the library's kernels
    # and the stream fork / join; eager if capture fails.
    def capture(fn):
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
            print(f"# CUDA graph capture of the end-to-end step failed ({exc}); timing eagerly", file=sys.stderr,
                  flush=True)
            return None

    e2e_graph = capture(e2e)
    e2e_total = max_over_ranks(timed(e2e_graph.replay if e2e_graph is not None else e2e, args.steps, args.warmup,
                                     flush))
    sync_all()
    e2e_all = lambda: e2e(copy_all=True)  # noqa: E731
    e2e_all_graph = capture(e2e_all)
    e2e_all_total = max_over_ranks(timed(e2e_all_graph.replay if e2e_all_graph is not None else e2e_all, args.steps,
                                         args.warmup, flush))
    sync_all()
    # Per-kernel device times of the library's launches (CUDA events around each launch, on the call's stream),
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
    fwd_ms, step_ms, e2e_ms, e2e_all_ms = fwd_total / K, step_total / K, e2e_total / K, e2e_all_total / K
    f_fwd, f_step = flops(Br, Hr, T, D, "fwd"), flops(Br, Hr, T, D, "fwd_bwd")
    peak, peak_src = load_peak()
    job_step = f_step * world / (step_ms * 1e-3) / 1e12
    job_fwd = f_fwd * world / (fwd_ms * 1e-3) / 1e12
    per_gpu_fwd = f_fwd / (fwd_ms * 1e-3) / 1e12
    per_gpu_step = f_step / (step_ms * 1e-3) / 1e12

    # Algorithmic FLOPs per launch (causal FlashAttention convention, unit G = B*H*T^2*D): the forward kernel does
    # the forward's 2G; the kv-pass does 4 of the backward's 5 G-sized products (S^T, dP^T, dV, dK); the q-pass does
    # dQ (its S and dP are the recomputation the convention does not count).
    G = float(Br) * Hr * T * T * D
    algo = {"fwd_tc": 2 * G, "fwd_simt": 2 * G, "bwd_kv_tc": 4 * G, "bwd_kv_simt": 4 * G, "bwd_q_tc": G,
            "bwd_q_simt": G}
    per_launch_us = {k: 1e3 * ms / n for k, (n, ms) in kernels.items()}
    dom = max(kernels, key=lambda k: kernels[k][1]) if kernels else None
    step_kernel_ms = sum(ms for (n, ms) in kernels.values()) / max(1, args.steps)
    if dom in algo:
        ach = algo[dom] / (per_launch_us[dom] * 1e-6) / 1e12
        roof = {"bound": "tensor", "kernel": dom, "achieved": ach, "peak": peak, "unit": "TFLOP/s",
                "frac": ach / peak, "peak_source": peak_src,
                "traffic": NCU_TRAFFIC_C2.get(dom) if (Br, Hr, T, D) == (4, 12, 2048, 64) else None,
                "traffic_unit": "bytes per launch (ncu dram__bytes_read.sum + dram__bytes_write.sum)",
                "share_of_step": kernels[dom][1] / max(1e-9, sum(ms for (n, ms) in kernels.values()))}
    else:
        roof = {"bound": "tensor", "kernel": "forward pass (field statistics + attention forward)",
                "achieved": per_gpu_fwd, "peak": peak, "unit": "TFLOP/s", "frac": per_gpu_fwd / peak,
                "peak_source": peak_src, "traffic": None}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        heads = 4
        dt, cores = cpu_oracle_sample(D, T, heads=heads)
        cpu = {"value": flops(1, heads, T, D, "fwd_bwd") / dt / 1e12, "unit": "TFLOP/s", "cores": cores,
               "kind": "port",
               "sample": f"{heads} of the {B * H} heads at T={T} D={D}, fwd+bwd, float64 NumPy oracle, {dt:.1f} s"}

    if rank == 0:
        line = {
            "metric": metric_for(B, H, T, D), "value": job_step, "unit": "TFLOP/s", "n_gpus": world, "steps": K,
            "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True, "scaling": args.scaling,
            "vs_baseline": (job_step / PUBLISHED_FWD_BWD_TFLOPS
                            if shape_label(B, H, T, D) == "configuration 2" else None),
            "dtype": "f16", "data": "synthetic",
            "config": {"workload": f"{shape_label(B, H, T, D)}: B{Br} H{Hr} T{T} D{D} fp16 fwd+bwd per GPU "
                                   f"({args.scaling})",
                       "global_heads": Br * Hr * world, "T": T, "D": D, "accumulate": "f32",
                       "parallelism": f"heads sharded over {world} GPU(s), no collective",
                       "l2": "flushed before every timed step (256 MiB write, outside the events)"},
            "fwd_ms": fwd_ms, "fwd_tflops": job_fwd, "fwd_pct_peak": 100 * per_gpu_fwd / peak,
            "fwd_bwd_ms": step_ms, "fwd_bwd_tflops": job_step, "fwd_bwd_pct_peak": 100 * per_gpu_step / peak,
            "roofline": roof,
            "kernels_us_per_launch": {k: round(v, 2) for k, v in sorted(per_launch_us.items())},
            "e2e": {"value": f_step * world / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4 * Br, "graph": e2e_graph is not None,
                    "result_read_back": "the loss sum(o * grad_o) of each sequence; gradients stay on the device",
                    "pipeline": f"{Br} sequences, one packed pinned block each; copy-in / 2 compute / copy-out "
                                "streams"},
            "e2e_all_outputs": {"value": f_step * world / (e2e_all_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                                "ms_per_step": e2e_all_ms, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                                "graph": e2e_all_graph is not None},
            "gpu_launches": launches,
            "step_graph": graph is not None,
            "clocks": sampler.summary(),
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

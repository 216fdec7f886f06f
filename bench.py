"""Benchmark: sink-attention kept-block TFLOP/s and layer latency at the Wan
32K shape, on 1..8 B200 GPUs (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one sink-attention forward of one Wan2.1 self-attention layer:
B=2 (CFG pair), H=12, S=32760 tokens padded to 32768 (256 blocks of 128),
D=128, bf16, with the benchmark's ~20% block mask (key block 0 | diagonal |
Bernoulli(0.2), seed 1). `value` is whole-job kept-block TFLOP/s
(4*D*sum of valid rows x valid cols over kept blocks, all ranks) over the
max-over-ranks device time of the K timed steps. Inputs (603 MB) exceed L2.

Multi-GPU (torchrun): the work shards by (batch, head) unit with no
collective on the data path. Strong scaling: the job is one Wan layer (24
units) on every N, split over the ranks (12, 6, 3 units per rank at N = 2, 4,
8); `value` is the layer's kept-block FLOPs over the slowest rank's time. At
N > 1 the line also carries the weak-scaling figure (every rank runs the
whole layer) and the same layer under Ulysses sequence parallelism (sequence
shards -> all-to-all -> units -> kernel -> all-to-all back).

Extra figures in the same JSON line: the density of the coverage-rule mask on
the stated generator (~0.83) and its TFLOP/s, the calibration pass (pooling
+ pooled softmax + batch mean + coverage mask of one cfg3 layer), the
end-to-end number through the reference-facing API with host buffers, the
roofline of the attention kernel, sampled clocks, and the CPU references
timed on the host cores: dense masked torch attention, and the calibration
path of two cfg3 layers (torch pooling and softmax, the oracle's coverage
mask).

--impl reference times the reference's CPU path for this operation (dense
masked fp32 attention in torch, as the benchmark defines its reference, on all
host threads), on a bounded sample of the same workload per step.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "sink-attn TFLOPS (kept blocks) & layer latency, Wan 32K seq, 1/2/4/8 B200"
UNIT = "TFLOP/s"
B, H, S, D = 2, 12, 32768, 128
NB = S // 128
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def load_traffic():
    """Per-launch DRAM bytes of the attention kernel from the committed ncu summary."""
    p = ROOT / "profiles" / "traffic.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except Exception:
            return {}
    return {}


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons around a region.

    A reader thread timestamps every sample. __enter__ returns once the first
    sample has arrived (so the sampler is live when timing starts); __exit__
    waits for one more sample. summary() uses the samples taken between the
    two."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int, period_ms: int = 50):
        self.idx = device_index
        self.period = period_ms
        self.proc = None
        self.samples: list[tuple[float, str]] = []
        self.t_start = self.t_end = None

    def _reader(self):
        for ln in self.proc.stdout:
            if ln.strip():
                self.samples.append((time.monotonic(), ln.strip()))

    def __enter__(self):
        import threading

        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", str(self.period), "-i", str(self.idx)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return self
        threading.Thread(target=self._reader, daemon=True).start()
        t0 = time.monotonic()
        while not self.samples and time.monotonic() - t0 < 10:
            time.sleep(0.005)
        self.t_start = time.monotonic()
        return self

    def __exit__(self, *exc):
        self.t_end = time.monotonic()
        if self.proc is not None:
            n = len(self.samples)
            t0 = time.monotonic()
            while len(self.samples) <= n and time.monotonic() - t0 < 2:
                time.sleep(0.005)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        return False

    def summary(self):
        if not self.samples or self.t_start is None:
            return None
        window = [ln for (t, ln) in self.samples
                  if self.t_start - self.period / 1e3 <= t <= self.t_end + self.period / 1e3]
        sm, mx, power, reasons = [], None, [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in window:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
                power.append(float(parts[3]))
            except ValueError:
                continue
            for n, val in zip(names, parts[5:9]):
                if val.lower() in ("active", "1"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(power) if power else None,
                "window_s": round(self.t_end - self.t_start, 3)}


_TRACE = os.environ.get("SINKATTN_BENCH_TRACE") == "1"


def trace(msg: str) -> None:
    """Timestamped progress line on stderr (SINKATTN_BENCH_TRACE=1)."""
    if _TRACE:
        print(f"[bench {time.strftime('%H:%M:%S')} rank {os.environ.get('RANK', '0')}] {msg}",
              file=sys.stderr, flush=True)


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def init_dist(world: int, backend: str, device=None):
    if world > 1:
        import datetime

        import torch.distributed as dist

        kw = {"device_id": device} if (backend == "nccl" and device is not None) else {}
        dist.init_process_group(backend=backend, timeout=datetime.timedelta(seconds=120), **kw)


def max_over_ranks(x: float, world: int, device) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: int, world: int, device) -> int:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return int(t.item())


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


# ---------------------------------------------------------------------------
# CPU (reference path) timing
# ---------------------------------------------------------------------------
def torch_masked_attention(q, k, v, block_mask, row_chunk=512):
    """Dense masked attention as the benchmark defines its reference (cfg1:
    dense torch attention with the block mask expanded to tokens and masked
    scores set to -inf), in fp32 torch on the CPU so that every host thread
    works: q [Sq,D], k/v [Sk,D], block_mask bool [nq,nk]. Returns out, lse."""
    Sq, D = q.shape
    Sk = k.shape[0]
    scale = 1.0 / math.sqrt(D)
    tok = block_mask.repeat_interleave(128, 0).repeat_interleave(128, 1)[:Sq, :Sk]
    out = torch.empty(Sq, D)
    lse = torch.empty(Sq)
    kt = k.t().contiguous()
    for r0 in range(0, Sq, row_chunk):
        r1 = min(Sq, r0 + row_chunk)
        sc = (q[r0:r1] @ kt) * scale
        sc.masked_fill_(~tok[r0:r1], float("-inf"))
        lse[r0:r1] = torch.logsumexp(sc, dim=-1)
        out[r0:r1] = torch.softmax(sc, dim=-1) @ v
    return out, lse


def cpu_attention_sample(q, k, v, mask, units, q_blocks):
    """Time dense masked fp32 attention on the host (torch, all threads) on
    `units` (b, h) pairs x `q_blocks` query blocks each. Returns (seconds,
    kept FLOPs of the sample)."""
    flops = 0.0
    t0 = time.perf_counter()
    for (b, h) in units:
        rows = slice(0, q_blocks * 128)
        m = mask[0, h, :q_blocks]
        torch_masked_attention(q[b, h, rows], k[b, h], v[b, h], m)
        flops += 4.0 * D * 128 * 128 * float(m.sum().item())
    return time.perf_counter() - t0, flops


def cpu_calibration_layer(q, k, oracle):
    """One cfg3 layer of the calibration path on the host, as the reference
    computes it with pooling_mode "mean" (sparse_attention.py:118-142, 575-582,
    268-376): fp32 means of Q and K over 128-token blocks, pooled logits scaled
    by 1/sqrt(D), a row softmax and the batch mean in torch on all threads,
    then the coverage mask (0.85, key block 0 kept) by the oracle's
    restatement. q, k: bf16 [B,H,S,D] with S a multiple of 128. Returns the
    mask [H,nb,nb]."""
    Bq, Hq, Sq, Dq = q.shape
    nb = Sq // 128
    qp = q.float().view(Bq, Hq, nb, 128, Dq).mean(3)
    kp = k.float().view(Bq, Hq, nb, 128, Dq).mean(3)
    scores = torch.softmax(torch.matmul(qp, kp.transpose(-1, -2)) / math.sqrt(Dq), dim=-1)
    bm = scores.mean(0)
    return oracle.coverage_mask(bm.numpy(), force_sink_col=True,
                                row_total=bm.sum(-1).numpy()).mask


def cpu_calibration_sample(layers=2):
    """Time `layers` cfg3 layers (seed = layer index) of cpu_calibration_layer
    after one untimed layer. Returns (seconds, algorithmic bytes: Q and K read
    in bf16 plus the 1-byte mask write, per layer)."""
    from oracle import sinkattn_oracle as oracle
    from tests.gen import wan_qk

    inputs = [wan_qk(seed=s, dtype=torch.bfloat16)[:2] for s in range(layers)]
    cpu_calibration_layer(*inputs[0], oracle)
    t0 = time.perf_counter()
    for q, k in inputs:
        cpu_calibration_layer(q, k, oracle)
    dt = time.perf_counter() - t0
    return dt, layers * (2 * B * H * S * D * 2 + H * NB * NB)


def make_cpu_sample(seed=0):
    from tests.gen import cfg1_mask, wan_qk

    q, k, v = wan_qk(seed=seed, B=1, H=2, dtype=torch.float32)
    mask = cfg1_mask(12, NB, NB, seed=1).unsqueeze(0)[:, :2]
    # bf16-valued fp32, like the GPU inputs
    q, k, v = (t.bfloat16().float().contiguous() for t in (q, k, v))
    return q, k, v, mask


def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    q, k, v, mask = make_cpu_sample()
    units = [(0, 0), (0, 1)]
    q_blocks = 32
    for _ in range(max(0, args.warmup)):
        cpu_attention_sample(q, k, v, mask, units[:1], 4)
    times, flops = [], 0.0
    for _ in range(args.steps):
        dt, flops = cpu_attention_sample(q, k, v, mask, units, q_blocks)
        times.append(dt)
    total = sum(times)
    value = flops * args.steps / total / 1e12
    sample = (f"{len(units)} (b,h) units x {q_blocks} query blocks x all 256 key blocks of the "
              f"Wan layer (cfg1-style mask, rho~0.21), dense masked fp32 torch attention per "
              f"step")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * total / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded, BASELINE cfg2 generator)",
        "config": {"workload": "wan_sink_attention_layer", "B": B, "H": H, "S": S, "D": D,
                   "mask": "col0|diag|bernoulli(0.2)", "sample": sample},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def kept_flops(mask_bhqk: torch.Tensor) -> float:
    # S is a multiple of 128 here: every kept block is a full 128 x 128 tile
    return 4.0 * D * 128 * 128 * float(mask_bhqk.sum().item())


def memcpy2d_async(dst: int, dpitch: int, src: int, spitch: int, width: int, height: int,
                   kind: str, stream) -> None:
    """One cudaMemcpy2DAsync (pinned host <-> device) on a torch stream."""
    from cuda.bindings import runtime as cudart

    k = (cudart.cudaMemcpyKind.cudaMemcpyHostToDevice if kind == "h2d"
         else cudart.cudaMemcpyKind.cudaMemcpyDeviceToHost)
    (err,) = cudart.cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, height, k,
                                      stream.cuda_stream)
    if err != cudart.cudaError_t.cudaSuccess:
        raise RuntimeError(f"cudaMemcpy2DAsync failed: {err}")


def time_steps(fn, steps, stream):
    """Device time of `steps` calls (ms) with CUDA events on `stream`."""
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for i in range(steps):
        starts[i].record(stream)
        fn()
        ends[i].record(stream)
    t1.record(stream)
    torch.cuda.synchronize()
    per = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    return t0.elapsed_time(t1), per


def run_ours(args):
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    init_dist(world, "nccl", dev)
    barrier(world)
    trace("process group up")
    from sinkattn_b200 import _lib, ops
    from sinkattn_b200.sharding import partition_units
    from tests.gen import cfg1_mask, wan_qk

    _lib.load()
    peaks, peak_kind = load_peaks()
    stream = torch.cuda.current_stream(dev)

    # inputs: Wan layout (BSHD memory viewed as BHSD), the same layer on every
    # rank; rank r computes its share of the (batch, head) units
    trace("generating inputs")
    qh, kh, vh = wan_qk(seed=0, dtype=torch.bfloat16)  # [B,H,S,D] on CPU
    trace("inputs generated")
    q_bshd = qh.permute(0, 2, 1, 3).contiguous()
    k_bshd = kh.permute(0, 2, 1, 3).contiguous()
    v_bshd = vh.permute(0, 2, 1, 3).contiguous()
    del qh, kh, vh
    q = q_bshd.to(dev).permute(0, 2, 1, 3)
    k = k_bshd.to(dev).permute(0, 2, 1, 3)
    v = v_bshd.to(dev).permute(0, 2, 1, 3)
    mask20 = cfg1_mask(H, NB, NB, seed=1).unsqueeze(0).expand(B, -1, -1, -1).contiguous().to(dev)
    flops20 = kept_flops(mask20)  # the whole layer: the job's fixed work
    out = torch.empty(B, S, H, D, dtype=torch.bfloat16, device=dev).permute(0, 2, 1, 3)
    lse = torch.empty(B, H, S, dtype=torch.float32, device=dev)
    units = partition_units(B * H, world, rank)
    segs = unit_segments(units, H)
    flops20_r = sum(kept_flops(mask20[b0:b1, h0:h1]) for b0, b1, h0, h1 in segs)

    def attn_units(mask):
        for b0, b1, h0, h1 in segs:
            sl = (slice(b0, b1), slice(h0, h1))
            ops.bsattn_fwd(q[sl], k[sl], v[sl], mask[sl], out=out[sl], lse=lse[sl])

    def step20():
        attn_units(mask20)

    def step20_full():
        ops.bsattn_fwd(q, k, v, mask20, out=out, lse=lse)

    # calibration layer on this layer's Q/K, one fused launch: pool -> pooled
    # logits -> softmax -> batch mean -> coverage mask (key block 0 forced)
    ws = ops.pool_scores_workspace(B, H, S, D, device=dev)
    calib = {"mask": torch.empty(H, NB, NB, dtype=torch.bool, device=dev)}

    def step_calib():
        ops.calibration_layer(q, k, want_batch_mean=False, mask_out=calib["mask"],
                              force_sink_col=True, workspace=ws)

    step_calib()
    torch.cuda.synchronize()
    trace("first calibration step done")
    mask83 = calib["mask"].unsqueeze(0).expand(B, -1, -1, -1).contiguous()
    density83 = float(mask83.float().mean().item())
    flops83 = kept_flops(mask83)

    def step83():
        attn_units(mask83)

    for i in range(max(3, args.warmup)):
        for name, fn in (("attn rho21", step20), ("attn coverage-mask", step83),
                         ("calibration", step_calib), ("attn full layer", step20_full)):
            fn()
            if _TRACE:
                torch.cuda.synchronize()
                trace(f"warm-up {i} {name} done")
    torch.cuda.synchronize()

    trace("warm-up done")
    # ---- headline: rho ~ 0.21 -------------------------------------------
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        total_ms, per_ms = time_steps(step20, args.steps, stream)
    torch.cuda.synchronize()
    barrier(world)
    max_ms = max_over_ranks(total_ms, world, dev)
    min_ms = -max_over_ranks(-total_ms, world, dev)
    ms_step = max_ms / args.steps
    value = flops20 * args.steps / (max_ms / 1e3) / 1e12
    avg_launch_ms = statistics.mean(per_ms) / len(segs)
    achieved = flops20_r / len(segs) / (avg_launch_ms / 1e3) / 1e12
    frac_r = flops20_r / (total_ms / args.steps / 1e3) / 1e12 / float(
        peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    frac_min = -max_over_ranks(-frac_r, world, dev)
    replicas = None
    if world > 1:
        # weak-scaling figure: every rank runs the whole layer
        barrier(world)
        t_rep, _ = time_steps(step20_full, args.steps, stream)
        barrier(world)
        t_rep = max_over_ranks(t_rep, world, dev)
        replicas = {"value": flops20 * world * args.steps / (t_rep / 1e3) / 1e12, "unit": UNIT,
                    "ms_per_step": t_rep / args.steps, "scaling": "weak",
                    "note": "every rank runs the whole layer (24 units); value = all ranks' "
                            "kept-block FLOPs over the max-over-ranks time"}

    trace("headline timed")
    # ---- coverage-rule mask (rho ~ 0.83) ----------------------------------
    barrier(world)
    t83, per83 = time_steps(step83, args.steps, stream)
    t83 = max_over_ranks(t83, world, dev)
    calib_legs = None
    if world == 1:
        calib_legs = calibration_legs(args, q, k, v, ws, step_calib, stream, dev, peaks)
    ulysses = None
    if world > 1:
        ulysses = ulysses_leg(args, q, k, v, mask20, world, rank, dev, stream)

    trace("e2e")
    te2e, h2d, d2h, hg = e2e_leg(args, q_bshd, k_bshd, v_bshd, mask20, segs, dev, stream, world)
    e2e_value = flops20 * args.steps / (te2e / 1e3) / 1e12

    trace("e2e timed")
    # ---- cfg5: the full DiT step (sequence parallel at N > 1) ---------------
    dit = None if args.skip_dit else dit_leg(args, world, rank, dev, stream)
    trace("dit timed")
    # ---- CPU baseline (rank 0, N=1 only) ------------------------------------
    cpu = cpu_cal = None
    if rank == 0 and world == 1 and not args.skip_cpu:
        cpu, cpu_cal = cpu_legs()

    traffic = load_traffic().get("bsattn_fwd_wan_rho21")
    if traffic is not None:
        # the committed capture is of the whole layer (24 units)
        traffic = traffic * len(units) / (B * H) / len(segs)
    peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded BASELINE cfg2 generator: N(0,1) + 0.5*PE3D, V ~ N(0,1))",
        "config": {"workload": "wan_sink_attention_layer (cfg2: B=2,H=12,S=32768,D=128)",
                   "global_batch": B, "seq_len": S, "heads": H, "head_dim": D,
                   "parallelism": f"(b,h)-unit sharding x{world}: the layer's 24 units split "
                                  f"over the ranks, no collective",
                   "mask": "col0|diag|bernoulli(0.2) seed 1",
                   "density": float(mask20.float().mean().item()),
                   "l2": "inputs 603 MB > L2 (no flush)"},
        "layer_latency_ms": ms_step,
        "per_gpu": {"units": len(units), "launches_per_step": len(segs),
                    "ms_slowest": max_ms / args.steps, "ms_fastest": min_ms / args.steps,
                    "frac_min": frac_min, "frac_rank0": frac_r},
        "replicas": replicas,
        "coverage_rule_mask": {"density": density83, "ms_per_step": t83 / args.steps,
                               "value": flops83 * args.steps / (t83 / 1e3) / 1e12,
                               "unit": UNIT},
        **(calib_legs or {}),
        "ulysses": ulysses,
        "dit_step_cfg5": dit,
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": te2e / args.steps,
                "chunk_heads": hg,
                "api": "sinkattn_b200.reference_api._block_sparse_attn",
                "note": "pinned host buffers [B,S,H,D]; each rank moves its own units in "
                        "chunks of (batch element, chunk_heads heads) as 2-D copies: H2D of "
                        "chunk c+1 overlaps the call on chunk c, D2H of c overlaps the later "
                        "H2D copies; bytes are the whole job's"},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": UNIT,
                     "frac": achieved / peak, "traffic": traffic,
                     "kernel": "sa::attn::bsattn_fwd_kernel",
                     "peak_kind": f"bf16_tflops ({peak_kind}, burst)",
                     # context: the same against the sustained figure (a GEMM loop held
                     # at the power cap), the regime the clock record shows when it
                     # lists sw_power_cap during the timed steps
                     "frac_of_sustained": achieved / float(
                         peaks.get("bf16_tflops_sustained",
                                   FALLBACK_PEAKS["bf16_tflops_sustained"])),
                     "algorithmic_flops_per_launch": flops20_r / len(segs)},
        "gpu_launches": args.steps * len(segs),
        "clocks": clk.summary(),
        "cpu_baseline": cpu,
        "cpu_baseline_calibration": cpu_cal,
    }
    from sinkattn_b200.ops import DeviceStatus

    DeviceStatus.check(dev)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return 0


def calibration_legs(args, q, k, v, ws, step_calib, stream, dev, peaks):
    """The calibration figures of one GPU: the fused calibration layer, the
    same without the mask, the device calibrator's record, and the 30-layer
    calibration pass with its check against the reference row totals."""
    from sinkattn_b200 import _lib, ops

    # The attention legs before this one hold the GPU at its power cap; right
    # after them the SM clocks run lower for a while (measured: the
    # calibration kernel about 17% slower). These legs start from 2 s idle.
    torch.cuda.synchronize()
    time.sleep(2.0)
    # ---- calibration layer ----------------------------------------------------
    tcal, _ = time_steps(step_calib, args.steps, stream)
    calib_bytes = 2 * B * H * S * D * 2 + H * NB * NB  # read Q,K (bf16) + write mask

    def step_pool_only():
        ops.pool_scores(q, k, want_scores=False, want_batch_mean=True, workspace=ws)

    step_pool_only()
    tpool, _ = time_steps(step_pool_only, args.steps, stream)

    # the device calibrator's record (reference default config with the mean
    # rule): one fused launch that also adds to the layer's running sums
    from sinkattn_b200.calibrator import DeviceSinkMaskCalibrator
    from tests.gen import default_config

    cal = DeviceSinkMaskCalibrator(default_config(pooling_mode="mean"))

    def step_record():
        cal.record(0, q, k, v)

    step_record()
    trec, _ = time_steps(step_record, args.steps, stream)

    trace("calibration layer timed")
    # ---- cfg3: the 30-layer calibration pass, layers pipelined on two streams
    from tests.gen import wan_qk_layers_on_device

    layers = wan_qk_layers_on_device(30, dev)
    masks30 = torch.empty(30, H, NB, NB, dtype=torch.bool, device=dev)

    def step_pass():
        ops.calibration_pass(layers, force_sink_col=True, masks_out=masks30, workspace=ws)

    for _ in range(2):
        step_pass()
    torch.cuda.synchronize()
    pass_steps = max(3, min(10, args.steps // 10))
    tpass, _ = time_steps(step_pass, pass_steps, stream)
    pass_ms = tpass / pass_steps
    pass_bytes = 30 * calib_bytes
    density30 = float(masks30.float().mean().item())
    # the pass's masks against the reference rule on the same batch means with
    # the reference's fp32 row totals (CPU torch.sum), outside the timed region
    _, bms30, flags30 = ops.calibration_pass(layers, force_sink_col=True, want_batch_mean=True,
                                             want_flags=True, workspace=ws)
    bms30_c = bms30.cpu()
    ref30 = torch.stack([ops.coverage_mask(bms30[l], force_sink_col=True,
                                           row_total=bms30_c[l].sum(-1).to(dev))[0]
                         for l in range(30)])
    diff30 = (ref30 != masks30).any(-1)
    near = (flags30 & (_lib.SA_ROW_NEAR_TARGET | _lib.SA_ROW_TIE_AT_CUT)) != 0
    pass_check = {"rows": int(diff30.numel()), "flagged_rows": int(near.sum()),
                  "differing_rows": int(diff30.sum()),
                  "differing_unflagged_rows": int((diff30 & ~near).sum())}
    del layers, bms30, ref30

    trace("calibration pass timed")
    hbm = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    pool_bytes = 2 * B * H * S * D * 2
    return {
        "calibration_layer": {"ms_per_layer": tcal / args.steps,
                              "pool_scores_ms": tpool / args.steps,
                              "calibrator_record_ms": trec / args.steps,
                              "bytes": calib_bytes,
                              "gbs": calib_bytes / (tcal / args.steps / 1e3) / 1e9,
                              "frac_of_hbm": calib_bytes / (tcal / args.steps / 1e3) / 1e9 / hbm,
                              "pool_scores_frac_of_hbm": pool_bytes
                              / (tpool / args.steps / 1e3) / 1e9 / hbm,
                              "note": "one fused launch (pool -> pooled logits -> softmax -> "
                                      "batch mean -> coverage mask); pool_scores_ms: the same "
                                      "without the mask (scores' batch mean only); "
                                      "calibrator_record_ms: DeviceSinkMaskCalibrator.record, "
                                      "mean rule, with the running sums; timed after 2 s idle "
                                      "following the attention legs"},
        "calibration_pass_30_layers": {
            "ms_per_pass": pass_ms, "ms_per_layer": pass_ms / 30,
            "bytes_per_pass": pass_bytes,
            "gbs": pass_bytes / (pass_ms / 1e3) / 1e9,
            "frac_of_hbm": pass_bytes / (pass_ms / 1e3) / 1e9 / hbm,
            "mask_density": density30,
            "vs_reference_totals": pass_check,
            "note": "cfg3: 30 layers x Q,K [2,12,32768,128] bf16 (GPU-generated, seed=layer); "
                    "one fused launch per layer (pool -> pooled logits -> softmax -> batch "
                    "mean -> coverage mask, sink column forced, device row totals); "
                    "vs_reference_totals: rows whose mask differs from the rule with the "
                    "reference's CPU fp32 row totals, all of which must be flagged"},
    }


def unit_segments(units, heads):
    """(b0, b1, h0, h1) rectangles covering a contiguous run of (batch, head)
    units u = b * heads + h: whole batch elements as one rectangle, a partial
    batch element as its own."""
    segs = []
    u, end = (units[0], units[-1] + 1) if units else (0, 0)
    while u < end:
        b, h = divmod(u, heads)
        if h == 0 and end - u >= heads:
            nb_ = (end - u) // heads
            segs.append((b, b + nb_, 0, heads))
            u += nb_ * heads
        else:
            h1 = min(heads, h + end - u)
            segs.append((b, b + 1, h, h1))
            u += h1 - h
    return segs


def e2e_leg(args, q_bshd, k_bshd, v_bshd, mask20, segs, dev, stream, world):
    """End to end through the reference-facing API with pinned host buffers:
    each rank copies in and out only its own units. Returns the
    max-over-ranks ms of the K steps, the whole job's H2D and D2H bytes per
    step, and the heads per chunk."""
    from sinkattn_b200.reference_api import _block_sparse_attn

    qp = q_bshd.pin_memory()
    kp = k_bshd.pin_memory()
    vp = v_bshd.pin_memory()
    out_h = torch.empty(B, S, H, D, dtype=torch.bfloat16).pin_memory()
    lse_h = torch.empty(B, H, S, 1, dtype=torch.bfloat16).pin_memory()
    q_d = torch.empty_like(q_bshd, device=dev)
    k_d = torch.empty_like(k_bshd, device=dev)
    v_d = torch.empty_like(v_bshd, device=dev)

    # The step moves the inputs in chunks of (batch element, group of heads):
    # the host-to-device copy of chunk c+1 (copy engine) overlaps the attention
    # call on chunk c, and the device-to-host copy of c's result overlaps the
    # later copies in (PCIe is full duplex). A head group of the [B,S,H,D]
    # buffers is a strided 2-D region (S rows of hg*D elements, pitch H*D), so
    # each tensor of a chunk is one cudaMemcpy2DAsync.
    hg = max(1, min(H, args.e2e_chunk_heads))
    while any((s1 - s0) % hg for _, _, s0, s1 in segs):
        hg -= 1
    chunks = [(b, h0) for b0, b1, s0, s1 in segs for b in range(b0, b1)
              for h0 in range(s0, s1, hg)]
    s_h2d, s_cmp, s_d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in chunks]
    ev_out = [torch.cuda.Event() for _ in chunks]
    pitch = H * D * 2
    width = hg * D * 2

    def step_e2e():
        for st_ in (s_h2d, s_cmp, s_d2h):
            st_.wait_stream(stream)
        for c, (b, h0) in enumerate(chunks):
            for dst, src in ((q_d, qp), (k_d, kp), (v_d, vp)):
                memcpy2d_async(dst[b, 0, h0].data_ptr(), pitch, src[b, 0, h0].data_ptr(), pitch,
                               width, S, "h2d", s_h2d)
            ev_in[c].record(s_h2d)
        for c, (b, h0) in enumerate(chunks):
            with torch.cuda.stream(s_cmp):
                s_cmp.wait_event(ev_in[c])
                sl = (slice(b, b + 1), slice(None), slice(h0, h0 + hg))
                o, l = _block_sparse_attn(q_d[sl].permute(0, 2, 1, 3), k_d[sl].permute(0, 2, 1, 3),
                                          v_d[sl].permute(0, 2, 1, 3),
                                          mask20[b:b + 1, h0:h0 + hg], return_lse=True)
                ev_out[c].record(s_cmp)
            o.record_stream(s_d2h)
            l.record_stream(s_d2h)
            with torch.cuda.stream(s_d2h):
                s_d2h.wait_event(ev_out[c])
                # o is [1,S,hg,D]-contiguous, viewed [1,hg,S,D]
                memcpy2d_async(out_h[b, 0, h0].data_ptr(), pitch, o.data_ptr(), width, width, S,
                               "d2h", s_d2h)
                lse_h[b, h0:h0 + hg].copy_(l[0], non_blocking=True)
        for st_ in (s_h2d, s_cmp, s_d2h):
            stream.wait_stream(st_)

    for _ in range(2):
        step_e2e()
    torch.cuda.synchronize()
    barrier(world)
    te2e, _ = time_steps(step_e2e, args.steps, stream)
    barrier(world)
    te2e = max_over_ranks(te2e, world, dev)
    n_heads = sum((b1 - b0) * (h1 - h0) for b0, b1, h0, h1 in segs)
    h2d = sum_over_ranks(3 * S * n_heads * D * 2, world, dev)
    d2h = sum_over_ranks(S * n_heads * D * 2 + n_heads * S * 2, world, dev)
    return te2e, h2d, d2h, hg


def dit_leg(args, world, rank, dev, stream):
    """BASELINE cfg5: one step of a random-weight Wan2.1-1.3B-shaped DiT (30
    blocks, latent [2,16,21,60,104] = 32760 tokens, text 512 x 4096, weights
    N(0,0.02) seed 0; tests/wan_dit.py) whose self-attention runs the
    reference's WanSinkSparseAttnProcessor2_0 with install() in place, each
    layer with its cfg3 calibration-pass mask and the Wan runtime default
    (pooled K/V gap 30, adaptive mix). At N > 1 the activations are
    sequence-sharded (S/N tokens per rank) and the attention goes through the
    peer-memory Ulysses exchange. Returns the max-over-ranks step time."""
    ref_dir = Path(os.environ.get("SINKATTN_REFERENCE", ROOT / "baseline" / "_ref"))
    if not (ref_dir / "wanx").exists():
        return {"unavailable": f"reference processors not installed under {ref_dir}"}
    if str(ref_dir) not in sys.path:
        sys.path.insert(0, str(ref_dir))
    from sinkattn_b200 import ops
    from sinkattn_b200 import reference_api as ra
    from tests import wan_dit
    from tests.gen import wan_qk_layers_on_device

    ra.install()
    layers = wan_qk_layers_on_device(30, dev)
    masks = ops.calibration_pass(layers, force_sink_col=True)[0]
    del layers
    torch.cuda.empty_cache()
    model, ex = wan_dit.build(masks, dev, world=world, rank=rank)
    x, t, text, rot = wan_dit.inputs(dev)
    shard = (rank, world) if world > 1 else None

    def step():
        with torch.no_grad():
            model(x, t, text, rot, shard=shard)

    steps = 3
    for _ in range(2):
        step()
    torch.cuda.synchronize()
    barrier(world)
    total, per = time_steps(step, steps, stream)
    barrier(world)
    ms = max_over_ranks(total / steps, world, dev)
    tokens = x.shape[0] * rot.shape[2]
    res = {"ms_per_step": ms, "tokens_per_s": tokens / (ms / 1e3), "layers": len(model.blocks),
           "tokens": tokens, "ranks": world, "steps": steps,
           "mask_density": float(masks.float().mean().item()),
           "parallelism": ("sequence parallel, Ulysses exchange over NVLink peer memory"
                           if world > 1 else "one GPU"),
           "attention": "reference WanSinkSparseAttnProcessor2_0 with install(): fused Q/K "
                        "RMSNorm + RoPE producer, fused sink + pooled-K/V dynamic kernel"}
    if ex is not None:
        ex.close()
    del model, x, text, rot, masks
    torch.cuda.empty_cache()
    return res


def cpu_legs():
    """The CPU baselines on all host threads: dense masked fp32 torch
    attention on 2 units x 32 query blocks, and the calibration path of two
    cfg3 layers."""
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cq, ck, cv, cm = make_cpu_sample()
    cpu_attention_sample(cq, ck, cv, cm, [(0, 0)], 2)
    dt, fl = cpu_attention_sample(cq, ck, cv, cm, [(0, 0), (0, 1)], 32)
    cpu = {"value": fl / dt / 1e12, "unit": UNIT, "cores": threads, "kind": "port",
           "sample": "2 (b,h) units x 32 query blocks x 256 key blocks, rho~0.21, "
                     "dense masked fp32 torch attention (the benchmark's reference)"}
    ct, cb = cpu_calibration_sample(2)
    cpu_cal = {"value": cb / ct / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
               "ms_per_layer": 1e3 * ct / 2,
               "sample": "2 cfg3 layers (seeds 0, 1) after 1 untimed: torch fp32 128-token "
                         "block means of Q and K, pooled softmax, batch mean, then the "
                         "oracle's coverage mask (0.85, key block 0 kept)"}
    return cpu, cpu_cal


def ulysses_leg(args, q, k, v, mask20, world, rank, dev, stream):
    """The same layer under sequence parallelism: each rank starts from its
    [B, S/P, H, D] sequence shard, one all-to-all per tensor turns the shards
    into whole-sequence (b, h) units, the kernel runs, and the inverse
    all-to-all returns the output in the sequence layout. Times the whole
    exchange + attention + exchange, over NCCL all-to-alls and over NVLink
    peer memory (UlyssesPeerExchange), and the kernel alone on the same
    units."""
    from sinkattn_b200.sharding import (_local_units_attention, sequence_to_units,
                                        ulysses_sink_attention, units_per_rank)

    Sr = S // world
    sl = slice(rank * Sr, (rank + 1) * Sr)
    qs, ks, vs = (x.permute(0, 2, 1, 3)[:, sl].contiguous() for x in (q, k, v))
    n_per = units_per_rank(B * H, world)
    steps = max(3, min(20, args.steps))

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        barrier(world)
        total, _ = time_steps(fn, steps, stream)
        barrier(world)
        return max_over_ranks(total / steps, world, dev)

    res = {"units_per_rank": n_per, "steps": steps,
           "exchange_mb_per_rank": 4 * B * Sr * H * D * 2 * (world - 1) / world / 1e6,
           "ms_layer": {}}
    res["ms_layer"]["1"] = timed(lambda: ulysses_sink_attention(qs, ks, vs, mask20))
    units = [sequence_to_units(x) for x in (qs, ks, vs)]
    m = mask20.reshape(B * H, NB, NB)
    ids = [rank * n_per + i for i in range(n_per)]
    mu = torch.stack([m[i] if i < B * H else torch.ones_like(m[0]) for i in ids]).contiguous()
    res["ms_attention_only"] = timed(lambda: _local_units_attention(*units, mu, ops_attn))
    res["exchange_overhead_nccl"] = min(res["ms_layer"].values()) / res["ms_attention_only"]
    # the exchange over NVLink peer memory: dispatch / combine kernels
    # writing into the owners' CUDA-IPC-mapped buffers
    from sinkattn_b200.sharding import UlyssesPeerExchange

    ex = UlyssesPeerExchange(B, S, H, device=dev)
    o_ref, l_ref = ulysses_sink_attention(qs, ks, vs, mask20)
    o_p, l_p = ex(qs, ks, vs, mask20)
    torch.cuda.synchronize()
    res["peer_equals_nccl"] = bool(torch.equal(o_p, o_ref) and torch.equal(l_p, l_ref))
    res["ms_layer_peer"] = timed(lambda: ex(qs, ks, vs, mask20))
    res["exchange_overhead"] = res["ms_layer_peer"] / res["ms_attention_only"]
    ex.close()
    del qs, ks, vs, units, o_ref, l_ref
    return res


def run_case(args):
    """Small single-GPU cases for profiler captures (inputs larger than L2,
    a few hundred MB on the device): one warm-up launch, then `--steps`
    launches of the named kernel chain."""
    from sinkattn_b200 import ops
    from tests.gen import cfg1_mask, wan_qk

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if args.case == "wan-runtime":
        # Wan runtime inner attention: sink mask | band 1, pooled K/V gap 30, adaptive mix
        from sinkattn_b200 import reference_api as ra

        q, k, v = wan_qk(seed=0, dtype=torch.bfloat16, device=dev)
        m = cfg1_mask(H, NB, NB, seed=1)
        ii = torch.arange(NB)
        m = m | ((ii[:, None] - ii[None, :]).abs() <= 1)
        mask = m.unsqueeze(0).expand(B, -1, -1, -1).contiguous().to(dev)

        class Cfg:
            mixing_mode = "adaptive"
            sample_gap = 30

        def fused():
            kp = ops.mean_pool_seq(k, 30)
            vp = ops.mean_pool_seq(v, 30)
            return ops.sink_dynamic_attn(q, k, v, mask, kp, vp, 30)

        def unfused():
            o_s, l_s = ra._block_sparse_attn(q, k, v, mask, return_lse=True)
            kp = ops.mean_pool_seq(k, 30)
            vp = ops.mean_pool_seq(v, 30)
            dm = torch.ones(B, H, NB, math.ceil(kp.shape[2] / 128), dtype=torch.bool, device=dev)
            o_d, l_d = ra._block_sparse_attn(q, kp, vp, dm, return_lse=True)
            return ra._mix_attention_outputs(o_s, l_s, o_d, l_d, Cfg, 30)

        res = {"case": args.case}
        skp = math.ceil(S / 30)
        flops = kept_flops(mask) + 4.0 * D * S * skp * B * H
        for name, fn in (("fused", fused), ("unfused", unfused)):
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            total, _ = time_steps(fn, args.steps, torch.cuda.current_stream(dev))
            res[name + "_ms"] = total / args.steps
            res[name + "_tflops"] = flops / (total / args.steps / 1e3) / 1e12
        print(json.dumps(res))
        return 0
    if args.case == "calib-pass":
        from tests.gen import wan_qk_layers_on_device

        layers = wan_qk_layers_on_device(30, dev)
        fn = lambda: ops.calibration_pass(layers, force_sink_col=True)  # noqa: E731
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        total, per = time_steps(fn, args.steps, torch.cuda.current_stream(dev))
        ms = total / args.steps
        gbs = 30 * (2 * B * H * S * D * 2 + H * NB * NB) / (ms / 1e3) / 1e9
        print(json.dumps({"case": args.case, "ms_per_pass": ms, "ms_per_layer": ms / 30, "gbs": gbs}))
        return 0
    if args.case == "qkrope-wan":
        # the Q/K producer (RMSNorm + rotary) at the Wan shape: B=2, 32760 tokens, 12 x 128
        tokens, hidden = 32760, H * D
        g = torch.Generator(device=dev).manual_seed(0)
        qa = torch.randn(B, tokens, hidden, generator=g, device=dev).bfloat16()
        ka = torch.randn(B, tokens, hidden, generator=g, device=dev).bfloat16()
        wq = torch.ones(hidden, device=dev).bfloat16()
        ang = torch.outer(torch.arange(tokens, device=dev, dtype=torch.float32),
                          torch.linspace(0, 1, D // 2, device=dev))
        cos, sin = torch.cos(ang), torch.sin(ang)
        qo, ko = torch.empty_like(qa), torch.empty_like(ka)
        fn = lambda: ops.qk_norm_rope(qa, ka, D, 1e-6, wq, wq, cos, sin, out_q=qo, out_k=ko)  # noqa: E731
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        total, _ = time_steps(fn, args.steps, torch.cuda.current_stream(dev))
        ms = total / args.steps
        nbytes = 4 * B * tokens * hidden * 2
        print(json.dumps({"case": args.case, "ms": ms, "bytes": nbytes,
                          "gbs": nbytes / (ms / 1e3) / 1e9}))
        return 0
    if args.case == "misc-wan":
        # the two bandwidth kernels of the unfused Wan runtime at its real shape
        # (B=2, H=12, 32760 tokens): sequence mean pooling with gap 30 (the pooled
        # K/V of the dynamic branch) and the adaptive LSE mix of the two branches.
        # Inputs are strided [B,S,H,D] storage as the processors produce them.
        tokens, gap = 32760, 30
        g = torch.Generator(device=dev).manual_seed(0)

        def bshd():
            x = torch.randn(B, tokens, H, D, generator=g, device=dev, dtype=torch.bfloat16)
            return x.permute(0, 2, 1, 3)

        xs = [bshd() for _ in range(2)]  # pooled alternately: 403 MB, more than L2
        o_s, o_d = bshd(), bshd()
        l_s = torch.randn(B, H, tokens, generator=g, device=dev) + 8.0
        l_d = torch.randn(B, H, tokens, generator=g, device=dev) + 5.0
        peak = float(load_peaks()[0].get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
        elems = B * H * tokens * D
        rows_out = math.ceil(tokens / gap)
        cases = {
            "mean_pool_seq": (lambda i: ops.mean_pool_seq(xs[i % 2], gap),
                              2 * elems + 2 * B * H * rows_out * D),
            "mix_outputs": (lambda i: ops.mix_outputs(o_s, l_s, o_d, l_d, gap),
                            3 * 2 * elems + 2 * 4 * B * H * tokens),
        }
        res = {"case": args.case, "B": B, "H": H, "S": tokens, "peak_gbs": peak}
        stream = torch.cuda.current_stream(dev)
        for name, (fn, nbytes) in cases.items():
            it = iter(range(1 << 30))
            call = lambda: fn(next(it))  # noqa: E731
            for _ in range(3):
                call()
            torch.cuda.synchronize()
            # a ~25 ms device spin first, so that every timed launch is queued
            # before the device reaches it and the per-launch events measure the
            # kernel rather than the host's launch rate
            torch.cuda._sleep(50_000_000)
            _, per = time_steps(call, args.steps, stream)
            ms = sorted(per)[len(per) // 2]
            res[name] = {"ms": ms, "bytes": nbytes, "gbs": nbytes / (ms / 1e3) / 1e9,
                         "frac": nbytes / (ms / 1e3) / 1e9 / peak}
        print(json.dumps(res))
        return 0
    if args.case == "exchange-local":
        # the Ulysses exchange kernels at the Wan layer (B=2, H=12, S=32768) with
        # the buffers of P=2 ranks on this one GPU: every store lands in local
        # HBM, so this times the kernels against HBM rather than NVLink. A
        # dispatch reads one rank's Q, K, V shards and writes them into both
        # ranks' receive buffers; a combine reads one rank's unit outputs and
        # LSE and writes them into both ranks' output shards.
        import ctypes

        from sinkattn_b200 import _lib
        from sinkattn_b200.sharding import units_per_rank

        P, Sr = 2, S // 2
        n_per = units_per_rank(B * H, P)
        lib = _lib.load()
        g = torch.Generator(device=dev).manual_seed(0)
        shards = [[torch.randn(B, Sr, H, D, generator=g, device=dev, dtype=torch.bfloat16)
                   for _ in range(3)] for _ in range(P)]
        recv = [torch.empty(3, n_per, S, D, dtype=torch.bfloat16, device=dev) for _ in range(P)]
        outs = [torch.randn(n_per, S, D, generator=g, device=dev, dtype=torch.bfloat16)
                for _ in range(P)]
        lses = [torch.randn(n_per, S, generator=g, device=dev) for _ in range(P)]
        out_dst = [torch.empty(B, Sr, H, D, dtype=torch.bfloat16, device=dev) for _ in range(P)]
        lse_dst = [torch.empty(B, H, Sr, device=dev) for _ in range(P)]
        VP = ctypes.c_void_p * P
        dst = VP(*[r.data_ptr() for r in recv])
        od = VP(*[o.data_ptr() for o in out_dst])
        ld = VP(*[o.data_ptr() for o in lse_dst])
        stream = torch.cuda.current_stream(dev)
        sh = ctypes.c_void_p(stream.cuda_stream)

        def dispatch(i):
            q, k, v = shards[i % P]
            src = (ctypes.c_void_p * 3)(q.data_ptr(), k.data_ptr(), v.data_ptr())
            st = (ctypes.c_int64 * 12)(*q.stride(), *k.stride(), *v.stride())
            _lib.check(lib.sa_ulysses_dispatch(3, src, st, B, Sr, H, D, P, i % P, n_per, dst,
                                               sh), "sa_ulysses_dispatch")

        def combine(i):
            r = i % P
            _lib.check(lib.sa_ulysses_combine(outs[r].data_ptr(), lses[r].data_ptr(), B, Sr, H, D,
                                              P, r, n_per, od, ld, sh), "sa_ulysses_combine")

        peak = float(load_peaks()[0].get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
        shard = B * Sr * H * D * 2
        cases = {"dispatch": (dispatch, 2 * 3 * shard),
                 "combine": (combine, 2 * (n_per * S * D * 2 + n_per * S * 4))}
        res = {"case": args.case, "B": B, "H": H, "S": S, "P": P, "peak_gbs": peak}
        for name, (fn, nbytes) in cases.items():
            it = iter(range(1 << 30))
            call = lambda: fn(next(it))  # noqa: E731
            for _ in range(3):
                call()
            torch.cuda.synchronize()
            torch.cuda._sleep(50_000_000)  # queue every timed launch ahead of the device
            _, per = time_steps(call, args.steps, stream)
            ms = sorted(per)[len(per) // 2]
            res[name] = {"ms": ms, "bytes": nbytes, "gbs": nbytes / (ms / 1e3) / 1e9,
                         "frac": nbytes / (ms / 1e3) / 1e9 / peak}
        print(json.dumps(res))
        return 0
    if args.case == "zimage":
        # cfg4 (Z-Image 2048x2048): B=1, H=30, 16384 image + 512 text tokens = 132 blocks;
        # text rows and columns forced dense as the Z-Image processor does
        from tests.gen import zimg_qkv

        q, k, v = zimg_qkv(seed=0, device=dev)
        _, bm = ops.pool_scores(q, k, want_scores=False, want_batch_mean=True)
        cov, _ = ops.coverage_mask(bm, force_sink_col=True)
        nbz = cov.shape[-1]
        t0 = nbz - 4

        def with_text(m):
            m = m.clone()
            m[:, :, t0:] = True
            m[:, t0:, :] = True
            return m.unsqueeze(0).contiguous()

        masks = {"coverage_rule": with_text(cov),
                 "bernoulli_0.2": with_text(cfg1_mask(30, nbz, nbz, seed=1).to(dev))}
        res = {"case": args.case, "B": 1, "H": 30, "S": int(q.shape[2])}
        for name, m in masks.items():
            fn = lambda: ops.bsattn_fwd(q, k, v, m)  # noqa: E731
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            total, _ = time_steps(fn, args.steps, torch.cuda.current_stream(dev))
            ms = total / args.steps
            res[name] = {"density": float(m.float().mean().item()), "ms": ms,
                         "tflops": kept_flops(m) / (ms / 1e3) / 1e12}
        print(json.dumps(res))
        return 0
    if args.case in ("stats-wan", "stats-small"):
        # the exact and max block-statistics modes (dense Q K^T on the tensor cores)
        Bc, Hc = (B, H) if args.case == "stats-wan" else (1, 2)
        q, k, _ = wan_qk(seed=0, B=Bc, H=Hc, dtype=torch.bfloat16, device=dev)
        res = {"case": args.case, "B": Bc, "H": Hc, "S": S}
        # Both modes run Q K^T once (2 D FLOP per (query, key) pair); the
        # exact mode also takes one exponential per pair. `exact_ref_tflops`
        # counts the reference's exact algorithm, which computes Q K^T twice
        # (a maximum sweep, then a mass sweep).
        for mode in ("exact", "max"):
            ws = torch.empty(max(1, ops._lib.load().sa_block_stats_workspace_size(
                Bc, Hc, S, ops._STATS_MODES[mode])), dtype=torch.uint8, device=dev)
            out = torch.empty(Bc, Hc, NB, NB, dtype=torch.float32, device=dev)
            fn = lambda: ops.block_stats(q, k, mode=mode, workspace=ws, out=out)  # noqa: E731
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            total, _ = time_steps(fn, args.steps, torch.cuda.current_stream(dev))
            ms = total / args.steps
            res[mode + "_ms"] = ms
            res[mode + "_mma_tflops"] = 2.0 * S * S * D * Bc * Hc / (ms / 1e3) / 1e12
            if mode == "exact":
                res["exact_ref_tflops"] = 2 * res["exact_mma_tflops"]
                res["exact_gexp_per_s"] = float(S) * S * Bc * Hc / (ms / 1e3) / 1e9
        print(json.dumps(res))
        return 0
    if args.case in ("attn-wan", "calib-wan"):
        # quick timing of one kernel chain at the full Wan shape (no e2e / CPU legs)
        q, k, v = wan_qk(seed=0, dtype=torch.bfloat16, device=dev)
        if args.case == "attn-wan":
            mask = cfg1_mask(H, NB, NB, seed=1).unsqueeze(0).expand(B, -1, -1, -1).contiguous().to(dev)
            flops = kept_flops(mask)
            fn = lambda: ops.bsattn_fwd(q, k, v, mask)  # noqa: E731
        else:
            # one layer's calibration as the product runs it: one fused launch
            ws = torch.empty(ops.pool_scores_workspace_size(B, H, S, D), dtype=torch.uint8, device=dev)
            cm = torch.empty(H, NB, NB, dtype=torch.bool, device=dev)
            flops = 0.0

            def fn():
                ops.calibration_layer(q, k, want_batch_mean=False, mask_out=cm,
                                      force_sink_col=True, workspace=ws)
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        total, per = time_steps(fn, args.steps, torch.cuda.current_stream(dev))
        ms = total / args.steps
        res = {"case": args.case, "ms": ms, "min_ms": min(per)}
        if flops:
            res["tflops"] = flops / (ms / 1e3) / 1e12
        print(json.dumps(res))
        return 0
    if args.case == "attn-small":
        q, k, v = wan_qk(seed=0, B=1, H=6, dtype=torch.bfloat16, device=dev)
        mask = cfg1_mask(6, NB, NB, seed=1).unsqueeze(0).to(dev)
        fn = lambda: ops.bsattn_fwd(q, k, v, mask)  # noqa: E731
    elif args.case == "calib-small":
        q, k, _ = wan_qk(seed=0, B=2, H=4, dtype=torch.bfloat16, device=dev)
        ws = torch.empty(ops.pool_scores_workspace_size(2, 4, S, D), dtype=torch.uint8, device=dev)
        cm = torch.empty(4, NB, NB, dtype=torch.bool, device=dev)

        def fn():
            ops.calibration_layer(q, k, want_batch_mean=False, mask_out=cm, force_sink_col=True,
                                  workspace=ws)
    else:
        raise SystemExit(f"unknown case {args.case}")
    fn()
    torch.cuda.synchronize()
    for _ in range(args.steps):
        fn()
    torch.cuda.synchronize()
    print(json.dumps({"case": args.case, "ok": True}))
    return 0


def run_ulysses(args):
    """The attention layer of the full-DiT config under sequence parallelism:
    each rank holds a [B, S/P, H, D] shard of the Wan-shape Q/K/V, an
    all-to-all turns them into whole-sequence (b, h) units, the kernel runs
    on them and a second all-to-all returns the output (and LSE). Timed with
    the exchange in one group (chunks=1) and overlapped with the kernel in
    groups of units (chunks=C), next to the kernel alone on the rank's units.
    Launch under torchrun with >= 2 processes."""
    world, rank, local = dist_env()
    if world < 2:
        print(json.dumps({"case": "ulysses", "unavailable": "needs torchrun with >= 2 ranks"}))
        return 0
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    init_dist(world, "nccl", dev)
    from sinkattn_b200.sharding import (_local_units_attention, sequence_to_units,
                                        ulysses_sink_attention, units_per_rank)
    from tests.gen import cfg1_mask, wan_qk

    q, k, v = wan_qk(seed=0, dtype=torch.bfloat16, device=dev)  # [B, H, S, D]
    Sr = S // world
    sl = slice(rank * Sr, (rank + 1) * Sr)
    qs, ks, vs = (x.permute(0, 2, 1, 3)[:, sl].contiguous() for x in (q, k, v))
    del q, k, v
    mask = cfg1_mask(H, NB, NB, seed=1).unsqueeze(0).expand(B, -1, -1, -1).contiguous().to(dev)
    n_per = units_per_rank(B * H, world)
    stream = torch.cuda.current_stream(dev)
    res = {"case": "ulysses", "n_gpus": world, "units_per_rank": n_per,
           "exchange_mb_per_rank": 4 * B * Sr * H * D * 2 * (world - 1) / world / 1e6}

    def timed(fn):
        for _ in range(max(3, args.warmup)):
            fn()
        torch.cuda.synchronize()
        barrier(world)
        total, _ = time_steps(fn, args.steps, stream)
        barrier(world)
        return max_over_ranks(total / args.steps, world, dev)

    res["ms_layer"] = {}
    for chunks in sorted({1, min(3, n_per), n_per}):
        res["ms_layer"][chunks] = timed(
            lambda: ulysses_sink_attention(qs, ks, vs, mask, chunks=chunks))
    # the kernel alone on this rank's units (inputs already exchanged)
    units = [sequence_to_units(x) for x in (qs, ks, vs)]
    m = mask.reshape(B * H, NB, NB)
    ids = [rank * n_per + i for i in range(n_per)]
    mu = torch.stack([m[i] if i < B * H else torch.ones_like(m[0]) for i in ids]).contiguous()
    res["ms_attention_only"] = timed(lambda: _local_units_attention(*units, mu, ops_attn))
    if rank == 0:
        print(json.dumps(res))
    import torch.distributed as dist

    dist.destroy_process_group()
    return 0


def ops_attn(q, k, v, m):
    from sinkattn_b200 import ops

    return ops.bsattn_fwd(q, k, v, m)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--skip-cpu", action="store_true", help="omit the CPU baseline leg")
    ap.add_argument("--skip-dit", action="store_true", help="omit the cfg5 full-DiT leg")
    ap.add_argument("--e2e-chunk-heads", type=int, default=1,
                    help="heads per host<->device chunk of the end-to-end leg")
    ap.add_argument("--case", choices=["attn-small", "calib-small", "attn-wan", "calib-wan",
                                       "calib-pass", "wan-runtime", "stats-wan", "stats-small",
                                       "qkrope-wan", "misc-wan", "ulysses", "zimage",
                                       "exchange-local"],
                    default=None,
                    help="run one small profiling case instead of the benchmark")
    args = ap.parse_args(argv)
    if args.case == "ulysses":
        return run_ulysses(args)
    if args.case:
        return run_case(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())

"""Benchmark of the sm_100a attention / KV-cache path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline (`value`): decode-attention HBM GB/s on config 3 -- 64 sequences,
32 query / 8 kv heads, head_dim 128, page 16, context U[1024, 8192] (seed 2),
one fused append + paged GQA decode per step, inputs resident in HBM (the
1.27 GB cache is larger than L2, so no flush is needed).  Algorithmic bytes
per step are counted from the drawn lengths (doe_b200/workloads.py).
Secondary numbers in the same line: config 4 (int8 KV, 32 long sequences),
its 512-token chunk quantise-append, and config 1 (f32 decode).

N > 1 (torchrun, one rank per GPU): every rank runs its own copy of the
workload (sequence-sharded decode needs no collective); NCCL carries only the
barrier and the max-over-ranks of the device times.  `scaling` is "weak".

`e2e` is the same metric through the backend C ABI (doe_cuda_dispatch) with
host buffers: each step writes Q / new K,V / lengths from pinned host memory
and reads the f32 output back.  `cpu_baseline` and `--impl reference` time
the C restatement of the reference's CPU path (oracle/, OpenMP, all host
cores) on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


# the headline metric; both arms (ours and --impl reference) report it
METRIC = "decode-attn HBM GB/s (config 3 paged GQA decode, fused append)"


def clock_max_mhz(index: int = 0):
    """The SM's maximum clock from NVML (None when NVML is unavailable)."""
    try:
        import pynvml

        pynvml.nvmlInit()
        return float(pynvml.nvmlDeviceGetMaxClockInfo(pynvml.nvmlDeviceGetHandleByIndex(index),
                                                      pynvml.NVML_CLOCK_SM))
    except Exception:
        return None


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured"}
    return {"hbm_gbs": FALLBACK_HBM_GBS, "bf16_tflops": FALLBACK_BF16_TFLOPS,
            "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def profiled_traffic() -> dict:
    p = ROOT / "profiles" / "traffic.json"
    return json.loads(p.read_text()) if p.exists() else {}


# ---------------------------------------------------------------------------
class ClockSampler:
    """SM clocks and throttle reasons sampled (NVML, ~2 ms) during a timed region."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap"}

    def __init__(self, index: int):
        import threading

        self.index = index
        self.samples: list[tuple[float, float, int]] = []
        self._stop = threading.Event()
        self._thread = None
        self._nvml = None

    def _run(self):
        nv = self._nvml
        h = nv.nvmlDeviceGetHandleByIndex(self.index)
        mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        while not self._stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.samples.append((float(sm), float(mx), int(reasons)))
            except Exception:
                pass
            self._stop.wait(0.002)

    def start(self):
        import threading

        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
        except Exception:
            self._nvml = None
            return
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()

    def stop(self) -> dict:
        if self._thread is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"]}
        self._stop.set()
        self._thread.join(timeout=5)
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [x[0] for x in self.samples]
        bits = 0
        for x in self.samples:
            bits |= x[2]
        reasons = sorted(n for b, n in self.REASONS.items() if bits & b)
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(x[1] for x in self.samples),
                "reasons": reasons, "samples": len(self.samples), "source": "nvml"}


# ---------------------------------------------------------------------------
def dist_setup():
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    import torch

    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(world, vals: list[float]) -> list[float]:
    import torch

    if world == 1:
        return vals
    import torch.distributed as dist

    t = torch.tensor(vals, dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


L2_FLUSH_NOTE = ("flushed between steps: a 256 MB write, then a 256 MB read of a second buffer, "
                 "so no line of the flush is still dirty in L2 when the timed call starts")


def l2_flusher():
    """A callable that leaves L2 holding none of the timed call's data: it
    writes one buffer larger than L2, then reads a second one, so the flush's
    own dirty lines are written back before the next timed call rather than
    during it."""
    import torch

    a = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    b = torch.zeros(256 << 20, dtype=torch.uint8, device="cuda")
    n = iter(range(1 << 62))

    def flush():
        a.fill_(next(n) & 0xff)
        b.amax()
    return flush


def time_steps(step, steps: int, warmup: int, world: int, flush=None):
    """Device time of `steps` calls: total (ms) and per-call event times (ms).
    With `flush` (a callable that overwrites L2), it runs before every call,
    outside the per-call events, and the total is the sum of those."""
    import torch

    for _ in range(warmup):
        if flush is not None:
            flush()
        step()
    barrier(world)
    stream = torch.cuda.current_stream()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    per = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    # keep the GPU busy (~1 ms per 10 steps) while the host enqueues the timed
    # steps, so host launch gaps never enter the device-timed region
    torch.cuda._sleep(2_000_000 * max(1, (steps + 9) // 10))
    ev0.record(stream)
    for a, b in per:
        if flush is not None:
            flush()
        a.record(stream)
        step()
        b.record(stream)
    ev1.record(stream)
    torch.cuda.synchronize()
    each = [a.elapsed_time(b) for a, b in per]
    total = sum(each) if flush is not None else ev0.elapsed_time(ev1)
    barrier(world)
    return total, each


# ---------------------------------------------------------------------------
def build_paged(w, fill_seed):
    import torch

    from doe_b200 import workloads
    from doe_b200.kv import PagedKVCache

    cache = PagedKVCache(num_pages=w.num_pages, page_size=w.page_size, num_kv_heads=w.num_kv_heads,
                         head_dim=w.head_dim, block_table=w.block_table, kv_dtype=w.kv_dtype)
    workloads.fill_pools(cache, fill_seed)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    dev = dict(q=t(w.q), lens=t(w.seq_lens), nk=t(w.new_k), nv=t(w.new_v))
    dev["out"] = torch.empty((w.num_seqs, w.num_heads, w.head_dim), dtype=torch.float32, device="cuda")
    dev["status"] = torch.zeros(1, dtype=torch.int32, device="cuda")
    return cache, dev


def paged_step_fn(w, cache, dev, split_pages=0):
    from doe_b200 import ops

    def step():
        ops.paged_decode(cache, dev["q"], dev["lens"], w.scale, new_k=dev["nk"], new_v=dev["nv"],
                         out=dev["out"], status=dev["status"], split_pages=split_pages)
    return step


def sharded(make, world, rank):
    """This rank's shard of the global batch: `world` copies of the config
    (seeds s, s+1, ...) split by sequence with LPT on token counts."""
    from doe_b200 import shard, workloads

    if world == 1:
        w = make(0)
        return w, w
    gw = workloads.concat([make(r) for r in range(world)])
    mine = shard.lpt_assign(gw.seq_lens, world)[rank]
    return workloads.subset(gw, mine), gw


def strong_split(w, world, rank):
    """This rank's shard of ONE batch split by sequence over `world` ranks
    (LPT on token counts): the same sequences on more GPUs, strong scaling."""
    from doe_b200 import shard, workloads

    if world == 1:
        return w, w
    return workloads.subset(w, shard.lpt_assign(w.seq_lens, world)[rank]), w


def measure_paged(w, fill_seed, steps, warmup, world, pk, split_pages=0, gw=None):
    gw = gw if gw is not None else w
    cache, dev = build_paged(w, fill_seed)
    step = paged_step_fn(w, cache, dev, split_pages)
    total, each = time_steps(step, steps, warmup, world)
    kern_local = float(np.mean(each))
    total, kern = max_over_ranks(world, [total, kern_local])
    assert int(dev["status"].item()) == 0, f"device status {int(dev['status'].item()):#x}"
    sb = w.step_bytes()
    res = {
        "ms_per_step": total / steps,
        "gbs": gw.step_bytes()["total"] * steps / (total / 1e3) / 1e9,
        "tokens_per_s": gw.tokens_per_step() * steps / (total / 1e3),
        "kernel_ms": kern_local,
        "kernel_gbs": sb["total"] / (kern_local / 1e3) / 1e9,
        "bytes_per_step": sb,
        "global_bytes_per_step": gw.step_bytes()["total"],
        "sequences_this_rank": w.num_seqs,
    }
    res["frac"] = res["kernel_gbs"] / pk["hbm_gbs"]
    return res, cache, dev


def measure_chunk_append(w, cache, steps, warmup, world, pk, chunk=512, gw=None):
    import torch

    from doe_b200 import ops

    g = np.random.default_rng(w.seed + 100)
    nk = g.standard_normal((w.num_seqs, chunk, w.num_kv_heads, w.head_dim), dtype=np.float32).astype(np.float16)
    nv = g.standard_normal((w.num_seqs, chunk, w.num_kv_heads, w.head_dim), dtype=np.float32).astype(np.float16)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    nk, nv = t(nk), t(nv)
    pos = t((w.ctx + 1).astype(np.int32))  # after the decode token
    status = torch.zeros(1, dtype=torch.int32, device="cuda")

    def step():
        ops.paged_append(cache, nk, nv, pos, status=status)
    # the chunk's 67 MB of input and 34 MB of output fit in L2 together: flush
    # it between calls so that every call reads and writes HBM
    total, each = time_steps(step, steps, warmup, world, flush=l2_flusher())
    local_ms = total
    total, = max_over_ranks(world, [total])
    assert int(status.item()) == 0
    def nbytes(seqs):
        rows = seqs * chunk * w.num_kv_heads
        return 2 * rows * w.head_dim * 2 + seqs * 4 + 2 * rows * (w.head_dim + 2)

    gw = gw if gw is not None else w
    job = nbytes(gw.num_seqs) * (world if gw is w else 1)
    return {"ms_per_step": total / steps, "gbs": job * steps / (total / 1e3) / 1e9,
            "bytes_per_step": nbytes(w.num_seqs), "job_bytes_per_step": job,
            "frac": nbytes(w.num_seqs) * steps / (local_ms / 1e3) / 1e9 / pk["hbm_gbs"],
            "l2": L2_FLUSH_NOTE}


def measure_f32(steps, warmup, world, pk):
    import torch

    from doe_b200 import ops, workloads

    d = workloads.decode_f32()
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    q, k, v = t(d.q), t(d.k), t(d.v)
    out = torch.empty_like(q)
    # flush L2 between iterations: the 2 MB problem would otherwise sit in L2
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    times = []
    for i in range(warmup + steps):
        flush.fill_(i & 0xff)
        # keep the GPU busy while the host enqueues the timed launches, so the
        # events bracket device time rather than host launch latency
        torch.cuda._sleep(200_000)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        ops.attention_decode_f32(q, k, v, d.scale, out=out)
        b.record()
        torch.cuda.synchronize()
        if i >= warmup:
            times.append(a.elapsed_time(b))
    ms, = max_over_ranks(world, [float(np.mean(times))])
    return {"us_per_step": ms * 1e3, "gbs": world * d.bytes_per_step / (ms / 1e3) / 1e9,
            "bytes_per_step": d.bytes_per_step, "l2": "flushed (256 MB write) between steps"}


def measure_ep(steps, warmup, world, pk):
    """The ORT EP's basic f32 operators at HBM-sized shapes (inputs + outputs
    larger than L2): Softmax and LayerNorm over [8192, 4096], Gelu over 64 Mi
    elements, Add over 32 Mi, and a 4096^3 MatMul against the FP32 pipe's
    nominal peak (SMs x 128 lanes x 2 flop x max SM clock)."""
    import torch

    from doe_b200 import ort_ep

    g = torch.Generator(device="cuda").manual_seed(6)
    rnd = lambda *shape: torch.randn(*shape, device="cuda", generator=g)
    x = rnd(8192, 4096)
    scale = rnd(4096)
    u = rnd(64 << 20)
    a2, b2 = rnd(32 << 20), rnd(32 << 20)
    ma, mb = rnd(4096, 4096), rnd(4096, 4096)
    cases = {
        "softmax": (lambda: ort_ep.execute("softmax", x), 2 * x.numel() * 4, None),
        "layernorm": (lambda: ort_ep.execute("layernorm", x, scale), 2 * x.numel() * 4, None),
        "gelu": (lambda: ort_ep.execute("gelu", u), 2 * u.numel() * 4, None),
        "add": (lambda: ort_ep.execute("add", a2, b2), 3 * a2.numel() * 4, None),
        "matmul": (lambda: ort_ep.execute("matmul", ma, mb), 3 * 4096 * 4096 * 4, 2 * 4096 ** 3),
    }
    props = torch.cuda.get_device_properties(0)
    clk = clock_max_mhz() or 1965.0
    fp32_peak = props.multi_processor_count * 128 * 2 * clk * 1e6 / 1e12
    out = {"config": "ORT EP basic f32 ops: softmax / layernorm [8192, 4096], gelu 64Mi, add 32Mi, "
                     "matmul 4096^3", "l2": "each step's inputs + outputs exceed L2"}
    for name, (fn, nbytes, flops) in cases.items():
        times = []
        for i in range(warmup + steps):
            ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            # keep the GPU busy while the host validates, allocates and
            # enqueues, so the events bracket device time only
            torch.cuda._sleep(1_000_000)
            ev[0].record()
            fn()
            ev[1].record()
            torch.cuda.synchronize()
            if i >= warmup:
                times.append(ev[0].elapsed_time(ev[1]))
        ms, = max_over_ranks(world, [float(np.mean(times))])
        r = {"ms": ms, "gbs": nbytes / (ms / 1e3) / 1e9}
        r["hbm_frac"] = r["gbs"] / pk["hbm_gbs"]
        if flops:
            r["tflops"] = flops / (ms / 1e3) / 1e12
            r["fp32_frac"] = r["tflops"] / fp32_peak
            r["fp32_peak_tflops"] = fp32_peak
        out[name] = r
    return out


def measure_prefill(steps, warmup, world, pk, rank=0):
    """Config 2: causal prefill (tcgen05) incl. the fused paged KV-cache write.

    With N ranks the prompt is sharded by KV head (each rank takes Hkv/N KV
    heads and their query heads; outputs and cache stay head-sharded, no
    collective): the same prompt on more GPUs, strong scaling."""
    import torch

    from doe_b200 import ops, workloads
    from doe_b200.kv import PagedKVCache

    w = workloads.prefill_f16()
    S = w.q.shape[0]
    H, Hkv = w.q.shape[1], w.k.shape[1]
    if Hkv % world:
        raise ValueError(f"{world} ranks do not divide {Hkv} KV heads")
    kvh, qh = Hkv // world, H // world
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    q = t(w.q[:, rank * qh:(rank + 1) * qh])
    k, v = t(w.k[:, rank * kvh:(rank + 1) * kvh]), t(w.v[:, rank * kvh:(rank + 1) * kvh])
    out = torch.empty((S, qh, 128), dtype=torch.float32, device="cuda")
    cache = PagedKVCache(num_pages=S // 16, page_size=16, num_kv_heads=kvh, head_dim=128,
                         block_table=np.arange(S // 16, dtype=np.int32)[None])
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    flush = l2_flusher()
    times = []
    for i in range(warmup + steps):
        flush()  # 48 MB of inputs + outputs would otherwise stay in L2
        torch.cuda._sleep(200_000)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        ops.attention_prefill_f16(q, k, v, w.scale, cache=cache, out=out, status=status)
        b.record()
        torch.cuda.synchronize()
        if i >= warmup:
            times.append(a.elapsed_time(b))
    assert int(status.item()) == 0, f"prefill status {int(status.item()):#x}"
    ms, = max_over_ranks(world, [float(np.mean(times))])
    tflops = w.flops / (ms / 1e3) / 1e12  # the whole prompt's flops over the slowest rank's time
    return {"config": "config 2: causal prefill S 2048, 32 heads, D 128, f16 in / f32 acc, seed 1, "
                      "+ paged KV-cache write", "ms": ms, "tflops": tflops,
            "parallelism": f"{world} ranks by KV head ({kvh} KV heads each)" if world > 1 else "one GPU",
            "scaling": "strong" if world > 1 else None,
            "frac_of_dense_peak": tflops / world / pk["bf16_tflops"], "flops": w.flops,
            "peak_tflops": pk["bf16_tflops"], "peak_note": "measured dense bf16 burst (f16 runs at the same rate)",
            "l2": L2_FLUSH_NOTE}


def kernel_shares(replay, world, rank, reps=5):
    """Device time per kernel name over `reps` replays, from the CUDA activity
    records of torch.profiler on rank 0 (the other ranks replay alongside).
    Shares only: times taken under a tracer are not bench values."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    barrier(world)
    if rank == 0:
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            for _ in range(reps):
                replay()
            torch.cuda.synchronize()
    else:
        for _ in range(reps):
            replay()
        torch.cuda.synchronize()
    barrier(world)
    if rank != 0:
        return None
    tot = {}
    for e in prof.key_averages():
        t = getattr(e, "device_time_total", None)
        if t is None:
            t = getattr(e, "cuda_time_total", 0.0)
        if t > 0:
            tot[e.key] = tot.get(e.key, 0.0) + t
    allt = sum(tot.values()) or 1.0
    top = sorted(tot.items(), key=lambda kv: -kv[1])[:8]
    return {"per_step_us": {k[:60]: round(v / reps, 2) for k, v in top},
            "share": {k[:60]: round(v / allt, 4) for k, v in top},
            "how": f"torch.profiler CUDA activity on rank 0 over {reps} graph replays (shares only)"}


def measure_decoder(steps, warmup, world, rank, pk, shares=False):
    """Config 5: the 4-layer bf16 decoder step (batch 32, ctx 4096), tensor
    parallel by KV head over the `world` ranks, captured in a CUDA graph."""
    import torch

    from doe_b200 import decoder

    cfg = decoder.DecoderConfig()
    dec = decoder.Decoder(cfg, seed=4, rank=rank, world=world)
    x0 = torch.from_numpy(np.random.default_rng(4).standard_normal((cfg.batch, cfg.hidden),
                                                                   dtype=np.float32)).cuda()
    x = x0.clone()
    dec.step(x)  # eager warm-up: NCCL, workspaces, tensor maps
    torch.cuda.synchronize()
    x.copy_(x0)
    dec.capture(x)
    launches = dec.launches_per_step()
    reduction = ("reduction fused into the RMSNorm over peer buffers (doe_tp_reduce_rmsnorm)"
                 if dec.peers is not None else "NCCL all-reduce")
    try:
        total, each = time_steps(dec.replay, steps, warmup, world)
        total = max_over_ranks(world, [total])[0]
        status = int(dec.status.item())
        finite = bool(torch.isfinite(x).all().item())
        ks = kernel_shares(dec.replay, world, rank) if shares else None
    finally:
        dec.release()
    ms = total / steps
    job_bytes = cfg.weight_bytes() + cfg.kv_read_bytes()
    rank_bytes = job_bytes / world
    return {"config": "config 5: 4-layer Llama-style decoder, hidden 4096, 32/8 heads, FFN 14336 SwiGLU, "
                      "bf16 weights N(0,0.02) seed 4, batch 32 at ctx 4096, f16 paged KV",
            "parallelism": f"tp{world} by KV head, {reduction} after o_proj and down_proj"
                           if world > 1 else "tp1",
            "scaling": "strong", "ms_per_step": ms, "tokens_per_s": cfg.batch / (ms / 1e3),
            "bytes_per_step": job_bytes, "gbs": job_bytes / (ms / 1e3) / 1e9,
            "per_gpu_frac": rank_bytes / (ms / 1e3) / 1e9 / pk["hbm_gbs"],
            "gpu_launches_per_step": launches, "graph": "one CUDA graph per step",
            "status": status, "output_finite": finite,
            **({"kernel_shares": ks} if ks is not None else {})}


LINEAR_SHAPES = {  # config 5's products at tp1: (n_out, k, SwiGLU)
    "qkv": (6144, 4096, False), "o_proj": (4096, 4096, False), "gate_up": (28672, 4096, True),
    "down_proj": (4096, 14336, False)}


def measure_linear(steps, warmup, world, pk, only=None):
    """doe_linear_bf16 on config 5's shapes (batch 32): each step one product,
    weights rotating over copies that together exceed L2."""
    import torch

    from doe_b200 import ops

    out = {}
    for name, (n, k, swiglu) in LINEAR_SHAPES.items():
        if only and name != only:
            continue
        copies = max(2, (300 << 20) // (n * k * 2) + 1)
        g = torch.Generator(device="cuda")
        g.manual_seed(5)
        ws = [(torch.randn((n, k), generator=g, device="cuda") * 0.02).to(torch.bfloat16) for _ in range(copies)]
        x = torch.randn((32, k), generator=g, device="cuda").to(torch.bfloat16)
        y = torch.empty((32, n // 2 if swiglu else n), dtype=torch.bfloat16, device="cuda")
        lws = ops.linear_workspace(n, k)
        it = iter(range(10 ** 9))
        total, each = time_steps(lambda: ops.linear(x, ws[next(it) % copies], [y], swiglu=swiglu, ws=lws),
                                 steps, warmup, world)
        total = max_over_ranks(world, [total])[0]
        us = total / steps * 1e3
        nbytes = n * k * 2 + 32 * k * 2 + y.numel() * 2
        out[name] = {"n_out": n, "k": k, "swiglu": swiglu, "us": us, "gbs": nbytes / us / 1e3,
                     "frac": nbytes / us / 1e3 / pk["hbm_gbs"]}
        del ws
        torch.cuda.empty_cache()
    return out


def measure_e2e(w, cache, steps, warmup, world, gw=None):
    """Same decode step through doe_cuda_dispatch with host buffers."""
    gw = gw if gw is not None else w
    import ctypes as C

    import torch

    from doe_b200.backend import Bind, CudaBackend

    be = CudaBackend(torch.cuda.current_device())
    # cache state lives on the device: upload the pools once (not timed)
    chunk = 64 << 20
    for h, pool in ((2, cache.k_pool), (3, cache.v_pool)):
        host = pool.cpu().numpy().view(np.uint8).reshape(-1)
        be.ensure_buffer(h, host.nbytes)
        for o in range(0, host.nbytes, chunk):
            be.execute_buffer_write_bytes(h, o, host[o:o + chunk])
    be.execute_buffer_write_bytes(4, 0, w.block_table)
    uni = np.array([w.num_seqs, w.num_heads, w.num_kv_heads, w.head_dim, w.page_size, w.num_pages,
                    w.block_table.shape[1], 0, np.float32(w.scale).view(np.uint32), 0], np.uint32)
    be.execute_buffer_write_bytes(1, 0, uni)
    be.flush_queue()
    # pinned host inputs / output
    pin = lambda a: torch.from_numpy(np.ascontiguousarray(a)).pin_memory()
    hq, hl, hk, hv = pin(w.q.view(np.uint16)), pin(w.seq_lens), pin(w.new_k.view(np.uint16)), pin(w.new_v.view(np.uint16))
    hout = torch.empty((w.num_seqs, w.num_heads, w.head_dim), dtype=torch.float32).pin_memory()
    out_bytes = hout.numel() * 4
    # two sets of per-step buffers (handles 10-14 and 20-24), alternating:
    # the backend orders each buffer's copies and kernels with events, so step
    # i + 1's uploads overlap step i's kernel and step i's capture overlaps
    # step i + 1's kernel
    binds = [[Bind(0, 1, size=40), Bind(1, 10 + o), Bind(2, 2), Bind(3, 3), Bind(4, 4), Bind(5, 11 + o),
              Bind(6, 12 + o, size=out_bytes), Bind(7, 13 + o), Bind(8, 14 + o)] for o in (0, 10)]
    h2d = hq.numel() * 2 + hl.numel() * 4 + hk.numel() * 2 + hv.numel() * 2
    parity = [0]

    def step():
        o = 10 * parity[0]
        be.write_ptr_async(10 + o, 0, hq.data_ptr(), hq.numel() * 2)
        be.write_ptr_async(11 + o, 0, hl.data_ptr(), hl.numel() * 4)
        be.write_ptr_async(13 + o, 0, hk.data_ptr(), hk.numel() * 2)
        be.write_ptr_async(14 + o, 0, hv.data_ptr(), hv.numel() * 2)
        be.execute_kernel_dispatch("attention_paged_decode", binds[parity[0]])
        # deferred capture: the host queues the next step while this one runs
        be.read_into_async(12 + o, 0, hout.data_ptr(), out_bytes)
        parity[0] ^= 1

    for _ in range(warmup):
        step()
    be.flush_queue()
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    enqueued = time.perf_counter() - t0
    be.flush_queue()
    elapsed = time.perf_counter() - t0
    elapsed, = max_over_ranks(world, [elapsed])
    be.close()
    # the e2e output must equal the operator path's output on the same inputs:
    # the same kernel and split plan, splits stitched in split order, so the
    # bits agree
    from doe_b200 import ops

    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    ref = ops.paged_decode(cache, t(w.q), t(w.seq_lens), w.scale, new_k=t(w.new_k), new_v=t(w.new_v))
    torch.cuda.synchronize()
    ok = bool(np.array_equal(hout.numpy(), ref.cpu().numpy()))
    if not ok:
        raise RuntimeError("e2e: the doe_cuda_dispatch output differs from the operator path's output")
    sb = gw.step_bytes()["total"]
    return {"value": sb * steps / elapsed / 1e9, "unit": "GB/s",
            "tokens_per_s": gw.tokens_per_step() * steps / elapsed,
            "ms_per_step": elapsed / steps * 1e3, "host_enqueue_ms_per_step": enqueued / steps * 1e3,
            "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": int(out_bytes),
            "timer": "host perf_counter around K steps (each step: 4 deferred H2D writes from pinned memory, "
                     "dispatch, deferred D2H capture, alternating two buffer sets; one flush at the end)",
            "output_equals_operator_path": ok}


# ---------------------------------------------------------------------------
_CPU_POOLS: dict = {}


def _cpu_pools(w, nseq: int):
    """Host pools for the first `nseq` sequences of `w`, pages renumbered densely
    (seeded N(0,1) f16 K/V, or int8 with f16 scales), cached per workload."""
    import oracle

    key = (w.name, w.seed, nseq)
    if key in _CPU_POOLS:
        return _CPU_POOLS[key]
    rng = np.random.default_rng(w.seed + 7)
    sel = np.arange(nseq)
    pages = [w.block_table[b][w.block_table[b] >= 0] for b in sel]
    npg = sum(len(p) for p in pages)
    table = np.full((nseq, w.block_table.shape[1]), -1, np.int32)
    o = 0
    for i, p in enumerate(pages):
        table[i, :len(p)] = np.arange(o, o + len(p))
        o += len(p)
    shape = (npg * w.page_size, w.num_kv_heads, w.head_dim)
    if w.kv_dtype == "f16":
        def pool():
            out = np.empty(shape, np.uint16)
            flat = out.reshape(shape[0], -1)
            for r0 in range(0, shape[0], 1 << 16):
                flat[r0:r0 + (1 << 16)] = rng.standard_normal(
                    flat[r0:r0 + (1 << 16)].shape, dtype=np.float32).astype(np.float16).view(np.uint16)
            return out
        kp, vp, ks, vs = pool(), pool(), None, None
    else:
        kp = rng.integers(-127, 128, shape, dtype=np.int8)
        vp = rng.integers(-127, 128, shape, dtype=np.int8)
        ks = oracle.f2h(np.full((npg, w.num_kv_heads, w.page_size), 0.01, np.float32))
        vs = ks.copy()
    _CPU_POOLS[key] = (table, kp, vp, ks, vs)
    return _CPU_POOLS[key]


def cpu_sample(w, target_s: float = 12.0, max_seqs: int | None = None):
    """Time the reference's CPU path (the C port of it) on the host's cores:
    the fused append + paged decode of the workload's sequences, repeated for
    about `target_s` seconds.  Returns GB/s of KV + Q/O bytes per pass.

    The timed code is oracle/cpu_baseline.c (OpenMP over (sequence, kv head),
    -O3 with AVX2 / F16C, the parity oracle's float order, bit-identical to
    it) when the CPU has AVX2 and F16C, else the parity oracle itself."""
    import oracle

    nseq = w.num_seqs if max_seqs is None else min(max_seqs, w.num_seqs)
    table, kp, vp, ks, vs = _cpu_pools(w, nseq)
    sel = np.arange(nseq)
    lens = w.seq_lens[sel]
    threads = os.cpu_count() or 1
    fast = oracle.fast_decode_available()
    decode = oracle.cpu_paged_decode if fast else oracle.paged_decode

    def one_pass():
        oracle.paged_append(w.new_k[sel][:, None].view(np.uint16), w.new_v[sel][:, None].view(np.uint16),
                            kp, vp, table, w.ctx[sel].astype(np.int32), page_size=w.page_size,
                            k_scale=ks, v_scale=vs, threads=threads)
        decode(w.q[sel].view(np.uint16), kp, vp, table, lens, w.scale, page_size=w.page_size, k_scale=ks,
               v_scale=vs, threads=threads)

    t0 = time.perf_counter()
    one_pass()
    first = time.perf_counter() - t0
    reps = int(max(1, min(200, target_s / max(first, 1e-3))))
    t0 = time.perf_counter()
    for _ in range(reps):
        one_pass()
    dt = (time.perf_counter() - t0) / reps
    nbytes = int(lens.sum()) * w.kv_bytes_per_token() + nseq * (w.num_heads * w.head_dim * 6)
    build = ("oracle/cpu_baseline.c (-O3 -mavx2 -mf16c -fopenmp, -ffp-contract=off, bit-identical to the "
             "parity oracle)" if fast else "oracle/doe_oracle.c (parity oracle, -O2 -fopenmp)")
    return {"value": nbytes / dt / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "cpu": oracle.cpu_model(), "build": build,
            "sample": f"all {nseq} of {w.num_seqs} sequences of {w.name} (fused append + decode), "
                      f"{reps} passes of {dt:.3f} s",
            "tokens_per_s": nseq / dt, "seconds": dt}


def run_reference(args):
    """--impl reference: the reference's CPU path (oracle port) on the same config/metric."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from doe_b200 import workloads

    w = workloads.paged_f16()
    vals = []
    for _ in range(args.warmup):
        cpu_sample(w, target_s=1.0)
    samples = []
    for _ in range(args.steps):
        s = cpu_sample(w, target_s=3.0)
        vals.append(s["value"])
        samples.append(s)
    v = float(np.mean(vals))
    line = {
        "impl": "reference", "metric": METRIC,
        "value": v, "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": float(np.mean([s["seconds"] for s in samples]) * 1e3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded)", "config": config_block(w),
        "tokens_per_s": float(np.mean([s["tokens_per_s"] for s in samples])),
        "cpu_baseline": {"value": v, "unit": "GB/s", "cores": samples[0]["cores"], "kind": "port",
                         "cpu": samples[0]["cpu"], "build": samples[0]["build"],
                         "sample": samples[0]["sample"]},
        "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference's attention runs through Vulkan/Metal (unavailable on this box) and "
                "its Zig host path cannot be built here; this is the C restatement of its CPU path",
    }
    print(json.dumps(line))


def config_block(w) -> dict:
    return {"workload": "config 3: paged GQA decode with fused append, 64 seqs, 32/8 heads, D 128, "
                        "page 16, ctx U[1024,8192] seed 2, f16 KV",
            "num_seqs": w.num_seqs, "num_heads": w.num_heads, "num_kv_heads": w.num_kv_heads,
            "head_dim": w.head_dim, "page_size": w.page_size, "tokens_in_cache": int(w.ctx.sum()),
            "pages": w.num_pages, "l2": "inputs larger than L2 (1.27 GB KV per step)",
            "parallelism": "N copies of the config (seeds 2..) sharded by sequence (LPT on tokens), "
                           "no data collective"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-extras", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--only", choices=["all", "headline", "prefill", "f32", "int8", "append", "decoder",
                                       "linear", "ep"],
                    default="all",
                    help="time one workload only (no e2e or CPU leg): headline = config 3, "
                         "append = config 4b chunk quantise-append, decoder = config 5, "
                         "linear = config 5's products one at a time")
    ap.add_argument("--linear-shape", choices=sorted(LINEAR_SHAPES), default=None,
                    help="with --only linear: time this product alone")
    ap.add_argument("--split-pages", type=int, default=0,
                    help="pages per split of the paged decode (0 = the library's choice)")
    ap.add_argument("--kernel-shares", action="store_true",
                    help="with --only decoder: per-kernel device-time shares of the step on rank 0 "
                         "(torch.profiler CUDA activity)")
    ap.add_argument("--seqs", type=int, default=0,
                    help="override the number of sequences (smaller cases for ncu captures)")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
        return
    args.warmup = max(args.warmup, 3)

    import torch

    world, rank, local = dist_setup()
    pk = peaks()
    from doe_b200 import workloads

    if args.only in ("prefill", "f32", "int8", "append", "decoder", "linear", "ep"):
        if args.only == "ep":
            r = measure_ep(args.steps, args.warmup, world, pk)
        elif args.only == "linear":
            r = measure_linear(args.steps, args.warmup, world, pk, args.linear_shape)
        elif args.only == "decoder":
            r = measure_decoder(args.steps, args.warmup, world, rank, pk, shares=args.kernel_shares)
        elif args.only == "prefill":
            r = measure_prefill(args.steps, args.warmup, world, pk, rank)
        elif args.only == "f32":
            r = measure_f32(args.steps, args.warmup, world, pk)
        elif args.only == "append":
            w4, g4 = strong_split(workloads.paged_int8(num_seqs=args.seqs or 32), world, rank)
            cache4, _ = build_paged(w4, 3)
            r = {"config": "config 4b: 32 x 512 tokens quantised into the paged cache",
                 "scaling": "strong" if world > 1 else None,
                 **measure_chunk_append(w4, cache4, args.steps, args.warmup, world, pk, gw=g4)}
        else:
            w4, g4 = strong_split(workloads.paged_int8(num_seqs=args.seqs or 32), world, rank)
            r, _, _ = measure_paged(w4, 3, args.steps, args.warmup, world, pk, args.split_pages, g4)
            r = {"config": "config 4: 32 seqs, ctx U[8192,32768] seed 3, int8 KV + f16 scales",
                 "scaling": "strong" if world > 1 else None,
                 "parallelism": f"the 32 sequences split over {world} ranks (LPT on tokens)", **r}
        if rank == 0:
            print(json.dumps({"only": args.only, **r}))
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return
    w, gw = sharded(lambda r: workloads.paged_f16(seed=2 + r, num_seqs=args.seqs or 64), world, rank)
    if args.only == "headline":
        args.no_extras = args.no_cpu = True
    clocks = ClockSampler(local)
    clocks.start()
    head, cache, dev = measure_paged(w, 2, args.steps, args.warmup, world, pk, args.split_pages, gw)
    clk = clocks.stop()
    del cache, dev
    torch.cuda.empty_cache()

    extras = {}
    if not args.no_extras:
        # config 4 as BASELINE.json states it: the same 32 sequences split by
        # sequence over the N GPUs (strong scaling)
        w4, g4 = strong_split(workloads.paged_int8(), world, rank)
        r4, cache4, _ = measure_paged(w4, 3, max(5, args.steps // 2), 3, world, pk, 0, g4)
        ca = measure_chunk_append(w4, cache4, 5, 3, world, pk, gw=g4)
        del cache4
        torch.cuda.empty_cache()
        par4 = (f"the 32 sequences split over {world} ranks (LPT on tokens, {w4.num_seqs} on rank 0)"
                if world > 1 else "one GPU")
        extras["int8_decode"] = {"config": "config 4: 32 seqs, ctx U[8192,32768] seed 3, int8 KV + f16 scales",
                                 "parallelism": par4, "scaling": "strong" if world > 1 else None,
                                 "gbs": r4["gbs"], "tokens_per_s": r4["tokens_per_s"],
                                 "ms_per_step": r4["ms_per_step"], "kernel_frac": r4["frac"],
                                 "bytes_per_step": r4["global_bytes_per_step"]}
        extras["int8_chunk_append"] = {"config": "config 4b: 32 x 512 tokens quantised into the paged cache",
                                       "parallelism": par4, "scaling": "strong" if world > 1 else None,
                                       **ca}
        extras["f32_decode"] = {"config": "config 1: 8 heads, D 64, 512 tokens, f32", **measure_f32(20, 5, world, pk)}
        try:
            extras["prefill"] = measure_prefill(10, 3, world, pk, rank)
        except Exception as e:  # reported, never hidden
            extras["prefill"] = {"error": str(e)[:300]}
        torch.cuda.empty_cache()
        extras["decoder"] = measure_decoder(10, 3, world, rank, pk)
        torch.cuda.empty_cache()
        try:
            extras["ort_ep"] = measure_ep(5, 3, world, pk)
        except Exception as e:  # reported, never hidden
            extras["ort_ep"] = {"error": str(e)[:300]}
        torch.cuda.empty_cache()

    e2e = None
    if args.only == "all":
        cache, dev = build_paged(w, 2)
        e2e = measure_e2e(w, cache, max(20, args.steps), 3, world, gw)
        del cache, dev

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_sample(w)

    traffic = profiled_traffic().get("paged_decode_f16")
    roof = {"bound": "hbm", "achieved": head["kernel_gbs"], "peak": pk["hbm_gbs"], "unit": "GB/s",
            "frac": head["frac"], "traffic": traffic,
            "kernel": "paged_decode_kernel<f16,4> (one launch per doe_paged_decode call, split stitch fused)",
            "peak_source": pk["source"] + " (MEASURED_PEAKS.json hbm_gbs, burst copy)",
            "algorithmic_bytes_per_launch": head["bytes_per_step"]["total"]}
    if rank == 0:
        line = {
            "metric": METRIC,
            "value": head["gbs"], "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic (seeded)",
            "config": config_block(gw), "tokens_per_s": head["tokens_per_s"],
            "roofline": roof, "clocks": clk, "e2e": e2e,
            "gpu_launches": args.steps,  # one paged_decode_kernel per step (plus a 2 KB counter memset)
            "cpu_baseline": cpu, **extras,
        }
        print(json.dumps(line))
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()

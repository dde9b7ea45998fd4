#!/usr/bin/env python
"""Benchmark of the ntops LLM operator hot path on B200.

Headline (one JSON line on rank 0): the Llama-3-8B decoder-layer op chain (
bf16, x [16, 2048, 4096], random-init weights ~N(0, 0.02), synthetic data) in tokens/s,
whole-job over N GPUs.  The 16 sequences are sharded over the ranks (strong scaling: the
global batch stays 16 at every N), one process per GPU, no collective on the data path; NCCL is
used only for barriers, the max-over-ranks timing reduction and gathering outputs to check them.

Measured quantities:
  value      tokens/s with inputs resident in HBM, timed with CUDA events over K steps (each step
             one CUDA-graph replay of the layer pass's 7 kernel launches);
  e2e        the same through the public API with the step's input copied from pinned host
             memory and its output copied back inside the timed region (double-buffered copy
             streams, one graph replay per step), with the copy and compute legs timed apart;
  roofline   the fused gate/up (SwiGLU) GEMM, the dominant kernel: algorithmic 2*M*N*K FLOPs per
             launch over its CUDA-event time, against the measured burst bf16 peak
             (MEASURED_PEAKS.json; the sustained-peak fraction is printed beside it);
  ops        N = 1: each BASELINE per-op configuration timed alone (GB/s or TFLOP/s and the
             fraction of the measured HBM copy / burst bf16 peak), each with PyTorch's CPU
             implementation of the same op timed on the host cores beside it;
             N > 1: the configurations BASELINE shards (config 4 by rows, config 5 by
             batch x heads and by M rows) run sharded over the ranks, whole-job throughput from
             the max-over-ranks time, outputs all-gathered over NCCL and compared with one
             unsharded launch on rank 0;
  cpu_baseline (N = 1, rank 0) PyTorch's CPU implementation of the same chain on a bounded
             sample (one sequence prefix), all host threads, warmed, median of several passes.

``--impl reference`` times the reference side of the comparison: the reference's kernels need
``ninetoothed`` (not installable here), so the arm runs the chain on PyTorch's CPU operators —
the oracle the reference's tests use — on the host cores, same metric and config.  That arm
imports nothing from ``ntops_b200`` (its process never loads the kernel library).
"""

import argparse
import datetime
import json
import os
import statistics
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

import torch  # noqa: E402

METRIC = "Llama-8B layer-chain tokens/s"
UNIT = "tokens/s"
GLOBAL_BATCH = 16
SEQ = 2048
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# DRAM bytes (read + write) of one launch of the fused gate/up (SwiGLU) projection at the full
# chain size: ncu dram__bytes_read.sum 5.720481 GB + dram__bytes_write.sum 0.931596 GB with A
# loaded evict-last (profiles/gemm_tc_pair_kernel-swiglu_32768x28672x4096_bf16.md).
SWIGLU_GEMM_TRAFFIC = 6_652_076_800


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return {k: float(d[k]) for k in FALLBACK_PEAKS}, "measured (MEASURED_PEAKS.json)"
    except Exception:
        return dict(FALLBACK_PEAKS), "fallback (profiling recipe)"


def config(world, global_batch=GLOBAL_BATCH):
    return {
        "workload": "llama3_8b_layer_chain (BASELINE config 3): rms_norm, q/k/v mm, rope, causal GQA sdpa, "
        "o mm, residual add, rms_norm, gate/up mm, silu*mul, down mm",
        "global_batch": global_batch,
        "seq_len": SEQ,
        "parallelism": f"dp{world} (sequences sharded, no data-path collective)",
        "l2": "inputs larger than L2 (x 268 MB + weights 436 MB per pass)",
        "fusions": "q/k/v projections + RoPE as one tcgen05 GEMM with a RoPE epilogue; gate/up projections + "
                   "silu*mul as one tcgen05 GEMM with a SwiGLU epilogue",
    }


# ------------------------------------------------------------------------- clocks ---------
class ClockSampler:
    """Samples SM clock and clock-event reasons with NVML every 20 ms (read-only)."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
        0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, index):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nv = None

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for bit, name in self.REASONS.items():
                    if r & bit and bit != 0x1:
                        self.reasons.add(name)
            except Exception:
                pass
            self._stop.wait(0.02)

    def __enter__(self):
        if self._nv is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self):
        return {
            "sm_mhz": statistics.median(self.samples) if self.samples else None,
            "sm_max_mhz": self.max_mhz,
            "reasons": sorted(self.reasons),
            "samples": len(self.samples),
        }


# ---------------------------------------------------------------------- CPU chain ---------
class CpuChain:
    """PyTorch's CPU implementation of the layer chain (oracle/chain.py:layer_forward_torch_cpu)
    on one sequence, weights built once; ``time(tokens)`` runs one pass over a prefix."""

    def __init__(self, threads=None):
        from oracle import chain as OC

        self.OC = OC
        self.threads = threads or host_threads()
        torch.set_num_threads(self.threads)
        g = torch.Generator().manual_seed(0)
        self.w = OC.random_weights(g)
        self.sin, self.cos = OC.rope_tables(SEQ)
        self.x = torch.randn((1, SEQ, OC.HIDDEN), generator=g).to(torch.bfloat16)

    def time(self, tokens):
        x = self.x[:, :tokens].contiguous()
        with torch.no_grad():
            t0 = time.perf_counter()
            y = self.OC.layer_forward_torch_cpu(x, self.w, self.sin[:tokens], self.cos[:tokens])
            dt = time.perf_counter() - t0
        assert torch.isfinite(y.float()).all()
        return dt

    def pick_tokens(self, target_s=4.0):
        """Largest power-of-two sequence prefix (128..2048) whose pass stays near target_s."""
        self.time(128)  # thread pool start-up, first-touch of the weights
        t128 = self.time(128)
        tokens = 128
        while tokens < SEQ and t128 * (tokens * 2 / 128) * 1.2 < target_s:
            tokens *= 2
        return tokens

    def sample_note(self, tokens):
        return (f"1 sequence x {tokens} tokens per pass (prefix of a {SEQ}-token sequence), bf16, "
                "PyTorch CPU operators")


def cpu_chain_baseline(passes=3):
    cc = CpuChain()
    tokens = cc.pick_tokens()
    cc.time(tokens)  # warm at the sampled size
    times = [cc.time(tokens) for _ in range(passes)]
    t = statistics.median(times)
    return {"value": tokens / t, "unit": UNIT, "cores": cc.threads, "kind": "port",
            "sample": cc.sample_note(tokens) + f"; median of {passes} passes after 1 warm-up pass"}


def run_reference(args, rank, world):
    if rank != 0:
        return
    cc = CpuChain()
    tokens = cc.pick_tokens()
    for _ in range(args.warmup):
        cc.time(tokens)
    times = [cc.time(tokens) for _ in range(args.steps)]
    total = sum(times)
    value = tokens * args.steps / total
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1000 * total / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": config(world),
        "impl": "reference",
        "reference_note": "reference kernels need ninetoothed (not installed, no network): the arm runs "
        "PyTorch's CPU operators, the oracle of the reference's own tests",
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cc.threads, "kind": "port",
                         "sample": cc.sample_note(tokens)},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------- per-op table ------
def time_op(fn, iters=10, warmup=3, flush=None):
    """Median CUDA-event time (ms) of fn(); `flush` (writing > L2) runs between iterations.

    All iterations are enqueued before one synchronisation, so the host runs ahead of the GPU
    and each event pair brackets device time only (no launch latency of an idle GPU)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    pairs = []
    for _ in range(iters):
        if flush is not None:
            flush()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        pairs.append((s, e))
    torch.cuda.synchronize()
    return statistics.median(s.elapsed_time(e) for s, e in pairs)


def time_cycled(fns, reps=5):
    """Mean device time (ms) per launch of fns (one launch each, over distinct inputs), captured
    as one CUDA graph so the launches run back to back with no host gaps; median of `reps`
    replays.  For operators whose input fits in L2: cycling through copies whose total exceeds
    L2 keeps every launch's input out of L2 without a flush kernel inside the timed region."""
    for f in fns:
        f()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for f in fns:
            f()
    graph.replay()
    torch.cuda.synchronize()
    times = []
    for _ in range(reps):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        graph.replay()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e) / len(fns))
    del graph
    return statistics.median(times)


def cpu_time(fn):
    """Wall time (ms) of one call of a PyTorch CPU operator after one warm-up call."""
    fn()
    t0 = time.perf_counter()
    fn()
    return (time.perf_counter() - t0) * 1e3


def cpu_rope(x, sin, cos):
    """Non-interleaved RoPE with PyTorch CPU operators (the reference test's restatement,
    tests/test_rotary_position_embedding.py:8-29)."""
    half = x.shape[-1] // 2
    x0, x1 = x[..., :half], x[..., half:]
    s4, c4 = sin[None, :, None, :], cos[None, :, None, :]
    return torch.cat((x0 * c4 - x1 * s4, x0 * s4 + x1 * c4), -1)


def per_op_table(dev, peaks, with_cpu=True):
    """Every BASELINE per-op configuration on one GPU, and (with_cpu) the same op on PyTorch's
    CPU implementation, all host threads, on the same sizes (a stated slice for config 5)."""
    import torch.nn.functional as F

    import ntops_b200.torch as nt

    threads = host_threads()
    torch.set_num_threads(threads)
    g = torch.Generator(device=dev).manual_seed(0)
    gc = torch.Generator().manual_seed(0)
    n = 1 << 28
    res = {}

    def cpu_entry(fn, amount, kind, sample="full size", scale=1.0):
        if not with_cpu:
            return None
        ms = cpu_time(fn) * scale
        rate = amount / (ms * 1e-3) / (1e9 if kind == "bw" else 1e12)
        key = "GB/s" if kind == "bw" else "TFLOP/s"
        return {"ms": round(ms, 2), key: round(rate, 3), "cores": threads, "sample": sample}

    def bw(name, fn, nbytes, cpu=None, cycled=None):
        ms = time_cycled(cycled) if cycled is not None else time_op(fn)
        gbs = nbytes / (ms * 1e-3) / 1e9
        res[name] = {"ms": round(ms, 4), "GB/s": round(gbs, 1), "frac": round(gbs / peaks["hbm_gbs"], 3)}
        if cpu is not None:
            res[name]["cpu"] = cpu_entry(cpu[0], nbytes, "bw", *cpu[1:])

    def tf(name, fn, flops, cpu=None):
        ms = time_op(fn, iters=5, warmup=2)
        t = flops / (ms * 1e-3) / 1e12
        res[name] = {"ms": round(ms, 3), "TFLOP/s": round(t, 1), "frac": round(t / peaks["bf16_tflops"], 3)}
        if cpu is not None:
            res[name]["cpu"] = cpu_entry(cpu[0], flops, "tf", *cpu[1:])

    for dt, tag in ((torch.float32, "f32"), (torch.float16, "f16"), (torch.bfloat16, "bf16")):
        es = torch.tensor([], dtype=dt).element_size()
        a = (torch.rand(n, generator=g, device=dev) * 8 - 4).to(dt)
        b = (torch.rand(n, generator=g, device=dev) * 8 - 4).to(dt)
        e = (torch.rand(n, generator=g, device=dev) * 1.5 + 0.5).to(dt)
        ac = (torch.rand(n, generator=gc) * 8 - 4).to(dt) if with_cpu else None
        bc = (torch.rand(n, generator=gc) * 8 - 4).to(dt) if with_cpu else None
        ec = (torch.rand(n, generator=gc) * 1.5 + 0.5).to(dt) if with_cpu else None
        for name, fn, cfn in (("add", lambda: nt.add(a, b), lambda: torch.add(ac, bc)),
                              ("mul", lambda: nt.mul(a, b), lambda: torch.mul(ac, bc)),
                              ("div", lambda: nt.div(a, b), lambda: torch.div(ac, bc)),
                              ("pow", lambda: nt.pow(a, e), lambda: torch.pow(ac, ec))):
            bw(f"{name}_{tag}", fn, 3 * n * es, cpu=(cfn,))
        for name, fn, cfn in (("silu", lambda: nt.silu(a), lambda: F.silu(ac)),
                              ("gelu_tanh", lambda: nt.gelu(a, approximate="tanh"),
                               lambda: F.gelu(ac, approximate="tanh")),
                              ("sigmoid", lambda: nt.sigmoid(a), lambda: torch.sigmoid(ac)),
                              ("exp", lambda: nt.exp(a), lambda: torch.exp(ac)),
                              ("clamp", lambda: nt.clamp(a, -1, 1), lambda: torch.clamp(ac, -1, 1))):
            bw(f"{name}_{tag}", fn, 2 * n * es, cpu=(cfn,))
        del a, b, e, ac, bc, ec
    ah = torch.randn(n, generator=g, device=dev).to(torch.float16)
    bh = torch.randn(n, generator=g, device=dev).to(torch.float16)
    ahc = torch.randn(n, generator=gc).to(torch.float16) if with_cpu else None
    bhc = torch.randn(n, generator=gc).to(torch.float16) if with_cpu else None
    bw("eq_f16", lambda: nt.eq(ah, bh), n * 5, cpu=(lambda: torch.eq(ahc, bhc),))
    bw("lt_f16", lambda: nt.lt(ah, bh), n * 5, cpu=(lambda: torch.lt(ahc, bhc),))
    del ah, bh, ahc, bhc
    ia = torch.randint(-2**31, 2**31 - 1, (n,), generator=g, device=dev, dtype=torch.int32)
    ib = torch.randint(-2**31, 2**31 - 1, (n,), generator=g, device=dev, dtype=torch.int32)
    iac = torch.randint(-2**31, 2**31 - 1, (n,), generator=gc, dtype=torch.int32) if with_cpu else None
    ibc = torch.randint(-2**31, 2**31 - 1, (n,), generator=gc, dtype=torch.int32) if with_cpu else None
    bw("bitwise_and_i32", lambda: nt.bitwise_and(ia, ib), 3 * n * 4, cpu=(lambda: torch.bitwise_and(iac, ibc),))
    bw("bitwise_or_i32", lambda: nt.bitwise_or(ia, ib), 3 * n * 4, cpu=(lambda: torch.bitwise_or(iac, ibc),))
    bw("bitwise_not_i32", lambda: nt.bitwise_not(ia), 2 * n * 4, cpu=(lambda: torch.bitwise_not(iac),))
    del ia, ib, iac, ibc
    # §8 f2, the elementwise members with special logic (not a BASELINE config; C2's 2^28 elements)
    fa = torch.randn(n, generator=g, device=dev) * 4
    fb = torch.randn(n, generator=g, device=dev) * 4
    fac = torch.randn(n, generator=gc) * 4 if with_cpu else None
    fbc = torch.randn(n, generator=gc) * 4 if with_cpu else None
    bw("copysign_f32", lambda: nt.copysign(fa, fb), 3 * n * 4, cpu=(lambda: torch.copysign(fac, fbc),))
    bw("nextafter_f32", lambda: nt.nextafter(fa, fb), 3 * n * 4, cpu=(lambda: torch.nextafter(fac, fbc),))
    bw("lgamma_f32", lambda: nt.lgamma(fa), 2 * n * 4, cpu=(lambda: torch.lgamma(fac),))
    bw("frac_f32", lambda: nt.frac(fa), 2 * n * 4, cpu=(lambda: torch.frac(fac),))
    del fb, fbc
    hb = fa.to(torch.bfloat16)
    hbc = fac.to(torch.bfloat16) if with_cpu else None
    bw("rad2deg_bf16", lambda: nt.rad2deg(hb), 2 * n * 2, cpu=(lambda: torch.rad2deg(hbc),))
    del fa, fac, hb, hbc
    la = torch.randint(1, 1 << 15, (n,), generator=g, device=dev, dtype=torch.int32)
    lb = torch.randint(1, 1 << 15, (n,), generator=g, device=dev, dtype=torch.int32)
    lac = torch.randint(1, 1 << 15, (n,), generator=gc, dtype=torch.int32) if with_cpu else None
    lbc = torch.randint(1, 1 << 15, (n,), generator=gc, dtype=torch.int32) if with_cpu else None
    bw("lcm_i32", lambda: nt.lcm(la, lb), 3 * n * 4, cpu=(lambda: torch.lcm(lac, lbc),))
    del la, lb, lac, lbc
    c1 = torch.randn(4096, 1, generator=g, device=dev)
    r1 = torch.randn(1, 65536, generator=g, device=dev)
    c1c, r1c = c1.cpu(), r1.cpu()
    bw("broadcast_add_f32", lambda: nt.add(c1, r1), 4096 * 65536 * 4 + (4096 + 65536) * 4,
       cpu=(lambda: torch.add(c1c, r1c),))
    # C1 rms_norm (134 MB, about the size of L2): launched back to back over 8 copies of the input
    # (1.07 GB in all), so each launch's input was evicted by the 7 launches before it and no
    # flush kernel's write-back lands inside the timed launch
    x1 = torch.randn(8, 512, 4096, generator=g, device=dev)
    w1 = 1 + 0.1 * torch.randn(4096, generator=g, device=dev)
    x1s = [x1.clone() for _ in range(8)]
    x1c, w1c = x1.cpu(), w1.cpu()
    bw("rms_norm_f32_8x512x4096", None, 2 * x1.numel() * 4 + 4096 * 4,
       cpu=(lambda: F.rms_norm(x1c, (4096,), w1c, 1e-6),),
       cycled=[(lambda t=t: nt.rms_norm(t, (4096,), w1, 1e-6)) for t in x1s])
    res["rms_norm_f32_8x512x4096"]["timing"] = "8 launches over 8 input copies (1.07 GB), one CUDA graph"
    del x1, x1c, x1s
    # C4
    xs = torch.randn(4096, 32768, generator=g, device=dev) * 2
    xsc = xs.cpu() if with_cpu else None
    bw("softmax_f32_4096x32768", lambda: nt.softmax(xs, -1), 2 * xs.numel() * 4,
       cpu=(lambda: torch.softmax(xsc, -1),))
    del xs, xsc
    xl = torch.randn(32768, 8192, generator=g, device=dev).to(torch.bfloat16)
    wl = (1 + 0.1 * torch.randn(8192, generator=g, device=dev)).to(torch.bfloat16)
    bl = (0.1 * torch.randn(8192, generator=g, device=dev)).to(torch.bfloat16)
    xlc, wlc, blc = (xl.cpu(), wl.cpu(), bl.cpu()) if with_cpu else (None, None, None)
    bw("layer_norm_bf16_32768x8192", lambda: nt.layer_norm(xl, (8192,), wl, bl, 1e-5), 2 * xl.numel() * 2 + 4 * 8192,
       cpu=(lambda: F.layer_norm(xlc, (8192,), wlc, blc, 1e-5),))
    del xl, xlc
    # RoPE at the chain's q / k sizes
    from ntops_b200.chain import rope_tables

    q = torch.randn(16, 2048, 32, 128, generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn(16, 2048, 8, 128, generator=g, device=dev).to(torch.bfloat16)
    sn, cs = rope_tables(2048, dev)
    qc, kc, snc, csc = (q.cpu(), k.cpu(), sn.cpu(), cs.cpu()) if with_cpu else (None,) * 4
    bw("rope_bf16_q", lambda: nt.rotary_position_embedding(q, sn, cs, interleaved=False), 2 * q.numel() * 2,
       cpu=(lambda: cpu_rope(qc, snc, csc),))
    # k is 64 MB (below L2): launched back to back over 16 copies (1.07 GB in all)
    ks = [k.clone() for _ in range(16)]
    bw("rope_bf16_k", None, 2 * k.numel() * 2, cpu=(lambda: cpu_rope(kc, snc, csc),),
       cycled=[(lambda t=t: nt.rotary_position_embedding(t, sn, cs, interleaved=False)) for t in ks])
    res["rope_bf16_k"]["timing"] = "16 launches over 16 input copies (1.07 GB), one CUDA graph"
    del q, k, qc, kc, ks
    # C5 (the CPU legs run a stated slice and scale it to the full size)
    A = (torch.randn(16384, 8192, generator=g, device=dev)).to(torch.bfloat16)
    B = (torch.randn(8192, 8192, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    bias = torch.randn(8192, generator=g, device=dev).to(torch.bfloat16)
    rows = 512
    Ac, Bc, biasc = (A[:rows].cpu(), B.cpu(), bias.cpu()) if with_cpu else (None,) * 3
    tf("addmm_bf16_16384x8192x8192", lambda: nt.addmm(bias, A, B), 2 * 16384 * 8192 * 8192,
       cpu=(lambda: torch.addmm(biasc, Ac, Bc), f"{rows} of 16384 rows, time x {16384 // rows}", 16384 / rows))
    del A, B, Ac, Bc
    qa = torch.randn(8, 32, 8192, 128, generator=g, device=dev).to(torch.bfloat16)
    ka = torch.randn(8, 32, 8192, 128, generator=g, device=dev).to(torch.bfloat16)
    va = torch.randn(8, 32, 8192, 128, generator=g, device=dev).to(torch.bfloat16)
    qac, kac, vac = (qa[:1, :1].cpu(), ka[:1, :1].cpu(), va[:1, :1].cpu()) if with_cpu else (None,) * 3
    fl = 4 * 8 * 32 * 8192 * 8192 * 128
    note = "1 of 256 (batch, head) pairs, time x 256"
    tf("sdpa_bf16_8x32x8192x128", lambda: nt.scaled_dot_product_attention(qa, ka, va), fl,
       cpu=(lambda: F.scaled_dot_product_attention(qac, kac, vac), note, 256.0))
    tf("sdpa_causal_bf16_8x32x8192x128", lambda: nt.scaled_dot_product_attention(qa, ka, va, is_causal=True),
       fl * (8192 + 1) / (2 * 8192),
       cpu=(lambda: F.scaled_dot_product_attention(qac, kac, vac, is_causal=True), note, 256.0))
    del qa, ka, va, qac, kac, vac
    # fp32 attention (not a BASELINE config; C5's shape with batch 2): tensor cores through fp16
    # copies in a workspace, staging included in the time
    qf, kf, vf = (torch.randn(2, 32, 8192, 128, generator=g, device=dev) for _ in range(3))
    qfc, kfc, vfc = (qf[:1, :1].cpu(), kf[:1, :1].cpu(), vf[:1, :1].cpu()) if with_cpu else (None,) * 3
    tf("sdpa_f32_2x32x8192x128", lambda: nt.scaled_dot_product_attention(qf, kf, vf), fl / 4,
       cpu=(lambda: F.scaled_dot_product_attention(qfc, kfc, vfc), "1 of 64 (batch, head) pairs, time x 64", 64.0))
    del qf, kf, vf, qfc, kfc, vfc
    # conv2d (§8 f3; not a BASELINE config): a ResNet-style 3x3 layer, bf16, N32 C256 56x56 ->
    # K256, pad 1 (the CPU leg times one image and scales by 32)
    xc = torch.randn(32, 256, 56, 56, generator=g, device=dev).to(torch.bfloat16)
    wc = (torch.randn(256, 256, 3, 3, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    xcc, wcc = (xc[:1].cpu(), wc.cpu()) if with_cpu else (None, None)
    tf("conv2d_bf16_n32_c256_56x56_k256_3x3", lambda: nt.conv2d(xc, wc, None, 1, 1), 2 * 32 * 256 * 256 * 9 * 56 * 56,
       cpu=(lambda: F.conv2d(xcc, wcc, None, 1, 1), "1 of 32 images, time x 32", 32.0))
    del xc, wc, xcc
    # dropout (§8 f3): p = 0.1 over 2^28 bf16 elements, HBM-bound (one read, one write)
    xdp = torch.randn(n, generator=g, device=dev).to(torch.bfloat16)
    xdpc = xdp.cpu() if with_cpu else None
    bw("dropout_bf16_p0.1", lambda: nt.dropout(xdp, 0.1), 2 * n * 2,
       cpu=(lambda: F.dropout(xdpc, 0.1, training=True),))
    del xdp, xdpc
    # decode step against an 8192-token KV cache (Llama-3-8B heads): HBM-bound on K / V; 4 copies
    # of the 268 MB cache launched back to back (1.07 GB in all)
    qd = torch.randn(8, 32, 1, 128, generator=g, device=dev).to(torch.bfloat16)
    kd = torch.randn(8, 8, 8192, 128, generator=g, device=dev).to(torch.bfloat16)
    vd = torch.randn(8, 8, 8192, 128, generator=g, device=dev).to(torch.bfloat16)
    qdc, kdc, vdc = (qd.cpu(), kd.cpu(), vd.cpu()) if with_cpu else (None,) * 3
    kvs = [(kd.clone(), vd.clone()) for _ in range(4)]
    bw("sdpa_decode_bf16_b8_hq32_hkv8_kv8192", None, (kd.numel() + vd.numel()) * 2 + 2 * qd.numel() * 2,
       cpu=(lambda: F.scaled_dot_product_attention(qdc, kdc, vdc, enable_gqa=True),),
       cycled=[(lambda kk=kk, vv=vv: nt.scaled_dot_product_attention(qd, kk, vv, enable_gqa=True)) for kk, vv in kvs])
    res["sdpa_decode_bf16_b8_hq32_hkv8_kv8192"]["timing"] = "4 launches over 4 K / V copies (1.07 GB), one CUDA graph"
    del kvs
    return res


def sharded_op_table(dev, rank, world, peaks):
    """BASELINE configs 4 and 5 sharded over the ranks with no exchange on the data path.

    Every rank builds the same global inputs from one seed and runs its shard: softmax and
    layer_norm by rows, attention by (batch x head) units, addmm by M rows (B and bias
    replicated).  Throughput = whole-job work / max-over-ranks median time.  Afterwards the
    shards are all-gathered over NCCL and rank 0 compares them with one unsharded launch of the
    same operator (outside the timed region)."""
    import torch.distributed as dist

    import ntops_b200.torch as nt
    from ntops_b200.shard import max_over_ranks, shard_range

    g = torch.Generator(device=dev).manual_seed(0)
    res = {}

    def gathered_equal(local, full_fn, total):
        if total % world:
            return "skipped (shards of unequal size)"  # the same decision on every rank
        out = torch.empty((world * local.shape[0],) + tuple(local.shape[1:]), dtype=local.dtype, device=dev)
        dist.all_gather_into_tensor(out, local.contiguous())
        verdict = None
        if rank == 0:
            ref = full_fn().reshape(out.shape)
            if torch.equal(out, ref):
                verdict = "bit-exact"
            else:
                verdict = f"max_abs_diff={float((out.float() - ref.float()).abs().max()):.3g}"
        dist.barrier()
        return verdict

    def record(name, ms_local, amount, kind, sharding, verdict):
        ms = max_over_ranks(ms_local, dev)
        if kind == "bw":
            rate = amount / (ms * 1e-3) / 1e9
            res[name] = {"ms": round(ms, 4), "GB/s": round(rate, 1), "frac": round(rate / (world * peaks["hbm_gbs"]), 3)}
        else:
            rate = amount / (ms * 1e-3) / 1e12
            res[name] = {"ms": round(ms, 3), "TFLOP/s": round(rate, 1),
                         "frac": round(rate / (world * peaks["bf16_tflops"]), 3)}
        res[name].update({"n_gpus": world, "sharding": sharding, "gathered_vs_unsharded": verdict})

    def timed(fn, **kw):
        dist.barrier()
        return time_op(fn, **kw)

    # C4 softmax fp32 [4096, 32768], rows sharded
    xs = torch.randn(4096, 32768, generator=g, device=dev) * 2
    r0, r1 = shard_range(4096, rank, world)
    xsl = xs[r0:r1]
    ms = timed(lambda: nt.softmax(xsl, -1))
    record("softmax_f32_4096x32768", ms, 2 * xs.numel() * 4, "bw", f"rows/{world}",
           gathered_equal(nt.softmax(xsl, -1), lambda: nt.softmax(xs, -1), 4096))
    del xs, xsl
    # C4 layer_norm bf16 [32768, 8192], rows sharded
    xl = torch.randn(32768, 8192, generator=g, device=dev).to(torch.bfloat16)
    wl = (1 + 0.1 * torch.randn(8192, generator=g, device=dev)).to(torch.bfloat16)
    bl = (0.1 * torch.randn(8192, generator=g, device=dev)).to(torch.bfloat16)
    r0, r1 = shard_range(32768, rank, world)
    xll = xl[r0:r1]
    ms = timed(lambda: nt.layer_norm(xll, (8192,), wl, bl, 1e-5))
    record("layer_norm_bf16_32768x8192", ms, 2 * xl.numel() * 2 + 4 * 8192, "bw", f"rows/{world}",
           gathered_equal(nt.layer_norm(xll, (8192,), wl, bl, 1e-5), lambda: nt.layer_norm(xl, (8192,), wl, bl, 1e-5),
                          32768))
    del xl, xll
    # C5 attention bf16 [8, 32, 8192, 128], (batch x head) units sharded
    qa = torch.randn(8, 32, 8192, 128, generator=g, device=dev).to(torch.bfloat16)
    ka = torch.randn(8, 32, 8192, 128, generator=g, device=dev).to(torch.bfloat16)
    va = torch.randn(8, 32, 8192, 128, generator=g, device=dev).to(torch.bfloat16)
    u0, u1 = shard_range(8 * 32, rank, world)

    def unit_view(t):
        return t.view(8 * 32, 8192, 128)[u0:u1].unsqueeze(0)

    ql, kl, vl = unit_view(qa), unit_view(ka), unit_view(va)
    fl = 4 * 8 * 32 * 8192 * 8192 * 128
    for causal, name, flops in ((False, "sdpa_bf16_8x32x8192x128", fl),
                                (True, "sdpa_causal_bf16_8x32x8192x128", fl * (8192 + 1) / (2 * 8192))):
        ms = timed(lambda: nt.scaled_dot_product_attention(ql, kl, vl, is_causal=causal), iters=5, warmup=2)
        local = nt.scaled_dot_product_attention(ql, kl, vl, is_causal=causal)[0]
        record(name, ms, flops, "tf", f"(batch x head) units/{world}",
               gathered_equal(local, lambda: nt.scaled_dot_product_attention(qa, ka, va, is_causal=causal), 256))
    del qa, ka, va, ql, kl, vl
    # C5 addmm bf16 [16384, 8192] x [8192, 8192] + bias, M rows sharded
    A = torch.randn(16384, 8192, generator=g, device=dev).to(torch.bfloat16)
    B = (torch.randn(8192, 8192, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    bias = torch.randn(8192, generator=g, device=dev).to(torch.bfloat16)
    r0, r1 = shard_range(16384, rank, world)
    Al = A[r0:r1]
    ms = timed(lambda: nt.addmm(bias, Al, B), iters=5, warmup=2)
    record("addmm_bf16_16384x8192x8192", ms, 2 * 16384 * 8192 * 8192, "tf", f"M rows/{world}",
           gathered_equal(nt.addmm(bias, Al, B), lambda: nt.addmm(bias, A, B), 16384))
    return res


# ----------------------------------------------------------------- single-op cases -------
def run_case(name, reps):
    """Runs one hot-path operator `reps` times on seeded inputs (for ncu captures of one kernel);
    prints the median CUDA-event time of the launches."""
    import ntops_b200.torch as nt

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(0)

    def rn(*shape, dt=torch.bfloat16, scale=1.0):
        return (torch.randn(shape, generator=g, device=dev) * scale).to(dt)

    if name == "gemm_gate":  # chain gate projection: [32768, 4096] x [4096, 14336]
        a, b = rn(32768, 4096), rn(4096, 14336, scale=0.02)
        fn = lambda: nt.mm(a, b)  # noqa: E731
    elif name == "swiglu":  # chain fused gate/up projection: [32768, 4096] x [4096, 2 x 14336]
        from ntops_b200.fused import swiglu_linear

        a, b = rn(32768, 4096), rn(4096, 2 * 14336, scale=0.02)
        fn = lambda: swiglu_linear(a, b)  # noqa: E731
    elif name == "addmm_c5":  # BASELINE config 5 addmm
        a, b, c = rn(16384, 8192), rn(8192, 8192, scale=0.02), rn(8192)
        fn = lambda: nt.addmm(c, a, b)  # noqa: E731
    elif name == "sdpa_causal":  # a quarter-size slice of config 5 attention (B2 H32 S4096 D128)
        q, k, v = rn(2, 32, 4096, 128), rn(2, 32, 4096, 128), rn(2, 32, 4096, 128)
        fn = lambda: nt.scaled_dot_product_attention(q, k, v, is_causal=True)  # noqa: E731
    elif name == "sdpa":
        q, k, v = rn(2, 32, 4096, 128), rn(2, 32, 4096, 128), rn(2, 32, 4096, 128)
        fn = lambda: nt.scaled_dot_product_attention(q, k, v)  # noqa: E731
    elif name == "sdpa_c5":  # config 5 attention at full size
        q, k, v = rn(8, 32, 8192, 128), rn(8, 32, 8192, 128), rn(8, 32, 8192, 128)
        fn = lambda: nt.scaled_dot_product_attention(q, k, v)  # noqa: E731
    elif name == "sdpa_causal_c5":
        q, k, v = rn(8, 32, 8192, 128), rn(8, 32, 8192, 128), rn(8, 32, 8192, 128)
        fn = lambda: nt.scaled_dot_product_attention(q, k, v, is_causal=True)  # noqa: E731
    elif name == "softmax_c4":
        x = rn(4096, 32768, dt=torch.float32, scale=2.0)
        fn = lambda: nt.softmax(x, -1)  # noqa: E731
    elif name == "layer_norm_c4":
        x, w, b = rn(32768, 8192), rn(8192), rn(8192)
        fn = lambda: nt.layer_norm(x, (8192,), w, b, 1e-5)  # noqa: E731
    elif name == "rms_norm_c1":
        x, w = rn(8, 512, 4096, dt=torch.float32), rn(4096, dt=torch.float32)
        fn = lambda: nt.rms_norm(x, (4096,), w, 1e-6)  # noqa: E731
    elif name == "sdpa_decode":
        q, k, v = rn(8, 32, 1, 128), rn(8, 8, 8192, 128), rn(8, 8, 8192, 128)
        fn = lambda: nt.scaled_dot_product_attention(q, k, v, enable_gqa=True)  # noqa: E731
    elif name in ("silu_bf16", "sigmoid_bf16", "silu_f16", "sigmoid_f16", "pow_bf16", "pow_f16"):
        op, tag = name.split("_")
        dt = torch.bfloat16 if tag == "bf16" else torch.float16
        x = (torch.rand(1 << 28, generator=g, device=dev) * 8 - 4).to(dt)
        e = (torch.rand(1 << 28, generator=g, device=dev) * 1.5 + 0.5).to(dt)
        fn = (lambda: nt.pow(x, e)) if op == "pow" else (lambda: getattr(nt, op)(x))  # noqa: E731
    elif name == "conv2d":  # the per-op table's ResNet-style 3x3 layer, bf16
        g = torch.Generator(device=dev).manual_seed(0)
        xc = torch.randn((32, 256, 56, 56), device=dev, generator=g).to(torch.bfloat16)
        wc = (torch.randn((256, 256, 3, 3), device=dev, generator=g) * 0.02).to(torch.bfloat16)
        fn = lambda: nt.conv2d(xc, wc, None, 1, 1)  # noqa: E731
    elif name == "sdpa_f32":  # the per-op table's fp32 attention line (staged to fp16)
        g = torch.Generator(device=dev).manual_seed(0)
        qf, kf, vf = (torch.randn((2, 32, 8192, 128), device=dev, generator=g) for _ in range(3))
        fn = lambda: nt.scaled_dot_product_attention(qf, kf, vf)  # noqa: E731
    elif name == "dropout":  # the per-op table's dropout line: p = 0.1 over 2^28 bf16 elements
        g = torch.Generator(device=dev).manual_seed(0)
        xdp = torch.randn(1 << 28, device=dev, generator=g).to(torch.bfloat16)
        fn = lambda: nt.dropout(xdp, 0.1)  # noqa: E731
    elif name == "rope_q":
        from ntops_b200.chain import rope_tables

        x = rn(16, 2048, 32, 128)
        sn, cs = rope_tables(2048, dev)
        fn = lambda: nt.rotary_position_embedding(x, sn, cs, interleaved=False)  # noqa: E731
    else:
        raise SystemExit(f"unknown case {name}")
    print(json.dumps({"case": name, "ms": time_op(fn, iters=reps, warmup=1)}), flush=True)


# ---------------------------------------------------------------------------- main --------
def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ntops_b200", choices=["ntops_b200", "reference"])
    ap.add_argument("--no-ops", action="store_true", help="skip the per-op table")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baselines")
    ap.add_argument("--global-batch", type=int, default=GLOBAL_BATCH,
                    help="sequences of 2048 tokens over all ranks (the BASELINE config is 16)")
    ap.add_argument("--no-graph", action="store_true", help="launch every operator from Python each step "
                    "instead of replaying the step as one CUDA graph")
    ap.add_argument("--case", default=None, help="run one operator case (for ncu) and exit")
    ap.add_argument("--reps", type=int, default=2)
    args = ap.parse_args()
    if args.case:
        return run_case(args.case, args.reps)
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        return run_reference(args, rank, world)

    import torch.distributed as dist

    import ntops_b200.torch as nt  # noqa: F401
    from ntops_b200 import _lib, chain
    from ntops_b200.shard import max_over_ranks, shard_range
    from ntops_b200.torch import utils as ntu

    assert args.warmup >= 3, "at least 3 warm-up steps"
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    peaks, peak_src = load_peaks()

    global_batch = args.global_batch
    s0, s1 = shard_range(global_batch, rank, world)
    batch = s1 - s0
    tokens = batch * SEQ
    wts = chain.LayerWeights(dev)
    sin, cos = chain.rope_tables(SEQ, dev)
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    x = torch.randn((batch, SEQ, chain.HIDDEN), generator=g, device=dev).to(torch.bfloat16)
    mm_flops, attn_flops = chain.layer_flops(batch, SEQ)

    for _ in range(args.warmup):
        chain.layer_forward(x, wts, sin, cos)
    torch.cuda.synchronize()

    gemm_events = []

    def mm_hook(fn, a, b):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        out = fn(a, b)
        e.record()
        gemm_events.append((s, e))
        return out

    # One layer pass as a CUDA graph (the step's kernels with no host launch gaps); the GEMM
    # timing events are recorded inside the captured pass, so they replay with it.
    use_graph = not args.no_graph
    graph = None
    step_launches = 0
    if use_graph:
        cap_events = []

        def cap_hook(fn, a, b):
            # external events become real event-record nodes of the graph (timestamps on replay)
            s = torch.cuda.Event(enable_timing=True, external=True)
            e = torch.cuda.Event(enable_timing=True, external=True)
            s.record()
            out = fn(a, b)
            e.record()
            cap_events.append((s, e))
            return out

        chain.layer_forward(x, wts, sin, cos, mm_hook=cap_hook)  # warm caches / attributes once more
        torch.cuda.synchronize()
        cap_events.clear()
        graph = torch.cuda.CUDAGraph()
        l0 = ntu.launch_count
        with torch.cuda.graph(graph, capture_error_mode="relaxed"):
            y_static = chain.layer_forward(x, wts, sin, cos, mm_hook=cap_hook)
        step_launches = ntu.launch_count - l0
        for _ in range(args.warmup):
            graph.replay()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    # ---- timed region: inputs resident in HBM
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = ntu.launch_count
    gemm_times = []
    with ClockSampler(local_rank) as clk:
        torch.cuda.synchronize()
        start.record()
        for _ in range(args.steps):
            if graph is not None:
                graph.replay()
            else:
                y = chain.layer_forward(x, wts, sin, cos, mm_hook=mm_hook)
        end.record()
        torch.cuda.synchronize()
    if graph is not None:
        y = y_static
        launches = step_launches * args.steps
        # the captured events hold the last replay's GEMM times: one pass's worth per step
        gemm_times = [s.elapsed_time(e) for s, e in cap_events] * args.steps
    else:
        launches = ntu.launch_count - launches0
        gemm_times = [s.elapsed_time(e) for s, e in gemm_events]
    ms_local = start.elapsed_time(end)
    gemm_ms = sum(gemm_times)
    # the fused gate/up (SwiGLU) projection among the GEMM launches of a pass
    shapes = chain.gemm_shapes(tokens)
    gi = chain.swiglu_index()
    gate_ms = statistics.mean(gemm_times[gi::len(shapes)])
    gm, gn, gk = shapes[gi]
    gate_tflops = 2 * gm * gn * gk / (gate_ms * 1e-3) / 1e12
    ms = max_over_ranks(ms_local, dev)
    value = global_batch * SEQ * args.steps / (ms * 1e-3)
    gemm_tflops = mm_flops * args.steps / (gemm_ms * 1e-3) / 1e12
    rc = _lib.load().ntb_check_device_error(None)
    assert rc == 0, "a kernel reported a device-side timeout"
    y_resident = y.clone()
    checksum = float(y_resident.float().abs().mean())
    assert checksum == checksum and checksum > 0, "non-finite layer output"

    # ---- end to end: every step's input comes from pinned host memory and its output goes
    # back to pinned host memory, through the public API.  The copies run on their own streams
    # (double-buffered), so step i+1's upload and step i-1's download overlap step i's kernels;
    # each step's kernels are one replay of a graph captured from chain.layer_forward on that
    # buffer, so the host issues a handful of calls per step whatever the GPU count.
    xh = x.cpu().pin_memory()
    yh = [torch.empty(y.shape, dtype=y.dtype).pin_memory() for _ in range(2)]
    xbuf = [x.clone() for _ in range(2)]
    comp = torch.cuda.current_stream(dev)
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    e2e_graphs, e2e_out = [], []
    if use_graph:
        for b in range(2):
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, capture_error_mode="relaxed"):
                e2e_out.append(chain.layer_forward(xbuf[b], wts, sin, cos))
            e2e_graphs.append(gr)
        torch.cuda.synchronize()

    def ev(timing=False):
        return torch.cuda.Event(enable_timing=timing)

    x_free, x_ready = [ev(), ev()], [ev(), ev()]
    y_ready, y_done = [ev(), ev()], [ev(), ev()]
    for i in range(2):
        x_free[i].record(comp)
        y_done[i].record(down)
    leg_events = []

    def e2e_steps(n, timing=False):
        legs = []
        for i in range(n):
            b = i & 1
            t = [ev(timing) for _ in range(4)] if timing else None
            with torch.cuda.stream(up):
                up.wait_event(x_free[b])
                if timing:
                    t[0].record(up)
                xbuf[b].copy_(xh, non_blocking=True)
                if timing:
                    t[1].record(up)
                x_ready[b].record(up)
            comp.wait_event(x_ready[b])
            if e2e_graphs:
                comp.wait_event(y_done[b])  # the previous download of this output buffer
                e2e_graphs[b].replay()
                out = e2e_out[b]
            else:
                out = chain.layer_forward(xbuf[b], wts, sin, cos)
            x_free[b].record(comp)
            y_ready[b].record(comp)
            with torch.cuda.stream(down):
                down.wait_event(y_ready[b])
                if timing:
                    t[2].record(down)
                yh[b].copy_(out, non_blocking=True)
                if timing:
                    t[3].record(down)
                if not e2e_graphs:
                    out.record_stream(down)
                y_done[b].record(down)
            if timing:
                legs.append(t)
        comp.wait_stream(up)
        comp.wait_stream(down)
        return legs

    e2e_steps(2)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record(comp)
    leg_events = e2e_steps(args.steps, timing=True)
    e2.record(comp)
    torch.cuda.synchronize()
    ms_e2e_local = s2.elapsed_time(e2)
    ms_e2e = max_over_ranks(ms_e2e_local, dev)
    e2e_value = global_batch * SEQ * args.steps / (ms_e2e * 1e-3)
    h2d_ms = statistics.mean(t[0].elapsed_time(t[1]) for t in leg_events)
    d2h_ms = statistics.mean(t[2].elapsed_time(t[3]) for t in leg_events)
    assert torch.equal(yh[(args.steps - 1) & 1], y_resident.cpu()), "end-to-end output differs from the resident run"
    del e2e_graphs, e2e_out, xbuf, yh

    ops = None
    cpu = None
    if world == 1 and rank == 0:
        if not args.no_ops:
            ops = per_op_table(dev, peaks, with_cpu=not args.no_cpu)
        if not args.no_cpu:
            cpu = cpu_chain_baseline()
    elif world > 1 and not args.no_ops:
        ops = sharded_op_table(dev, rank, world, peaks)

    if rank == 0:
        n_bytes = x.numel() * 2
        line = {
            "metric": METRIC,
            "value": value,
            "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms / args.steps,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded randn inputs, random-init weights ~N(0,0.02))",
            "config": config(world, global_batch),
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": n_bytes * world,
                    "d2h_bytes_per_step": y.numel() * 2 * world,
                    "legs_rank0": {"ms_per_step": ms_e2e_local / args.steps, "h2d_ms": h2d_ms,
                                   "compute_ms": ms_local / args.steps, "d2h_ms": d2h_ms,
                                   "h2d_GBps": n_bytes / (h2d_ms * 1e-3) / 1e9,
                                   "d2h_GBps": y.numel() * 2 / (d2h_ms * 1e-3) / 1e9},
                    "graph_replay": bool(use_graph)},
            "gpu_launches": launches * world,
            "roofline": {"bound": "tensor", "kernel": "gemm_tc_pair_kernel (SwiGLU epilogue)",
                         "launch": f"fused gate/up projection [{gm}x{gk}]x[{gk}x{gn}] bf16 -> [{gm}x{gn // 2}] "
                                   "(largest of the 4 per step)",
                         "achieved": gate_tflops, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": gate_tflops / peaks["bf16_tflops"],
                         "peak_source": f"bf16_tflops (burst), {peak_src}",
                         "frac_of_sustained": gate_tflops / peaks["bf16_tflops_sustained"],
                         "traffic": SWIGLU_GEMM_TRAFFIC if batch == GLOBAL_BATCH else None,
                         "traffic_note": "measured at the full one-GPU size (16 x 2048 tokens)",
                         "traffic_algorithmic": (gm * gk + gk * gn + gm * gn // 2) * 2,
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch of this "
                                           "shape (profiles/gemm_tc_pair_kernel-swiglu_32768x28672x4096_bf16.md)",
                         "all_gemms": {"achieved": gemm_tflops, "frac": gemm_tflops / peaks["bf16_tflops"],
                                       "share_of_step": gemm_ms / ms_local}},
            "step_tflops": (mm_flops + attn_flops) * global_batch / batch / (ms / args.steps * 1e-3) / 1e12,
            "cuda_graph": use_graph,
            "clocks": clk.summary(),
            "cpu_baseline": cpu,
            "ops": ops,
            "peaks": {k: v for k, v in peaks.items()},
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

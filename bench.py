#!/usr/bin/env python
"""Benchmark of the B200 FlashAttention hot path (one JSON line on rank 0).

Headline: dense FA forward + backward TFLOP/s on the BASELINE configuration the target
is quoted on -- q/k/v [B=8, S=4096, H=32, D=128] bf16, causal;
a step is one forward + backward through the public API (tilelang_flash_attn_func and
autograd) over that batch.  FLOPs are counted on visible (query, key) pairs:
4 D per pair forward, 10 D per pair backward.

Scaling is weak: with N ranks the global problem is N x that batch, sharded by
(batch x heads) so every rank owns exactly one B=8 x H=32 shard; no collective runs in
the timed region (NCCL is used only for the barrier, the max-over-ranks timing and the
gathered correctness check).  value = N x per-rank FLOPs / max-over-ranks time.

Also reported in the same line: e2e (same metric through the public API with the
inputs copied from pinned host memory and out/dq/dk/dv copied back every step), the
roofline of the dominant kernel (the backward dK/dV kernel, timed live with CUDA
events on its launch stream), the CPU baseline (the reference's PyTorch attention in
fp32 on the host cores, on a bounded sample), clocks sampled during the timed region,
and secondary workloads (the other BASELINE configs: dense fp16 D=64, non-square
causal, paged GQA prefill, split-KV decode GB/s).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""
import argparse
import datetime
import json
import math
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "tilelang-fa-v100_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "dense FA fwd+bwd TFLOP/s"
UNIT = "TFLOP/s"
CFG = dict(B=8, S=4096, H=32, D=128, causal=True)
WORKLOAD = "dense_fa_fwd_bwd_bf16_B8_S4096_H32_D128_causal (BASELINE configs[2])"


def visible_pairs(b, h, sq, skv, causal):
    if not causal:
        return float(b) * h * sq * skv
    off = skv - sq
    i = np.arange(sq, dtype=np.int64)
    return float(b) * h * float(np.clip(i + off + 1, 0, skv).sum())


def step_flops(b, h, sq, skv, d, causal):
    return 14.0 * d * visible_pairs(b, h, sq, skv, causal)


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as fh:
            d = json.load(fh)
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def ncu_traffic(name):
    """DRAM bytes per launch recorded in profiles/<name>.md ('dram_bytes_per_launch: N')."""
    p = os.path.join(ROOT, "profiles", name + ".md")
    if not os.path.exists(p):
        return None
    m = re.search(r"dram_bytes_per_launch:\s*([0-9.eE+]+)", open(p).read())
    return float(m.group(1)) if m else None


class ClockSampler:
    """nvidia-smi clocks, power and throttle reasons sampled every 20 ms; the summary
    uses the samples taken between mark_start() and mark_stop() (the timed region)."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = None
        self.t_start = self.t_stop = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "--query-gpu=" + self.FIELDS, "--format=csv,noheader,nounits",
                 "-lms", "20", "-i", str(self.gpu)],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def mark_start(self):
        self.t_start = datetime.datetime.now()

    def mark_stop(self):
        self.t_stop = datetime.datetime.now()

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.05)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.path is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows, smax = [], None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in open(self.path):
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(f[0], "%Y/%m/%d %H:%M:%S.%f")
                mhz, smax, watts = float(f[2]), float(f[3]), float(f[4])
            except ValueError:
                continue
            rows.append((ts, mhz, watts, [nm for nm, val in zip(names, f[6:10]) if val.lower() == "active"]))
        os.unlink(self.path)
        window = [r for r in rows if self.t_start and self.t_stop and self.t_start <= r[0] <= self.t_stop]
        if not window and self.t_start:  # region shorter than the sampling period: next sample
            window = [r for r in rows if r[0] >= self.t_start][:1]
        reasons = sorted({nm for r in window for nm in r[3]})
        return {"sm_mhz": statistics.median(r[1] for r in window) if window else None,
                "sm_max_mhz": smax, "reasons": reasons,
                "power_w": statistics.median(r[2] for r in window) if window else None,
                "samples": len(window), "sampling_ms": 20}


# --------------------------------------------------------------------------- our arm
def dense_inputs(dev, b, s, h, d, dtype, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    mk = lambda: torch.randn(b, s, h, d, generator=g, device=dev, dtype=torch.float32).to(dtype)
    return mk(), mk(), mk(), mk()


def run_dense_steps(fa, q, k, v, do, causal, n, prof_events=None):
    """n fwd+bwd steps through the public API; optionally arms the dK/dV kernel events."""
    from tilelang_fa_v100 import _ext
    for i in range(n):
        q.grad = k.grad = v.grad = None
        out = fa.tilelang_flash_attn_func(q, k, v, causal=causal)
        if prof_events is not None:
            _ext.profile_next_launch(_ext.PROF_BWD_DKDV, *prof_events[i])
        out.backward(do)
    return out


def time_dense(fa, dev, b, s, h, d, dtype, causal, steps, warmup, seed, dist=None, profile=False,
               clk=None):
    from tilelang_fa_v100 import _ext
    q, k, v, do = dense_inputs(dev, b, s, h, d, dtype, seed)
    q, k, v = (x.requires_grad_(True) for x in (q, k, v))
    run_dense_steps(fa, q, k, v, do, causal, warmup)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps)] if profile else None
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    n0 = _ext.launch_count()
    if clk is not None:
        clk.mark_start()
    t0.record()
    out = run_dense_steps(fa, q, k, v, do, causal, steps, ev)
    t1.record()
    torch.cuda.synchronize(dev)
    if clk is not None:
        clk.mark_stop()
    launches = _ext.launch_count() - n0
    if dist is not None:
        dist.barrier()
    ms = t0.elapsed_time(t1) / steps
    kern_ms = statistics.mean(a.elapsed_time(b_) for a, b_ in ev) if profile else None
    return ms, kern_ms, launches, (q, k, v, do, out)


def check_dense(tensors, causal):
    """Max-abs error of one (batch, head) slice of out against fp32 torch on the GPU."""
    q, k, v, do, out = tensors
    torch.backends.cuda.matmul.allow_tf32 = False
    qs, ks, vs = q[0, :, 0].float(), k[0, :, 0].float(), v[0, :, 0].float()
    sc = (qs @ ks.T) / math.sqrt(q.shape[-1])
    if causal:
        m, n = sc.shape
        sc = sc.masked_fill(torch.ones(m, n, device=sc.device).tril(n - m) == 0, float("-inf"))
    ref = torch.softmax(sc, -1) @ vs
    return float((out.detach()[0, :, 0].float() - ref).abs().max())


def time_e2e(fa, dev, b, s, h, d, dtype, causal, steps, warmup, seed):
    """Public API with host buffers.  Every step uploads its q, k, v, dO from pinned host
    memory, runs fwd + bwd and downloads its out, dq, dk, dv into pinned host memory.
    Neighbouring steps overlap the way a training loop that streams its batches does:
    the upload of step k+1 and the download of step k-1 run on two copy streams while
    step k computes (device buffers double-buffered, events order each slot's reuse)."""
    q, k, v, do = dense_inputs(dev, b, s, h, d, dtype, seed)
    host_in = [x.cpu().pin_memory() for x in (q, k, v, do)]
    del q, k, v, do
    shape, nb = (b, s, h, d), 2
    dev_in = [[torch.empty(shape, dtype=dtype, device=dev) for _ in range(4)] for _ in range(nb)]
    for slot in dev_in:
        for t in slot[:3]:
            t.requires_grad_(True)
    dev_out = [[torch.empty(shape, dtype=dtype, device=dev) for _ in range(4)] for _ in range(nb)]
    host_out = [[torch.empty(shape, dtype=dtype).pin_memory() for _ in range(4)] for _ in range(nb)]
    s_up, s_comp, s_down = (torch.cuda.Stream(dev) for _ in range(3))
    ev_up = [torch.cuda.Event() for _ in range(nb)]
    ev_comp = [torch.cuda.Event() for _ in range(nb)]
    ev_down = [torch.cuda.Event() for _ in range(nb)]
    main = torch.cuda.current_stream(dev)
    for e in ev_comp + ev_down:
        e.record(main)

    def upload(i):
        sl = i % nb
        s_up.wait_event(ev_comp[sl])  # step i-2 has consumed this slot's inputs
        with torch.cuda.stream(s_up), torch.no_grad():
            for dst, src in zip(dev_in[sl], host_in):
                dst.copy_(src, non_blocking=True)
        ev_up[sl].record(s_up)

    def compute(i):
        sl = i % nb
        s_comp.wait_event(ev_up[sl])
        s_comp.wait_event(ev_down[sl])  # step i-2's outputs have left the device
        qd, kd, vd, ddo = dev_in[sl]
        with torch.cuda.stream(s_comp):
            qd.grad = kd.grad = vd.grad = None
            out = fa.tilelang_flash_attn_func(qd, kd, vd, causal=causal)
            out.backward(ddo)
            with torch.no_grad():
                for dst, src in zip(dev_out[sl], (out, qd.grad, kd.grad, vd.grad)):
                    dst.copy_(src)
        ev_comp[sl].record(s_comp)

    def download(i):
        sl = i % nb
        s_down.wait_event(ev_comp[sl])
        with torch.cuda.stream(s_down):
            for dst, src in zip(host_out[sl], dev_out[sl]):
                dst.copy_(src, non_blocking=True)
        ev_down[sl].record(s_down)

    def run(n):
        upload(0)
        for i in range(n):
            if i + 1 < n:
                upload(i + 1)
            compute(i)
            download(i)
        main.wait_event(ev_down[(n - 1) % nb])

    run(max(warmup, 2))
    torch.cuda.synchronize(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(main)
    for e in ev_comp + ev_down:  # every stream starts after t0
        e.record(main)
    run(steps)
    t1.record(main)
    torch.cuda.synchronize(dev)
    ms = t0.elapsed_time(t1) / steps

    # The host link's floor for the same bytes: one step's four uploads and four downloads
    # issued together on the two copy streams with no compute (best of 3).
    link_ms = float("inf")
    for _ in range(3):
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record(main)
        s_up.wait_stream(main)
        s_down.wait_stream(main)
        with torch.no_grad():
            with torch.cuda.stream(s_up):
                for dst, src in zip(dev_in[0], host_in):
                    dst.copy_(src, non_blocking=True)
            with torch.cuda.stream(s_down):
                for dst, src in zip(host_out[0], dev_out[0]):
                    dst.copy_(src, non_blocking=True)
        main.wait_stream(s_up)
        main.wait_stream(s_down)
        c1.record(main)
        torch.cuda.synchronize(dev)
        link_ms = min(link_ms, c0.elapsed_time(c1))
    nbytes = b * s * h * d * 2
    return ms, 4 * nbytes, 4 * nbytes, link_ms


def time_paged(dev, steps, warmup):
    """16 x 1024 tokens, H 32 / Hkv 8, D 128, page 16, shuffled pages."""
    from tilelang_fa_v100 import _ext
    rng = np.random.default_rng(0)
    g = torch.Generator(device=dev).manual_seed(1)
    kc = torch.randn(1024, 16, 8, 128, generator=g, device=dev).half()
    vc = torch.randn(1024, 16, 8, 128, generator=g, device=dev).half()
    bt = torch.from_numpy(rng.permutation(1024).astype(np.int32).reshape(16, 64)).to(dev)
    q = torch.randn(16384, 32, 128, generator=g, device=dev).half()
    qsl = torch.arange(0, 16385, 1024, dtype=torch.int32, device=dev)
    sl = torch.full((16,), 1024, dtype=torch.int32, device=dev)
    pkl = torch.zeros(16, dtype=torch.int32, device=dev)
    out = torch.empty_like(q)
    lse = torch.empty(32, 16384, device=dev)
    run = lambda: _ext.paged_prefill(q, kc, vc, bt, sl, qsl, pkl, out, lse, 16, 8, 128 ** -0.5,
                                     True, -1, -1)
    for _ in range(warmup):
        run()
    torch.cuda.synchronize(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        run()
    t1.record()
    torch.cuda.synchronize(dev)
    ms = t0.elapsed_time(t1) / steps
    return ms, 4 * 128 * visible_pairs(16, 32, 1024, 1024, True) / ms / 1e9


def decode_problem(dev, seed, batch=256, hkv=8, d=128, heads=32):
    """256 seqs, L ~ U[512, 8192], H 32 / Hkv 8, D 128, page 16, bf16
    (other head layouts with the same length distribution on request)."""
    rng = np.random.default_rng(seed)
    lens = rng.integers(512, 8193, size=batch).astype(np.int32)
    pps = (lens + 15) // 16
    total = int(pps.sum())
    perm = rng.permutation(total).astype(np.int32)
    bt = np.zeros((batch, 512), np.int32)
    c = 0
    for i in range(batch):
        bt[i, :pps[i]] = perm[c:c + pps[i]]
        c += pps[i]
    g = torch.Generator(device=dev).manual_seed(seed + 1)
    kc = torch.randn(total, 16, hkv, d, generator=g, device=dev).to(torch.bfloat16)
    vc = torch.randn(total, 16, hkv, d, generator=g, device=dev).to(torch.bfloat16)
    q = torch.randn(batch, heads, d, generator=g, device=dev).to(torch.bfloat16)
    nbytes = int(lens.sum()) * hkv * d * 2 * 2 + 2 * batch * heads * d * 2 + total * 4
    return q, kc, vc, torch.from_numpy(bt).to(dev), torch.from_numpy(lens).to(dev), nbytes


def time_decode(dev, steps, warmup, seed=0, hkv=8, d=128, heads=32):
    import tilelang_fa_v100 as fa
    q, kc, vc, bt, sl, nbytes = decode_problem(dev, seed, hkv=hkv, d=d, heads=heads)
    run = lambda: fa.tilelang_decode_forward(q, kc, vc, bt, sl)
    for _ in range(warmup):
        run()
    torch.cuda.synchronize(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        run()
    t1.record()
    torch.cuda.synchronize(dev)
    ms = t0.elapsed_time(t1) / steps
    return ms, nbytes / ms / 1e6


def time_kv_write(dev, steps, warmup, tokens=65536, hkv=8, d=128, page=16):
    """Paged KV-cache write of one large prefill step: bytes = read key + value and
    write them into the cache (slot_mapping excluded), scattered slots."""
    from tilelang_fa_v100.cache import write_kv_cache
    g = torch.Generator(device=dev).manual_seed(17)
    key = torch.randn(tokens, hkv, d, generator=g, device=dev).to(torch.bfloat16)
    value = torch.randn(tokens, hkv, d, generator=g, device=dev).to(torch.bfloat16)
    pages = 2 * tokens // page
    kc = torch.empty(pages, page, hkv, d, device=dev, dtype=torch.bfloat16)
    vc = torch.empty_like(kc)
    slots = torch.randperm(pages * page, generator=torch.Generator().manual_seed(3))[:tokens]
    slots = slots.to(dev)
    run = lambda: write_kv_cache(key, value, kc, vc, slots)
    for _ in range(warmup):
        run()
    torch.cuda.synchronize(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        run()
    t1.record()
    torch.cuda.synchronize(dev)
    ms = t0.elapsed_time(t1) / steps
    nbytes = 2 * 2 * tokens * hkv * d * 2
    return ms, nbytes / ms / 1e6


def cpu_baseline(budget_s=15.0):
    """The reference's PyTorch attention (fp32, autograd) on the host cores, on a bounded
    sample of the headline workload: whole (batch, head) slices of configs[2]."""
    from oracle import attention_ref_torch as RT
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    s, d = CFG["S"], CFG["D"]
    g = torch.Generator().manual_seed(0)
    mk = lambda: torch.randn(1, 1, s, d, generator=g)
    q, k, v, do = mk(), mk(), mk(), mk()
    RT.fwd_bwd(q[:, :, :256], k[:, :, :256], v[:, :, :256], do[:, :, :256], True)  # warm-up
    n, t_start = 0, time.perf_counter()
    while True:
        RT.fwd_bwd(q, k, v, do, CFG["causal"])
        n += 1
        el = time.perf_counter() - t_start
        if el > budget_s or n >= CFG["B"] * CFG["H"]:
            break
    fl = n * step_flops(1, 1, s, s, d, CFG["causal"])
    return {"value": fl / el / 1e12, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": "%d whole (batch, head) slices of configs[2] (S=4096, D=128, causal), "
                      "fwd+bwd by torch autograd in fp32 on CPU, %.1f s; scaled per FLOP" % (n, el)}


def run_ours(args):
    import tilelang_fa_v100 as fa
    from tilelang_fa_v100 import _ext
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    from tilelang_fa_v100 import sharding
    # Weak scaling: the global batch is world x configs[2]'s batch; rank r owns batch rows
    # [r*B, (r+1)*B) with all heads (a (batch x heads) shard, no data exchange).
    s, h, d, causal = CFG["S"], CFG["H"], CFG["D"], CFG["causal"]
    b0, b1 = sharding.dense_batch_slice(CFG["B"] * world, world, rank)
    b = b1 - b0
    dtype = torch.bfloat16
    with ClockSampler(local) as clk:
        ms, kern_ms, launches, tensors = time_dense(fa, dev, b, s, h, d, dtype, causal, args.steps,
                                                    args.warmup, seed=1000 + rank, dist=dist,
                                                    profile=True, clk=clk)
    clocks = clk.summary()
    err = check_dense(tensors, causal)
    del tensors
    if dist is not None:
        t = torch.tensor([ms, err], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)  # max over ranks (time and error)
        ms, err = float(t[0]), float(t[1])
    fl = step_flops(b, h, s, s, d, causal)
    value = world * fl / ms / 1e9  # TFLOP/s (ms -> s: /1e-3, TFLOP: /1e12)
    # as many e2e steps as timed steps: the first upload and the last download of a
    # pipelined run are exposed once, so short runs understate the streaming rate
    e2e_ms, h2d, d2h, link_ms = time_e2e(fa, dev, b, s, h, d, dtype, causal, args.steps, 2,
                                         seed=1000 + rank)
    if dist is not None:
        t = torch.tensor([e2e_ms, link_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms, link_ms = float(t[0]), float(t[1])
    peaks, src = measured_peaks()
    bwd_fl = 10.0 * d * visible_pairs(b, h, s, s, causal)
    achieved = bwd_fl / kern_ms / 1e9
    peak = peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops"))
    traffic = ncu_traffic("fa_bwd_dkdv_cfg3")
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: q/k/v/dO i.i.d. N(0,1) from per-rank seeds (no dataset involved)",
        "config": {"workload": WORKLOAD, "global_batch": b * world, "seq_len": s, "heads": h,
                   "head_dim": d, "causal": causal, "parallelism": "dp%d (batch x heads shards)" % world,
                   "l2": "inputs larger than L2 (q/k/v/dO 268 MB each > 126 MB)"},
        "clocks": clocks,
        "e2e": {"value": world * fl / e2e_ms / 1e9, "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms,
                "schedule": "per step: H2D of q,k,v,dO -> fwd+bwd -> D2H of out,dq,dk,dv; "
                            "uploads / downloads of neighbouring steps overlap the compute "
                            "(two copy streams, double-buffered device tensors)",
                "link_floor_ms": link_ms, "frac_of_link_floor": link_ms / e2e_ms,
                "link_floor": "the same step's uploads and downloads issued together with no "
                              "compute: the host link bounds e2e when frac_of_link_floor ~ 1"},
        "gpu_launches": launches,
        "roofline": {"kernel": "fa_bwd_dkdv_kernel (dense backward dK/dV + fused dQ)",
                     "bound": "tensor", "achieved": achieved, "peak": peak, "unit": UNIT,
                     "frac": achieved / peak, "traffic": traffic,
                     "peak_source": "%s bf16_tflops_sustained (kernel timed inside repeated steps)" % src,
                     "algorithmic": "10*D FLOP per visible (q,k) pair = %.4g FLOP per launch" % bwd_fl,
                     "kernel_ms": kern_ms},
        "check": {"max_abs_err_out_vs_fp32": err},
    }
    if not args.no_secondary and world == 1:  # secondary configs: single-GPU runs only
        sec = {}
        sms, _, _, tt = time_dense(fa, dev, 4, 2048, 16, 64, torch.float16, True, args.steps, 3,
                                   seed=7 + rank)
        del tt
        sec["cfg2_dense_fp16_B4_S2048_H16_D64"] = {
            "tflops": step_flops(4, 16, 2048, 2048, 64, True) / sms / 1e9, "ms": sms}
        # forward-only and backward-only rooflines on the headline shape
        q, k, v, do = dense_inputs(dev, b, s, h, d, dtype, 5)
        for _ in range(3):
            _ext.dense_forward(q, k, v, d ** -0.5, True)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        fts = []
        for _ in range(5):
            _ext.profile_next_launch(_ext.PROF_FWD, e0, e1)
            o, lse = _ext.dense_forward(q, k, v, d ** -0.5, True)
            torch.cuda.synchronize(dev)
            fts.append(e0.elapsed_time(e1))
        fwd_fl = 4.0 * d * visible_pairs(b, h, s, s, True)
        sec["cfg3_forward_kernel"] = {"tflops": fwd_fl / statistics.mean(fts) / 1e9,
                                      "ms": statistics.mean(fts),
                                      "frac_of_burst_peak": fwd_fl / statistics.mean(fts) / 1e9 / peaks.get("bf16_tflops", peak)}
        sec["cfg3_backward_dkdv_kernel"] = {"tflops": achieved, "ms": kern_ms,
                                            "frac_of_burst_peak": achieved / peaks.get("bf16_tflops", peak)}
        del q, k, v, do, o, lse
        # non-square: Sq = 1024, Skv = 4096 needs its own inputs
        qn, kn, vn, don = dense_inputs(dev, 8, 1024, 32, 128, dtype, 11)
        kn = torch.randn(8, 4096, 32, 128, device=dev).to(dtype)
        vn = torch.randn(8, 4096, 32, 128, device=dev).to(dtype)
        qn, kn, vn = (x.requires_grad_(True) for x in (qn, kn, vn))
        run_dense_steps(fa, qn, kn, vn, don, True, 3)
        torch.cuda.synchronize(dev)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        run_dense_steps(fa, qn, kn, vn, don, True, args.steps)
        t1.record()
        torch.cuda.synchronize(dev)
        nms = t0.elapsed_time(t1) / args.steps
        sec["cfg3_nonsquare_bf16_Sq1024_Skv4096"] = {
            "tflops": step_flops(8, 32, 1024, 4096, 128, True) / nms / 1e9, "ms": nms}
        del qn, kn, vn, don
        pms, ptf = time_paged(dev, args.steps, 3)
        sec["cfg4_paged_prefill_fp16"] = {"tflops": ptf, "ms": pms}
        dms, dgbs = time_decode(dev, args.steps, 3, seed=rank)
        sec["cfg5_decode_bf16_GBps"] = {"gbs": dgbs, "ms": dms,
                                        "frac_of_hbm": dgbs / peaks.get("hbm_gbs", 6538.6),
                                        "peak_source": src + " hbm_gbs"}
        d2ms, d2gbs = time_decode(dev, args.steps, 3, seed=rank, hkv=2, d=256, heads=32)
        sec["decode_bf16_H32_Hkv2_D256_GBps"] = {
            "gbs": d2gbs, "ms": d2ms, "frac_of_hbm": d2gbs / peaks.get("hbm_gbs", 6538.6),
            "note": "the reference's 32/2 D=256 test configuration, cfg5 length distribution"}
        kms, kgbs = time_kv_write(dev, args.steps, 3)
        sec["kv_cache_write_bf16_65536tok_Hkv8_D128_GBps"] = {
            "gbs": kgbs, "ms": kms, "frac_of_hbm": kgbs / peaks.get("hbm_gbs", 6538.6)}
        line["secondary"] = sec
        err_code = _ext.read_device_error(clear=True)
        line["device_error"] = list(err_code)
    if rank == 0:
        if world == 1:  # the host-core baseline is reported at N = 1 only
            line["cpu_baseline"] = cpu_baseline(budget_s=args.cpu_budget)
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


# --------------------------------------------------------------------------- reference arm
def run_reference(args):
    """The reference's own CPU-runnable implementation of the path (its PyTorch attention,
    restated in oracle/attention_ref_torch.py) timed on the host cores on bounded samples
    of the same workload; rank 0 alone runs under torchrun."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    from oracle import attention_ref_torch as RT
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    s, d = CFG["S"], CFG["D"]
    g = torch.Generator().manual_seed(0)
    mk = lambda: torch.randn(1, 1, s, d, generator=g)
    q, k, v, do = mk(), mk(), mk(), mk()
    for _ in range(args.warmup):
        RT.fwd_bwd(q[:, :, :512], k[:, :, :512], v[:, :, :512], do[:, :, :512], True)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        RT.fwd_bwd(q, k, v, do, CFG["causal"])
    el = (time.perf_counter() - t0) / args.steps
    fl = step_flops(1, 1, s, s, d, CFG["causal"])
    value = fl / el / 1e12
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": el * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": WORKLOAD, "global_batch": CFG["B"], "seq_len": s,
                       "heads": CFG["H"], "head_dim": d, "causal": CFG["causal"],
                       "parallelism": "host CPU, rank 0 only"},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                             "sample": "each step = one whole (batch, head) slice of configs[2] "
                                       "(S=4096, D=128, causal) fwd+bwd, torch autograd fp32"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_profile_case(args):
    """Small cases for ncu captures.  dense: B=2 of configs[2] (q/k/v/dO 67 MB each,
    268 MB together > the 126 MB L2), fwd+bwd steps.  decode: 64 sequences of
    configs[4] (L ~ U[512, 8192], ~1.1 GB of K/V pages), decode steps.  paged: configs[3]
    itself (q 134 MB > L2, K/V pages 34 MB), paged prefill steps."""
    import tilelang_fa_v100 as fa
    dev = torch.device("cuda", 0)
    if args.profile_case == "paged":
        ms, tflops = time_paged(dev, args.steps, args.warmup)
        print(json.dumps({"profile_case": "paged_cfg4_fp16", "ms": ms, "tflops": tflops}), flush=True)
        return
    if args.profile_case == "decode":
        q, kc, vc, bt, sl, nbytes = decode_problem(dev, 0, batch=64)
        for _ in range(args.warmup + args.steps):
            fa.tilelang_decode_forward(q, kc, vc, bt, sl)
        torch.cuda.synchronize(dev)
        print(json.dumps({"profile_case": "decode_B64_bf16", "bytes": nbytes}), flush=True)
        return
    b, s, h, d = 2, CFG["S"], CFG["H"], CFG["D"]
    ms, kern_ms, launches, _ = time_dense(fa, dev, b, s, h, d, torch.bfloat16, True, args.steps,
                                          args.warmup, seed=3, profile=True)
    print(json.dumps({"profile_case": "B2_S4096_H32_D128_bf16_causal", "ms_per_step": ms,
                      "dkdv_ms": kern_ms, "launches": launches}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-secondary", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--profile-case", choices=["dense", "decode", "paged"], default=None,
                    help="small case for ncu captures (no e2e / CPU / secondary)")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.profile_case:
        run_profile_case(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

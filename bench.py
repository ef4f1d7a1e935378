#!/usr/bin/env python
"""Benchmark of the B200 FlashAttention hot path (one JSON line on rank 0).

Headline: dense FA forward + backward TFLOP/s on the BASELINE configuration the target
is quoted on -- q/k/v [B=8, S=4096, H=32, D=128] bf16, causal;
a step is one forward + backward through the public API (tilelang_flash_attn_func and
autograd) over that batch.  FLOPs are counted on visible (query, key) pairs:
4 D per pair forward, 10 D per pair backward.

Scaling is weak: with N ranks the global problem is N x that batch, sharded by
(batch x heads) so every rank owns exactly one B=8 x H=32 shard; no collective runs in
the timed region.  value = N x per-rank FLOPs / max-over-ranks time.  Every input unit
(batch row, sequence) is drawn from its own seed, so the check can regenerate it on
rank 0 independently of the sharding: sampled outputs of every rank are broadcast to
rank 0 over NCCL and compared there with an fp32 torch reference (`check`).

Also reported in the same line: e2e (same metric through the public API with the
inputs copied from pinned host memory and out/dq/dk/dv copied back every step), the
roofline of the dominant kernel (the backward dK/dV kernel, timed live with CUDA
events on its launch stream), the CPU baseline (the reference's PyTorch attention in
fp32 on the host cores, on a bounded sample), clocks sampled during the timed region,
and secondary workloads at the same N (the other BASELINE configs: dense fp16 D=64,
non-square causal, paged GQA prefill sharded by sequence, split-KV decode GB/s sharded
by sequence with balanced token counts; the forward kernel and the whole backward).

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
# Every input unit of every workload -- a dense batch row, a paged or decode sequence --
# is drawn from its own seed (SEED_* + its global index), so the rank that owns a unit
# and rank 0, which regenerates it for the gathered check, produce the same values
# independently of how the units are sharded.
SEED_DENSE, SEED_DENSE2, SEED_NONSQ, SEED_PAGED, SEED_DECODE = 1000, 3000, 5000, 7000, 9000
SEED_VARLEN = 11000
U_BF16, U_F16 = 2.0 ** -8, 2.0 ** -11  # unit roundoff of the 16-bit input types


def reduce_max(dist, dev, *vals):
    """Element-wise max over ranks of host floats (identity on one GPU)."""
    if dist is None:
        return vals
    t = torch.tensor(vals, device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return tuple(float(x) for x in t)


def reduce_sum(dist, dev, *vals):
    if dist is None:
        return vals
    t = torch.tensor(vals, device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return tuple(float(x) for x in t)


def timed_ms(dev, dist, steps, fn):
    """ms per call of fn over `steps` calls, CUDA events on the current stream, barrier +
    synchronize on both sides, max over ranks."""
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        fn()
    t1.record()
    torch.cuda.synchronize(dev)
    return reduce_max(dist, dev, t0.elapsed_time(t1) / steps)[0]


def dense_row(dev, g, sq, skv, h, hk, d, dtype, seed_base):
    """q [Sq,H,D], k / v [Skv,Hk,D], dO [Sq,H,D] of global batch row g (its own seed)."""
    gen = torch.Generator(device=dev).manual_seed(seed_base + g)
    mk = lambda n, hh: torch.randn(n, hh, d, generator=gen, device=dev, dtype=torch.float32).to(dtype)
    return mk(sq, h), mk(skv, hk), mk(skv, hk), mk(sq, h)


def dense_shard(dev, g0, g1, sq, skv, h, hk, d, dtype, seed_base):
    """Batch rows [g0, g1) of the global problem as BSHD tensors (q, k, v, dO)."""
    q = torch.empty(g1 - g0, sq, h, d, dtype=dtype, device=dev)
    do = torch.empty_like(q)
    k = torch.empty(g1 - g0, skv, hk, d, dtype=dtype, device=dev)
    v = torch.empty_like(k)
    for i, g in enumerate(range(g0, g1)):
        q[i], k[i], v[i], do[i] = dense_row(dev, g, sq, skv, h, hk, d, dtype, seed_base)
    return q, k, v, do


def run_dense_steps(fa, q, k, v, do, causal, n, prof_events=None):
    """n fwd+bwd steps through the public API; optionally arms the dK/dV kernel events."""
    from tilelang_fa_v100 import _ext
    out = None
    for i in range(n):
        q.grad = k.grad = v.grad = None
        out = fa.tilelang_flash_attn_func(q, k, v, causal=causal)
        if prof_events is not None:
            _ext.profile_next_launch(_ext.PROF_BWD_DKDV, *prof_events[i])
        out.backward(do)
    return out


def time_dense(fa, dev, q, k, v, do, causal, steps, warmup, dist=None, profile=False, clk=None):
    """The headline step (fwd + bwd through the API) timed over `steps`; max over ranks.
    With profile, also the mean dK/dV kernel time from events around its launches."""
    from tilelang_fa_v100 import _ext
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
    run_dense_steps(fa, q, k, v, do, causal, steps, ev)
    t1.record()
    torch.cuda.synchronize(dev)
    if clk is not None:
        clk.mark_stop()
    launches = _ext.launch_count() - n0
    ms = t0.elapsed_time(t1) / steps
    kern_ms = statistics.mean(a.elapsed_time(b_) for a, b_ in ev) if profile else 0.0
    ms, kern_ms = reduce_max(dist, dev, ms, kern_ms)
    return ms, kern_ms, launches


class ErrStats:
    """Running error statistics of sampled outputs against a reference."""

    def __init__(self):
        self.d = {}

    def _get(self, name):
        return self.d.setdefault(name, {"n": 0, "max_abs_err": 0.0, "sum_abs_err": 0.0})

    def north_star(self, name, got, ref):
        """|got - ref| <= 2e-3 + 1e-2 |ref| elementwise (non-finite refs must match)."""
        got, ref = got.double(), ref.double()
        fin = torch.isfinite(ref)
        same_inf = ~fin & (got == ref)
        err = torch.where(fin, (got - ref.nan_to_num(0.0)).abs(), torch.zeros_like(got))
        err = torch.where(fin | same_inf, err, torch.full_like(err, float("inf")))
        excess = err - (2e-3 + 1e-2 * ref.nan_to_num(0.0, posinf=0.0, neginf=0.0).abs())
        e = self._get(name)
        e["n"] += err.numel()
        e["max_abs_err"] = max(e["max_abs_err"], float(err.max()))
        e["sum_abs_err"] += float(err[torch.isfinite(err)].sum())
        e["north_star_fail"] = e.get("north_star_fail", 0) + int((excess > 0).sum())
        e["north_star_max_excess"] = max(e.get("north_star_max_excess", -1.0), float(excess.max()))

    def grad(self, name, got, ref, u):
        """Gradients: max-abs error (north-star bar 1e-2) and the error left after the
        output's own rounding (err - u |ref|)."""
        got, ref = got.double(), ref.double()
        err = (got - ref).abs()
        e = self._get(name)
        e["n"] += err.numel()
        e["max_abs_err"] = max(e["max_abs_err"], float(err.max()))
        e["sum_abs_err"] += float(err.sum())
        e["gt_1e-2"] = e.get("gt_1e-2", 0) + int((err > 1e-2).sum())
        e["max_err_beyond_output_rounding"] = max(e.get("max_err_beyond_output_rounding", -1.0),
                                                  float((err - u * ref.abs()).max()))

    def bound(self, name, got, ref, bnd, atol=1e-4):
        """|got - ref| <= atol + bnd, the operand-rounding bound."""
        err = (got.double() - ref.double()).abs()
        e = self._get(name)
        e["rounding_bound_fail"] = e.get("rounding_bound_fail", 0) + int((err > atol + bnd.double()).sum())
        e["rounding_bound_max_ratio"] = max(e.get("rounding_bound_max_ratio", 0.0),
                                            float((err / (atol + bnd.double())).max()))

    def summary(self):
        out = {}
        for k, e in self.d.items():
            e = dict(e)
            e["mean_abs_err"] = e.pop("sum_abs_err") / max(1, e["n"])
            if "north_star_fail" in e:
                e["north_star_fail_frac"] = e["north_star_fail"] / max(1, e["n"])
            out[k] = e
        return out


def _bcast(dist, t, src):
    if dist is not None:
        dist.broadcast(t, src=src)
    return t


def check_dense(fa, dev, dist, rank, world, rows, tensors, sq, skv, h, d, dtype, causal, seed_base):
    """Gathered check of the headline step.  Sampled (batch row, head) slices -- one on
    every rank plus the first and last of the global problem -- are broadcast from the
    rank that owns them; rank 0 regenerates that row's inputs from its seed and compares
    out, lse, dQ, dK, dV with the fp32 torch reference (TF32 off).  Returns the
    statistics on rank 0 (None elsewhere)."""
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from slice_ref import slice_ref_2d
    q, k, v, do = tensors
    qd, kd, vd = (x.detach().clone().requires_grad_(True) for x in (q, k, v))
    out, lse, _ = fa.tilelang_flash_attn_func(qd, kd, vd, causal=causal, return_attn_probs=True)
    out.backward(do)
    torch.cuda.synchronize(dev)
    u = U_BF16 if dtype == torch.bfloat16 else U_F16
    n = world * rows
    samples = [(0, 0), (n - 1, h - 1)] + [(r * rows + rows // 2, (11 * r + 5) % h) for r in range(world)]
    samples = list(dict.fromkeys(samples))
    st = ErrStats()
    for g, hh in samples:
        owner = g // rows
        shapes = [((sq, d), dtype), ((sq,), torch.float32), ((sq, d), dtype), ((skv, d), dtype),
                  ((skv, d), dtype)]
        if rank == owner:
            li = g - rank * rows
            pack = [out[li, :, hh], lse[li, hh], qd.grad[li, :, hh], kd.grad[li, :, hh],
                    vd.grad[li, :, hh]]
            pack = [t.detach().contiguous() for t in pack]
        else:
            pack = [torch.empty(s, dtype=dt, device=dev) for s, dt in shapes]
        pack = [_bcast(dist, t, owner) for t in pack]
        if rank != 0:
            continue
        qg, kg, vg, dog = dense_row(dev, g, sq, skv, h, h, d, dtype, seed_base)
        o_s, lse_s, dq_s, dk_s, dv_s = pack
        r = slice_ref_2d(qg[:, hh], kg[:, hh], vg[:, hh], dog[:, hh], o_s, causal, u)
        st.north_star("out", o_s, r["out"])
        st.north_star("lse", lse_s, r["lse"])
        st.bound("out", o_s, r["out"], r["bo"])
        for nm, got in (("dq", dq_s), ("dk", dk_s), ("dv", dv_s)):
            st.grad(nm, got, r[nm], u)
            st.bound(nm, got, r[nm + "_f"], r["b" + nm[1]])
    del qd, kd, vd, out, lse
    if rank != 0:
        return None
    res = st.summary()
    res["samples"] = ["batch %d head %d (rank %d)" % (g, hh, g // rows) for g, hh in samples]
    res["criteria"] = (
        "fp32 torch on the GPU (TF32 off), inputs regenerated on rank 0 from each row's seed; "
        "out / lse: north-star |d| <= 2e-3 + 1e-2 |ref| (fail count, fraction, max excess); "
        "grads: max-abs vs the 1e-2 bar (gt_1e-2) and the error beyond the output's own "
        "rounding u|ref| (u = %g); rounding_bound_*: |d| <= 1e-4 + u (sum |operand| ...) against "
        "the reference with D = rowsum(dO * O) from the returned O -- the worst case of rounding "
        "P, dS and the outputs to %s" % (u, str(dtype).split(".")[-1]))
    return res


def time_e2e(fa, dev, q, k, v, do, causal, steps, warmup):
    """Public API with host buffers.  Every step uploads its q, k, v, dO from pinned host
    memory, runs fwd + bwd and downloads its out, dq, dk, dv into pinned host memory.
    Neighbouring steps overlap the way a training loop that streams its batches does:
    the upload of step k+1 and the download of step k-1 run on two copy streams while
    step k computes (device buffers double-buffered, events order each slot's reuse)."""
    host_in = [x.detach().cpu().pin_memory() for x in (q, k, v, do)]
    shape, dtype, nb = tuple(q.shape), q.dtype, 2
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
    nbytes = q.numel() * q.element_size()
    return ms, 4 * nbytes, 4 * nbytes, link_ms


# ---- paged prefill and decode: sequences with their own seeds
def seq_inputs(dev, i, q_len, kv_len, h, hkv, d, dtype, seed_base):
    """q [q_len,H,D] (the sequence's last q_len rows), k / v [kv_len,Hkv,D] of sequence i."""
    gen = torch.Generator(device=dev).manual_seed(seed_base + i)
    mk = lambda n, hh: torch.randn(n, hh, d, generator=gen, device=dev, dtype=torch.float32).to(dtype)
    return mk(q_len, h), mk(kv_len, hkv), mk(kv_len, hkv)


def paged_problem(dev, seqs, q_lens, kv_lens, h, hkv, d, page, dtype, seed_base, perm_seed,
                  max_blocks=None):
    """The vLLM-layout inputs of the given sequences (global indices): every sequence's
    pages are scattered over the rank's page pool by a seeded permutation; block-table
    rows are padded with page 0 up to max_blocks."""
    pps = [-(-int(n) // page) for n in kv_lens]
    total = max(1, sum(pps))
    perm = torch.from_numpy(np.random.default_rng(perm_seed).permutation(total).astype(np.int64))
    mb = max(pps) if max_blocks is None else max_blocks
    bt = torch.zeros(len(seqs), mb, dtype=torch.int32)
    kc = torch.zeros(total, page, hkv, d, dtype=dtype, device=dev)
    vc = torch.zeros_like(kc)
    q = torch.empty(int(sum(q_lens)), h, d, dtype=dtype, device=dev)
    c = t = 0
    for j, i in enumerate(seqs):
        pages = perm[c:c + pps[j]]
        bt[j, :pps[j]] = pages.to(torch.int32)
        c += pps[j]
        qi, ki, vi = seq_inputs(dev, i, int(q_lens[j]), pps[j] * page, h, hkv, d, dtype, seed_base)
        q[t:t + int(q_lens[j])] = qi
        t += int(q_lens[j])
        pg = pages.to(dev)
        kc[pg] = ki.view(pps[j], page, hkv, d)
        vc[pg] = vi.view(pps[j], page, hkv, d)
    qsl = torch.tensor(np.concatenate([[0], np.cumsum(q_lens)]), dtype=torch.int32, device=dev)
    sl = torch.tensor(np.asarray(kv_lens), dtype=torch.int32, device=dev)
    return q, kc, vc, bt.to(dev), sl, qsl, total


PAGED = dict(seqs=16, q_len=1024, kv_len=1024, h=32, hkv=8, d=128, page=16)  # configs[3]
# head_dim 512 paged prefill (the reference's _BEST_CONFIGS[512] entry), configs[3]'s
# sequence shape with 16 query / 4 kv heads
PAGED512 = dict(seqs=16, q_len=1024, kv_len=1024, h=16, hkv=4, d=512, page=16)


def paged_run(dev, dist, rank, world, steps, warmup, c=PAGED, dtype=torch.float16):
    """configs[3] (or `c`), weak: every rank runs 16 x 1024-token sequences (global
    sequences 16 r .. 16 r + 15, contiguous); returns aggregate TFLOP/s, ms and the
    gathered check."""
    import tilelang_fa_v100 as fa
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from slice_ref import sequence_ref
    n = c["seqs"]
    seqs = list(range(rank * n, (rank + 1) * n))
    q, kc, vc, bt, sl, qsl, _ = paged_problem(dev, seqs, [c["q_len"]] * n, [c["kv_len"]] * n,
                                              c["h"], c["hkv"], c["d"], c["page"], dtype,
                                              SEED_PAGED, 11 + rank)
    pkl = torch.zeros(n, dtype=torch.int32, device=dev)
    out = torch.empty_like(q)
    lse = torch.empty(c["h"], q.shape[0], device=dev)
    run = lambda: fa.tilelang_paged_forward(q, kc, vc, bt, sl, qsl, pkl, out=out)
    for _ in range(warmup):
        run()
    ms = timed_ms(dev, dist, steps, run)
    out, lse = fa.tilelang_paged_forward(q, kc, vc, bt, sl, qsl, pkl, out=out)
    torch.cuda.synchronize(dev)
    flops = world * 4.0 * c["d"] * visible_pairs(n, c["h"], c["q_len"], c["kv_len"], True)
    # gathered check: the first and last sequence of the global batch + one per rank
    total = world * n
    samples = list(dict.fromkeys([0, total - 1] + [r * n + (5 * r + 3) % n for r in range(world)]))
    st = ErrStats()
    for i in samples:
        owner = i // n
        if rank == owner:
            j = i - owner * n
            pack = [out[j * c["q_len"]:(j + 1) * c["q_len"]].contiguous(),
                    lse[:, j * c["q_len"]:(j + 1) * c["q_len"]].contiguous()]
        else:
            pack = [torch.empty(c["q_len"], c["h"], c["d"], dtype=dtype, device=dev),
                    torch.empty(c["h"], c["q_len"], device=dev)]
        pack = [_bcast(dist, t, owner) for t in pack]
        if rank != 0:
            continue
        qi, ki, vi = seq_inputs(dev, i, c["q_len"], c["kv_len"], c["h"], c["hkv"], c["d"],
                                dtype, SEED_PAGED)
        ro, rl = sequence_ref(qi, ki, vi, c["kv_len"] - c["q_len"], True)
        st.north_star("out", pack[0], ro)
        st.north_star("lse", pack[1], rl)
    del q, kc, vc, out, lse
    chk = None
    if rank == 0:
        chk = st.summary()
        chk["samples"] = ["sequence %d (rank %d)" % (i, i // n) for i in samples]
    return flops / ms / 1e9, ms, chk


VARLEN = dict(seqs=16, lo=256, hi=4096, h=32, d=128)  # packed mixed-length batch per rank


def varlen_run(dev, dist, rank, world, steps, warmup):
    """Dense varlen (FA2 flash_attn_varlen_func), weak: every rank packs 16 causal
    sequences of L ~ U[256, 4096] tokens (global sequences 16 r .. 16 r + 15, each from
    its own seed), bf16, 32 heads, D 128; a step is the forward and the backward through
    the C ABI.  Returns aggregate TFLOP/s (14 D per visible pair of every rank's
    sequences over the slowest rank's time), ms, rank 0's check of one head of its first
    and last sequence against the fp32 reference, and rank 0's lengths."""
    from tilelang_fa_v100 import _ext
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from slice_ref import slice_ref_2d
    c = VARLEN
    n, h, d = c["seqs"], c["h"], c["d"]
    lens = np.random.default_rng(SEED_VARLEN).integers(c["lo"], c["hi"] + 1, size=world * n)
    mine = [int(x) for x in lens[rank * n:(rank + 1) * n]]
    rows = [dense_row(dev, rank * n + i, L, L, h, h, d, torch.bfloat16, SEED_VARLEN)
            for i, L in enumerate(mine)]
    q, k, v, do = (torch.cat([r[j] for r in rows]) for j in range(4))
    del rows
    cu = torch.tensor(np.concatenate([[0], np.cumsum(mine)]), dtype=torch.int32, device=dev)
    mx, sc = max(mine), d ** -0.5
    state = {}

    def step():
        o, lse = _ext.varlen_forward(q, k, v, cu, cu, mx, mx, sc, True)
        state["g"] = _ext.varlen_backward(q, k, v, o, do, lse, cu, cu, mx, mx, sc, True)
        state["o"] = o
    for _ in range(warmup):
        step()
    ms = timed_ms(dev, dist, steps, step)
    pairs = h * sum(int(L) * (int(L) + 1) // 2 for L in lens)  # every rank's sequences
    chk = None
    if rank == 0:
        st = ErrStats()
        o, (dq, dk, dv) = state["o"], state["g"]
        for i in (0, n - 1):
            a, b_ = int(cu[i]), int(cu[i + 1])
            r = slice_ref_2d(q[a:b_, 0], k[a:b_, 0], v[a:b_, 0], do[a:b_, 0], o[a:b_, 0], True,
                             2.0 ** -8)
            st.north_star("out", o[a:b_, 0], r["out"])
            st.bound("out", o[a:b_, 0], r["out"], r["bo"])
            for nm, g_, bn in (("dq", dq, "bq"), ("dk", dk, "bk"), ("dv", dv, "bv")):
                st.grad(nm, g_[a:b_, 0], r[nm + "_f"], 2.0 ** -8)
                st.bound(nm, g_[a:b_, 0], r[nm + "_f"], r[bn])
        chk = st.summary()
        chk["samples"] = ["sequence %d head 0 (L %d)" % (i, mine[i]) for i in (0, n - 1)]
    del q, k, v, do, state
    return 14.0 * d * pairs / ms / 1e9, ms, chk, mine


def decode_lengths(world, batch=256, seed=0):
    """Global KV lengths of configs[4] (L ~ U[512, 8192]) for world x batch sequences."""
    return np.random.default_rng(seed).integers(512, 8193, size=world * batch).astype(np.int32)


def decode_problem(dev, rank, world, batch=256, hkv=8, d=128, heads=32, seed_base=SEED_DECODE):
    """Rank `rank`'s share of world x batch decode sequences, balanced longest-first by
    token count (sharding.balance_sequences).  Returns the inputs, the rank's sequence
    ids and the HBM bytes one decode reads and writes (K/V actually read + q + out +
    block table)."""
    from tilelang_fa_v100 import sharding
    lens = decode_lengths(world, batch)
    owned = sharding.balance_sequences(lens, world)
    mine = owned[rank]
    q, kc, vc, bt, sl, _, total = paged_problem(dev, mine, [1] * len(mine), lens[mine], heads,
                                                hkv, d, 16, torch.bfloat16, seed_base,
                                                100 + rank, max_blocks=512)
    nbytes = int(lens[mine].sum()) * hkv * d * 2 * 2 + 2 * len(mine) * heads * d * 2 + total * 4
    return q, kc, vc, bt, sl, nbytes, mine, owned, lens


FP8_SCALE = 1.0 / 64  # e4m3 cache scale for N(0,1) keys / values: |x| / scale stays < 448


def to_e4m3(x):
    """The fp8 cache a serving engine would hold for x (x / scale, saturated)."""
    return (x.float() / FP8_SCALE).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)


def decode_run(dev, dist, rank, world, steps, warmup, hkv=8, d=128, heads=32, check=True,
               fp8=False):
    """configs[4] at N GPUs (weak: N x 256 sequences, sharded by sequence with balanced
    token counts); fp8: the same sequences in e4m3 caches with per-tensor scales.  Returns
    aggregate GB/s, ms, the gathered check and the max/mean per-rank token load."""
    import tilelang_fa_v100 as fa
    q, kc, vc, bt, sl, nbytes, mine, owned, lens = decode_problem(dev, rank, world, hkv=hkv, d=d,
                                                                  heads=heads)
    kw = {}
    if fp8:
        kc, vc = to_e4m3(kc), to_e4m3(vc)
        kw = dict(k_scale=FP8_SCALE, v_scale=FP8_SCALE)
        nbytes -= int(lens[mine].sum()) * hkv * d * 2  # one byte per cached element, not two
    run = lambda: fa.tilelang_decode_forward(q, kc, vc, bt, sl, **kw)
    for _ in range(warmup):
        run()
    ms = timed_ms(dev, dist, steps, run)
    tot_bytes = reduce_sum(dist, dev, float(nbytes))[0]
    loads = [int(lens[o].sum()) for o in owned]
    res_chk = None
    if check:
        sys.path.insert(0, os.path.join(ROOT, "tests"))
        from slice_ref import sequence_ref
        out = run()
        torch.cuda.synchronize(dev)
        samples = list(dict.fromkeys([0, len(lens) - 1] + [o[len(o) // 2] for o in owned]))
        st = ErrStats()
        for i in samples:
            owner = next(r for r, o in enumerate(owned) if i in o)
            if rank == owner:
                pack = out[mine.index(i)].contiguous()
            else:
                pack = torch.empty(heads, d, dtype=torch.bfloat16, device=dev)
            pack = _bcast(dist, pack, owner)
            if rank != 0:
                continue
            L = int(lens[i])
            qi, ki, vi = seq_inputs(dev, i, 1, -(-L // 16) * 16, heads, hkv, d, torch.bfloat16,
                                    SEED_DECODE)
            if fp8:  # the reference attends over the dequantised cache
                ki, vi = (to_e4m3(x).float() * FP8_SCALE for x in (ki, vi))
            ro, _ = sequence_ref(qi, ki[:L], vi[:L], 0, False)
            st.north_star("out", pack, ro[0])
        if rank == 0:
            res_chk = st.summary()
            res_chk["samples"] = ["sequence %d (rank %d)" % (i, next(r for r, o in enumerate(owned) if i in o))
                                  for i in samples]
    del q, kc, vc
    balance = {"max_rank_tokens": max(loads), "mean_rank_tokens": sum(loads) / len(loads)}
    return tot_bytes / ms / 1e6, ms, res_chk, balance


def time_kv_write(dev, dist, steps, warmup, tokens=65536, hkv=8, d=128, page=16):
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
    ms = timed_ms(dev, dist, steps, run)
    nbytes = 2 * 2 * tokens * hkv * d * 2
    return ms, nbytes / ms / 1e6


def kernel_events_ms(dev, dist, kind, fn, reps=5):
    """Mean duration of one library kernel (events the library records around its
    launch on the launch stream), max over ranks."""
    from tilelang_fa_v100 import _ext
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ts = []
    for _ in range(reps):
        _ext.profile_next_launch(kind, e0, e1)
        fn()
        torch.cuda.synchronize(dev)
        ts.append(e0.elapsed_time(e1))
    return reduce_max(dist, dev, statistics.mean(ts))[0]


def peak_for_clocks(peaks, clocks):
    """Burst bf16 peak when the timed region ran at max SM clock with no power cap, the
    sustained one otherwise (a region long enough to hit the 1000 W cap)."""
    mhz, mx = clocks.get("sm_mhz"), clocks.get("sm_max_mhz")
    burst = (mhz is not None and mx and mhz >= 0.97 * mx
             and "sw_power_cap" not in (clocks.get("reasons") or []))
    if burst:
        return peaks["bf16_tflops"], "bf16_tflops (burst): the timed region ran at %.0f of %.0f MHz with no power cap" % (mhz, mx)
    return peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"]), \
        "bf16_tflops_sustained: the timed region ran below max clock or under sw_power_cap"


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
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    from tilelang_fa_v100 import sharding
    peaks, src = measured_peaks()
    hbm = peaks.get("hbm_gbs", 6538.6)
    # Weak scaling: the global batch is world x configs[2]'s batch; rank r owns batch rows
    # [r*B, (r+1)*B) with all heads (a (batch x heads) shard, no data exchange).
    s, h, d, causal = CFG["S"], CFG["H"], CFG["D"], CFG["causal"]
    g0, g1 = sharding.dense_batch_slice(CFG["B"] * world, world, rank)
    b = g1 - g0
    dtype = torch.bfloat16
    tensors = dense_shard(dev, g0, g1, s, s, h, h, d, dtype, SEED_DENSE)
    with ClockSampler(local) as clk:
        ms, kern_ms, launches = time_dense(fa, dev, *tensors, causal, args.steps, args.warmup,
                                           dist=dist, profile=True, clk=clk)
    clocks = clk.summary()
    fl = step_flops(b, h, s, s, d, causal)
    value = world * fl / ms / 1e9  # TFLOP/s (ms -> s: /1e-3, TFLOP: /1e12)
    check = check_dense(fa, dev, dist, rank, world, b, tensors, s, s, h, d, dtype, causal,
                        SEED_DENSE)
    # as many e2e steps as timed steps: the first upload and the last download of a
    # pipelined run are exposed once, so short runs understate the streaming rate
    e2e_ms, h2d, d2h, link_ms = time_e2e(fa, dev, *tensors, causal, args.steps, 2)
    e2e_ms, link_ms = reduce_max(dist, dev, e2e_ms, link_ms)
    bwd_fl = 10.0 * d * visible_pairs(b, h, s, s, causal)
    achieved = bwd_fl / kern_ms / 1e9
    peak, peak_why = peak_for_clocks(peaks, clocks)
    traffic = ncu_traffic("fa_bwd_dkdv_cfg3")
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: q/k/v/dO i.i.d. N(0,1), each batch row from its own seed (no dataset involved)",
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
                     "peak_source": "%s %s" % (src, peak_why),
                     "algorithmic": "10*D FLOP per visible (q,k) pair = %.4g FLOP per launch" % bwd_fl,
                     "kernel_ms": kern_ms},
        "check": check,
    }
    if not args.no_secondary:
        sec = {}
        burst = peaks["bf16_tflops"]
        # forward kernel alone and the whole backward (prep + dK/dV + dQ convert) on the
        # headline shard; each rank times its own, max over ranks
        q, k, v, do = tensors
        out, lse = _ext.dense_forward(q, k, v, d ** -0.5, True)
        fwd_ms = kernel_events_ms(dev, dist, _ext.PROF_FWD,
                                  lambda: _ext.dense_forward(q, k, v, d ** -0.5, True))
        fwd_fl = 4.0 * d * visible_pairs(b, h, s, s, True)
        sec["cfg3_forward_kernel"] = {"tflops": world * fwd_fl / fwd_ms / 1e9, "ms": fwd_ms,
                                      "frac_of_burst_peak": fwd_fl / fwd_ms / 1e9 / burst}
        for _ in range(2):
            _ext.dense_backward(q, k, v, out, do, lse, d ** -0.5, True)
        bwd_ms = timed_ms(dev, dist, 5, lambda: _ext.dense_backward(q, k, v, out, do, lse,
                                                                    d ** -0.5, True))
        sec["cfg3_backward_total"] = {
            "tflops": world * bwd_fl / bwd_ms / 1e9, "ms": bwd_ms,
            "frac_of_burst_peak": bwd_fl / bwd_ms / 1e9 / burst,
            "what": "prep (row dot) + dK/dV (+ fused dQ adds) + dQ convert, event-timed on the "
                    "stream, 10*D FLOP per visible pair"}
        sec["cfg3_backward_dkdv_kernel"] = {"tflops": world * achieved, "ms": kern_ms,
                                            "frac_of_burst_peak": achieved / burst}
        del q, k, v, do, out, lse, tensors
        # fp16 D = 64, B = 4 rows per rank
        t2 = dense_shard(dev, 4 * rank, 4 * rank + 4, 2048, 2048, 16, 16, 64, torch.float16,
                         SEED_DENSE2)
        sms, _, _ = time_dense(fa, dev, *t2, True, args.steps, 3, dist=dist)
        sec["cfg2_dense_fp16_B4_S2048_H16_D64"] = {
            "tflops": world * step_flops(4, 16, 2048, 2048, 64, True) / sms / 1e9, "ms": sms}
        del t2
        # configs[2] non-square variant: Sq = 1024, Skv = 4096, 8 rows per rank
        tn = dense_shard(dev, g0, g1, 1024, 4096, 32, 32, 128, dtype, SEED_NONSQ)
        nms, _, _ = time_dense(fa, dev, *tn, True, args.steps, 3, dist=dist)
        sec["cfg3_nonsquare_bf16_Sq1024_Skv4096"] = {
            "tflops": world * step_flops(b, 32, 1024, 4096, 128, True) / nms / 1e9, "ms": nms}
        del tn
        ptf, pms, pchk = paged_run(dev, dist, rank, world, args.steps, 3)
        sec["cfg4_paged_prefill_fp16"] = {"tflops": ptf, "ms": pms,
                                          "frac_of_burst_peak": ptf / world / burst,
                                          "sharding": "16 sequences per rank (contiguous)",
                                          "check": pchk}
        dgbs, dms, dchk, bal = decode_run(dev, dist, rank, world, args.steps, 3)
        sec["cfg5_decode_bf16_GBps"] = {"gbs": dgbs, "ms": dms,
                                        "frac_of_hbm": dgbs / world / hbm,
                                        "peak_source": src + " hbm_gbs",
                                        "sharding": "256 sequences per rank, balanced longest-first "
                                                    "by token count", "balance": bal,
                                        "check": dchk}
        f8gbs, f8ms, f8chk, _ = decode_run(dev, dist, rank, world, args.steps, 3, fp8=True)
        sec["cfg5_decode_fp8kv_GBps"] = {
            "gbs": f8gbs, "ms": f8ms, "frac_of_hbm": f8gbs / world / hbm,
            "speedup_vs_bf16_cache": dms / f8ms,
            "note": "configs[4] sequences with e4m3 K/V caches (per-tensor scale 1/64); bytes "
                    "count one byte per cached element; checked against the dequantised cache",
            "check": f8chk}
        p5tf, p5ms, p5chk = paged_run(dev, dist, rank, world, args.steps, 3, c=PAGED512)
        sec["paged_prefill_fp16_D512_16x1024_H16_Hkv4"] = {
            "tflops": p5tf, "ms": p5ms, "frac_of_burst_peak": p5tf / world / burst,
            "note": "useful FLOPs (4*D per visible pair); each q block computes S twice "
                    "(half-width output items), so executed tensor work is 1.5x",
            "check": p5chk}
        d5gbs, d5ms, _, _ = decode_run(dev, dist, rank, world, args.steps, 3, hkv=4, d=512,
                                       heads=16, check=False)
        sec["decode_bf16_H16_Hkv4_D512_GBps"] = {
            "gbs": d5gbs, "ms": d5ms, "frac_of_hbm": d5gbs / world / hbm,
            "note": "configs[4] length distribution, head_dim 512"}
        d2gbs, d2ms, _, _ = decode_run(dev, dist, rank, world, args.steps, 3, hkv=1, d=256,
                                       heads=8, check=False)
        sec["decode_bf16_H8_Hkv1_D256_GBps"] = {
            "gbs": d2gbs, "ms": d2ms, "frac_of_hbm": d2gbs / world / hbm,
            "note": "the reference's synthetic 8/1 D=256 configuration, configs[4] length "
                    "distribution"}
        vtf, vms, vchk, vlens = varlen_run(dev, dist, rank, world, args.steps, 3)
        sec["varlen_fwd_bwd_bf16_16seq_U256_4096_H32_D128_causal"] = {
            "tflops": vtf, "ms": vms, "frac_of_burst_peak": vtf / world / burst,
            "note": "dense varlen (FA2 flash_attn_varlen_func): forward + backward of a packed "
                    "mixed-length batch per rank through the C ABI; 14*D FLOP per visible "
                    "pair; ranks draw their own lengths, so their work differs",
            "tokens_rank0": int(sum(vlens)), "check": vchk}
        kms, kgbs = time_kv_write(dev, dist, args.steps, 3)
        sec["kv_cache_write_bf16_65536tok_Hkv8_D128_GBps"] = {
            "gbs": world * kgbs, "ms": kms, "frac_of_hbm": kgbs / hbm}
        line["secondary"] = sec
        code = _ext.read_device_error(clear=True)
        line["device_error"] = list(code)
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
    itself (q 134 MB > L2, K/V pages 34 MB), paged prefill steps.  paged512: the head_dim
    512 paged workload (q 268 MB, K/V pages 134 MB)."""
    import tilelang_fa_v100 as fa
    dev = torch.device("cuda", 0)
    if args.profile_case == "paged":
        tflops, ms, _ = paged_run(dev, None, 0, 1, args.steps, args.warmup)
        print(json.dumps({"profile_case": "paged_cfg4_fp16", "ms": ms, "tflops": tflops}), flush=True)
        return
    if args.profile_case == "paged512":  # the head_dim 512 secondary line's workload
        tflops, ms, _ = paged_run(dev, None, 0, 1, args.steps, args.warmup, c=PAGED512)
        print(json.dumps({"profile_case": "paged_D512_16x1024_H16_Hkv4_fp16", "ms": ms,
                          "tflops": tflops}), flush=True)
        return
    if args.profile_case == "decode":
        q, kc, vc, bt, sl, nbytes, _, _, _ = decode_problem(dev, 0, 1, batch=64)
        for _ in range(args.warmup + args.steps):
            fa.tilelang_decode_forward(q, kc, vc, bt, sl)
        torch.cuda.synchronize(dev)
        print(json.dumps({"profile_case": "decode_B64_bf16", "bytes": nbytes}), flush=True)
        return
    if args.profile_case == "d64":  # configs[1] itself: fp16 [4, 2048, 16, 64] causal
        t = dense_shard(dev, 0, 4, 2048, 2048, 16, 16, 64, torch.float16, SEED_DENSE2)
        ms, kern_ms, launches = time_dense(fa, dev, *t, True, args.steps, args.warmup, profile=True)
        print(json.dumps({"profile_case": "cfg2_B4_S2048_H16_D64_fp16_causal", "ms_per_step": ms,
                          "dkdv_ms": kern_ms, "launches": launches}), flush=True)
        return
    if args.profile_case == "d256":  # head_dim 256: bf16 [2, 4096, 16, 256] causal (67 MB / tensor)
        t = dense_shard(dev, 0, 2, 4096, 4096, 16, 16, 256, torch.bfloat16, SEED_DENSE)
        ms, kern_ms, launches = time_dense(fa, dev, *t, True, args.steps, args.warmup, profile=True)
        print(json.dumps({"profile_case": "B2_S4096_H16_D256_bf16_causal", "ms_per_step": ms,
                          "dkdv_ms": kern_ms, "launches": launches}), flush=True)
        return
    s, h, d = CFG["S"], CFG["H"], CFG["D"]
    t = dense_shard(dev, 0, 2, s, s, h, h, d, torch.bfloat16, SEED_DENSE)
    ms, kern_ms, launches = time_dense(fa, dev, *t, True, args.steps, args.warmup, profile=True)
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
    ap.add_argument("--profile-case", choices=["dense", "decode", "paged", "paged512", "d64", "d256"], default=None,
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

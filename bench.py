#!/usr/bin/env python
"""Benchmark of the SF37 KV-cache hot path on B200.

Headline: one decode step of a synthetic 48-layer stack,
64 query heads / 8 KV heads, head_dim 128, f16 KV caches with 32768 cached
positions, batch 1.  Per layer and step: append one K/V row, then GQA
attention over 32769+ positions (the position advances every step).  One
step = one sf37kv_decode() call over all 48 layers.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

N > 1 (under torchrun): KV heads sharded 8/N per GPU; every rank's decode
kernels store their output heads into all ranks' buffers over NVLink (peer
memory); total work is fixed (strong scaling).  After the timed region the
gathered outputs are checked (bit-equal to an NCCL all-gather of the local
outputs, and within the north-star tolerance of the CPU oracle) and the line
carries "parity"; a mismatch exits non-zero.

The default line also carries, after the headline's timed region, one
compact object per other BASELINE config ("configs": cfg1, cfg3, cfg4,
cfg5a, cfg5b) and the engine's per-layer call pattern ("per_layer"), each
with its own timing, roofline fraction and clock record.

Output: one JSON line on rank 0 (see the repository's build contract).
"""
import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode-attn KV-read GB/s (% of 8 TB/s) and tokens/s at 32K ctx, 1/2/4/8 B200"
QH, KVH, HD, CTX = 64, 8, 128, 32768
EMBD = 4096  # model width: o_proj output (sf37.c:36)
LAYERS = 48  # --layers overrides (profiling runs use a small stack)
WORKLOADS = {
    "decode": "cfg2: 48-layer decode step (append + GQA attention) at 32768 cached tokens, 64 Q / 8 KV heads, "
              "d 128, batch 1",
    "long": "cfg5a: 48-layer decode step at 131072 cached tokens, KV heads sharded across GPUs",
    "hybrid": "cfg3: 48 layers, 12 full (il%4==0) + 36 sliding (window 512, 512-row ring), decode after a "
              "65536-token prefix",
}
# north-star tolerance for attention outputs (elementwise: abs or rel)
ATOL, RTOL = 2e-3, 1e-2


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def _tensor_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return float(json.load(open(p)).get("bf16_tflops_sustained", 1400.0)), "measured sustained"
    return 1400.0, "fallback sustained"


def _traffic_from_profiles(name):
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu
    summary (a line 'traffic_bytes_per_launch: N'), or None."""
    p = os.path.join(ROOT, "profiles", name)
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.strip().startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi sampling during a timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            time.sleep(0.3)  # let nvidia-smi start before the timed region
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.proc = None

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def _dev():
    import torch
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    return dev


def _max_over_ranks(x, world, dev):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(world, dev):
    import torch
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize(dev)


def decode_config(wl, world, prep=False, oproj=False, gather="peer"):
    """The `config` object of a decode line; the reference arm prints the
    same object for the same workload and N."""
    return {"workload": WORKLOADS[wl], "layers": LAYERS,
            "ctx": {"decode": CTX, "long": 131072, "hybrid": 65536}[wl],
            "q_heads": QH, "kv_heads": KVH, "head_dim": HD, "kv_heads_per_gpu": KVH // world,
            "qk_prep_fused": bool(prep), "oproj_q8_0": bool(oproj),
            "parallelism": f"kv-head shard x{world}" + (
                "" if world == 1 else " + row-parallel o_proj, partial sums reduced over peer memory" if oproj
                else " + NCCL all-gather" if gather == "nccl"
                else " + output gather by peer-memory stores from the decode kernels"),
            "l2": "no flush needed: every step reads >= 3.4 GB of KV, far more than the 126 MB L2"}


# ---------------------------------------------------------------- CPU legs
_CPU_DATA = {}


def cpu_reference_step_time(threads, n_layers, rows):
    """One decode step of `n_layers` layers through the reference's own CPU
    code (kv_cache_push + attention_decode + gate, oracle/_ref), spread over
    `threads` threads (contiguous blocks of layers per thread).  Each layer
    has its own fp32 cache (the reference's only cache type) holding
    f16-valued N(0,1) data.  Returns seconds."""
    import oracle
    R = oracle.ref()
    kd = KVH * HD
    cap = rows
    key = (n_layers, rows)
    if key not in _CPU_DATA:
        _CPU_DATA.clear()
        rng = np.random.default_rng(0)
        k0 = rng.standard_normal((cap, kd), dtype=np.float32).astype(np.float16).astype(np.float32)
        v0 = rng.standard_normal((cap, kd), dtype=np.float32).astype(np.float16).astype(np.float32)
        d = dict(k=[k0] + [k0.copy() for _ in range(n_layers - 1)],
                 v=[v0] + [v0.copy() for _ in range(n_layers - 1)],
                 q=[rng.standard_normal((QH, HD), dtype=np.float32) for _ in range(n_layers)],
                 g=[rng.standard_normal((QH,), dtype=np.float32) for _ in range(n_layers)],
                 o=[np.zeros((QH, HD), np.float32) for _ in range(n_layers)],
                 kn=[rng.standard_normal((kd,), dtype=np.float32) for _ in range(n_layers)],
                 vn=[rng.standard_normal((kd,), dtype=np.float32) for _ in range(n_layers)])

        def parr(lst):
            a = (ctypes.c_void_p * len(lst))()
            for i, x in enumerate(lst):
                a[i] = x.ctypes.data
            return a
        d["p"] = {n: parr(d[n]) for n in ("k", "v", "q", "g", "o", "kn", "vn")}
        d["sliding"] = (ctypes.c_int * n_layers)(*([0] * n_layers))
        _CPU_DATA[key] = d
    d = _CPU_DATA[key]
    p = d["p"]
    # cap-1 live rows; the push of this step fills the last row
    n_live = (ctypes.c_uint32 * n_layers)(*([cap - 1] * n_layers))
    t0 = time.perf_counter()
    ok = R.sf37ref_decode_step_layers(p["k"], p["v"], n_live, cap, p["kn"], p["vn"], p["q"], p["g"],
                                      p["o"], d["sliding"], QH, n_layers, threads)
    dt = time.perf_counter() - t0
    assert ok
    return dt


def _cpu_layers(rows):
    """All LAYERS layers if the host has the memory for their fp32 caches
    (12.9 GB at config 2) with headroom, else the largest count that fits."""
    need = rows * KVH * HD * 4 * 2
    try:
        import psutil
        avail = psutil.virtual_memory().available
    except Exception:
        avail = 64 << 30
    return max(1, min(LAYERS, int(avail * 0.6 // need)))


def cpu_baseline(rows):
    """The reference CPU decode step of all 48 layers, on all host threads,
    timed directly (no extrapolation) when the host memory allows."""
    import oracle
    if not oracle.ref_available():
        return None
    threads = os.cpu_count() or 1
    n = _cpu_layers(rows)
    cpu_reference_step_time(threads, n, rows)  # warm (page-in)
    dt = min(cpu_reference_step_time(threads, n, rows) for _ in range(2))
    _CPU_DATA.clear()
    full = dt * LAYERS / n
    return {"value": 1.0 / full, "unit": "tokens/s", "cores": threads, "kind": "reference",
            "sample": (f"one whole decode step, {n} layers x {rows} rows" if n == LAYERS else
                       f"{n} of {LAYERS} layers x {rows} rows, scaled to {LAYERS} layers") +
                      " through the reference's own kv_cache_push + attention_decode + gate (fp32 cache "
                      "holding f16 values); best of 2 after one warm step",
            "kv_read_GBps": n * rows * KVH * HD * 2 * 4 / dt / 1e9}


def run_reference(args, rank, world):
    """--impl reference: the reference's own CPU implementation of the path
    (config 2), every step a whole 48-layer decode step on the host cores."""
    if rank != 0:
        return
    import oracle
    if not oracle.ref_available():
        print(json.dumps({"impl": "reference",
                          "unavailable": "oracle/_ref/libsf37ref.so was not built (needs the reference tree)"}))
        return
    threads = os.cpu_count() or 1
    rows = CTX + 1
    n = _cpu_layers(rows)
    for _ in range(args.warmup):
        cpu_reference_step_time(threads, n, rows)
    ts = [cpu_reference_step_time(threads, n, rows) for _ in range(args.steps)]
    step = sum(ts) / len(ts) * LAYERS / n
    val = 1.0 / step
    sample = (f"every step is a whole decode step: {LAYERS} layers x {rows} rows" if n == LAYERS else
              f"{n} of {LAYERS} layers per step (host memory), scaled to {LAYERS}")
    line = {"impl": "reference", "metric": METRIC, "value": val, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": step * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic N(0,1) f16-valued K/V in fp32 caches (the reference's only cache type), fp32 q",
            "config": decode_config("decode", world),
            "cpu_baseline": {"value": val, "unit": "tokens/s", "cores": threads, "kind": "reference",
                             "sample": sample + " through kv_cache_push + attention_decode + gate "
                                                "(sf37.c:2054-2101, 2235-2239), layers spread over the threads"},
            "e2e": {"value": val, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- parity
def _host_f16_bits(t):
    return t.cpu().view(__import__("torch").int16).numpy().view(np.uint16)


def decode_parity(rank, world, dev, stream, kc, vc, caps, sliding, pos, qh_l, kvh_l, pg, gen):
    """After the timed region: one more decode step (no append) at `pos`
    with fresh q / gate, twice (both halves of the peer buffer).  Checks
      * every rank's gathered outputs (peer-memory stores from the decode
        kernels) bit-equal an NCCL all-gather of the ranks' local outputs;
      * each rank's local heads of layers 0, 1 and LAYERS-1 against the CPU
        oracle (the reference's attention restated) on the cache contents,
        within the north-star tolerance (2e-3 abs or 1e-2 rel).
    Returns {"max_abs", "bad", "gather_equal", "ok", ...} reduced over ranks."""
    import torch
    import torch.distributed as dist
    import oracle
    from sf37_b200 import kv
    n_layers = len(kc)
    check_layers = sorted({0, min(1, n_layers - 1), n_layers - 1})
    worst, bad, gather_bad, steps_checked = 0.0, 0, 0, 0
    for rep in range(2):
        q = torch.randn(n_layers, qh_l, HD, device=dev, generator=gen)
        gate = torch.randn(n_layers, qh_l, device=dev, generator=gen)
        out = torch.full((n_layers, qh_l, HD), float("nan"), device=dev)
        desc = kv.decode_layers_desc([dict(k_cache=kc[l], v_cache=vc[l], cap=caps[l], sliding=sliding[l],
                                           window=512, pos=pos, q=q[l], gate=gate[l], out=out[l])
                                      for l in range(n_layers)])
        if pg is not None:
            # the kernels write this rank's heads into its own slot of the
            # peer buffer and store the same values into every other rank's
            pg.step(desc, kv.F16, stream)
            peer = pg.gathered[pg.epoch & 1].clone()
            out = peer[rank].contiguous()
        else:
            kv.decode(desc, qh_l, kvh_l, HD, kv.F16, stream)
        if world > 1:
            ref = torch.empty(world, n_layers, qh_l, HD, device=dev)
            dist.all_gather_into_tensor(ref, out)
            if pg is not None and not torch.equal(peer, ref):
                gather_bad += 1
        torch.cuda.synchronize(dev)
        got = out.cpu().numpy()
        for l in check_layers:
            want = oracle.attention_decode_at(q[l].cpu().numpy(), _host_f16_bits(kc[l]), _host_f16_bits(vc[l]),
                                              gate[l].cpu().numpy(), pos, caps[l], qh_l, kvh_l, HD,
                                              int(sliding[l]), 512)
            diff = np.abs(got[l] - want)
            worst = max(worst, float(diff.max()))
            bad += int(((diff > ATOL) & (diff > RTOL * np.abs(want))).sum() + (~np.isfinite(got[l])).sum())
        steps_checked += 1
    if pg is not None and kv.device_error(1):
        gather_bad += 1000
    t = torch.tensor([worst, float(bad), float(gather_bad)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    worst, bad, gather_bad = float(t[0]), int(t[1]), int(t[2])
    return {"max_abs": worst, "bad_elements": bad,
            "gather_equal": (gather_bad == 0) if world > 1 else None,
            "checked": f"{steps_checked} steps at position {pos}; layers {check_layers} of every rank's heads vs "
                       f"the CPU oracle (atol {ATOL} or rtol {RTOL})" +
                       ("; gathered [world][layers][heads][d] bit-equal to an NCCL all-gather of the local "
                        "outputs" if world > 1 and pg is not None else ""),
            "ok": bad == 0 and gather_bad == 0}


# ---------------------------------------------------------------- decode legs
def decode_leg(args, rank, world, wl, headline):
    """Config 2 (decode), 3 (hybrid) or 5a (long).  Returns the line (on
    every rank; rank 0 prints)."""
    import torch
    import torch.distributed as dist
    from sf37_b200 import kv

    dev = _dev()
    assert KVH % world == 0, "world size must divide the 8 KV heads"
    kvh_l = KVH // world
    qh_l = QH // world
    kd = kvh_l * HD
    steps, warm = args.steps, args.warmup
    oproj_on = headline and args.oproj
    prep_on = headline and args.prep
    gather = args.gather
    ctx = {"decode": CTX, "long": 131072, "hybrid": 65536}[wl]
    full_cap = ctx + warm + steps + 16
    # hybrid (config 3): layers il % 4 != 0 are sliding-window layers with a
    # 512-row ring (cache indexed modulo 512); the others are full layers.
    sliding = [wl == "hybrid" and (l % 4) != 0 for l in range(LAYERS)]
    caps = [512 if sliding[l] else full_cap for l in range(LAYERS)]
    g = torch.Generator(device=dev)
    g.manual_seed(1234 + rank)
    stream = torch.cuda.current_stream(dev)

    # Caches: KV rows of positions < ctx filled with N(0,1) (f16 RNE); every
    # step appends one row at the next position.
    kc, vc = [], []
    for l in range(LAYERS):
        k = torch.empty(caps[l], kd, dtype=torch.float16, device=dev)
        v = torch.empty(caps[l], kd, dtype=torch.float16, device=dev)
        k.normal_(generator=g)
        v.normal_(generator=g)
        kc.append(k)
        vc.append(v)
    q = torch.randn(LAYERS, qh_l, HD, device=dev, generator=g)
    gate = torch.randn(LAYERS, qh_l, device=dev, generator=g)
    kn = torch.randn(LAYERS, kd, device=dev, generator=g)
    vn = torch.randn(LAYERS, kd, device=dev, generator=g)
    out = torch.empty(LAYERS, qh_l, HD, device=dev)
    gathered = torch.empty(world, LAYERS, qh_l, HD, device=dev)

    def descs(pos, with_append=True):
        return kv.decode_layers_desc([
            dict(k_cache=kc[l], v_cache=vc[l], cap=caps[l], sliding=sliding[l], window=512, pos=pos,
                 q=q[l], gate=gate[l], out=out[l],
                 k_new=kn[l] if with_append else None, v_new=vn[l] if with_append else None)
            for l in range(LAYERS)])

    all_desc = [descs(ctx + i) for i in range(warm + steps)]

    # Multi-GPU output gather: by default the decode kernels store every
    # output head straight into all ranks' buffers over NVLink (PeerGather);
    # --gather nccl runs the decode and then an NCCL all-gather instead.
    pg = None
    if world > 1 and gather == "peer" and not oproj_on:
        from sf37_b200.shard import PeerGather, ShardPlan
        pg = PeerGather(ShardPlan(world, rank, KVH, QH, HD), LAYERS)

    # --prep: q / new K heads arrive before head norm + RoPE, which run inside
    # the decode kernel (full layers rotary 64 / theta 5e6 / llama3, sliding
    # layers 128 / 1e4, sf37.c:1983-1993).
    prep_arr = None
    if prep_on:
        qw = torch.randn(LAYERS, HD, device=dev, generator=g).mul_(0.3).to(torch.bfloat16)
        kw = torch.randn(LAYERS, HD, device=dev, generator=g).mul_(0.3).to(torch.bfloat16)
        prep_arr = kv.qk_prep_desc([
            dict(q_norm=qw[l], k_norm=kw[l], rotary_dim=64 if l % 4 == 0 else 128,
                 theta=5e6 if l % 4 == 0 else 1e4, llama3=int(l % 4 == 0), eps=1e-5) for l in range(LAYERS)])

    # --oproj: the step continues with each layer's attention output
    # projection (Q8_0 weights [4096][8192], sf37.c:3367): one more launch.
    # With N GPUs the projection is row-parallel: rank r keeps the weight
    # columns of its own heads (1/N of each row), multiplies its heads, and
    # the partial outputs are summed across ranks over peer memory
    # (PeerReduce); the heads themselves are never gathered.
    op_arr = pr = op_w = op_out = None
    in_local = QH * HD // world
    if oproj_on:
        from sf37_b200 import _lib
        op_w = torch.randint(0, 256, (LAYERS, EMBD, (in_local // 32) * 34), dtype=torch.uint8, device=dev,
                             generator=g)
        op_w.view(LAYERS, EMBD, in_local // 32, 34)[..., 0:2] = torch.tensor([0x1f, 0x22], dtype=torch.uint8,
                                                                              device=dev)  # f16 scales ~0.004
        op_out = torch.empty(LAYERS, EMBD, device=dev)
        op_arr = (_lib.OprojLayer * LAYERS)(*[_lib.OprojLayer(op_w[l].data_ptr(), out[l].data_ptr(),
                                                              op_out[l].data_ptr()) for l in range(LAYERS)])
        if world > 1:
            from sf37_b200.shard import PeerReduce
            pr = PeerReduce(world, rank, LAYERS, EMBD)

    def run_oproj(arr, dst):
        if pr is not None:
            pr.step(arr, in_local, (in_local // 32) * 34, dst, stream)
        else:
            kv.oproj(arr, in_local, EMBD, stream)

    def step(i):
        if pg is not None:
            pg.step(all_desc[i], kv.F16, stream)
            return
        if prep_arr is not None:
            kv.decode_prep(all_desc[i], prep_arr, qh_l, kvh_l, HD, kv.F16, stream)
        else:
            kv.decode(all_desc[i], qh_l, kvh_l, HD, kv.F16, stream)
        if op_arr is not None:
            run_oproj(op_arr, op_out)
            return
        if world > 1:
            dist.all_gather_into_tensor(gathered, out)

    for i in range(warm):
        step(i)
    _barrier(world, dev)
    n0 = kv.launch_count()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk = ClockSampler(dev.index).__enter__()
    ev0.record(stream)
    for i in range(warm, warm + steps):
        step(i)
    ev1.record(stream)
    _barrier(world, dev)
    launches = kv.launch_count() - n0
    ms = _max_over_ranks(ev0.elapsed_time(ev1) / steps, world, dev)

    def rows_at(pos, l):
        return min(pos + 1, 512) if sliding[l] else pos + 1
    kv_bytes_step = sum(rows_at(ctx + i, l) for i in range(warm, warm + steps) for l in range(LAYERS)) \
        * KVH * HD * 2 * 2 / steps  # whole job, f16 K+V
    tok_s = 1000.0 / ms

    if args.quick:  # profiling runs: the timed steps only
        clk.__exit__()
        if rank == 0:
            print(json.dumps({"quick": True, "layers": LAYERS, "ms_per_step": ms, "value": tok_s,
                              "gpu_launches": launches}), flush=True)
        return None

    # Roofline leg: the attention kernel alone (no append), one launch per
    # call, CUDA events on the launching stream around each launch.
    att_desc = descs(ctx + warm + steps - 1, with_append=False)
    for _ in range(3):
        kv.decode(att_desc, qh_l, kvh_l, HD, kv.F16, stream)
    torch.cuda.synchronize(dev)
    # at least ~0.5 s of launches so the clock samples cover the kernel
    n_roof = max(steps, int(500.0 / max(ms, 0.05)))
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(n_roof)]
    for a, b in evs:
        a.record(stream)
        kv.decode(att_desc, qh_l, kvh_l, HD, kv.F16, stream)
        b.record(stream)
    torch.cuda.synchronize(dev)
    att_ms = _max_over_ranks(sum(a.elapsed_time(b) for a, b in evs) / len(evs), world, dev)
    att_bytes = sum(rows_at(ctx + warm + steps - 1, l) * kd * 2 * 2 + qh_l * HD * 4 * 2 + qh_l * 4
                    for l in range(LAYERS))
    peak, peak_kind = _peaks()
    achieved = att_bytes / (att_ms * 1e-3) / 1e9
    op_line = oproj_leg(dev, stream, op_arr, op_w, out, op_out, steps, peak) if (op_arr is not None and
                                                                                  world == 1) else None
    # ncu DRAM bytes of the full 8-KV-head launch; a rank's launch reads
    # kvh_l/8 of the same rows, so the capture scales by that share
    traffic = _traffic_from_profiles("decode_f16_pipe_cfg2.md") if (LAYERS == 48 and wl == "decode") else None
    if traffic is not None:
        traffic *= kvh_l / KVH

    # End-to-end leg through the C ABI with host buffers: every step copies its
    # inputs (q, gate, new K/V rows) in from pinned host memory and its
    # outputs back out.  The copies run on side streams with double-buffered
    # device inputs/outputs, so step i's copies overlap steps i-1 / i+1.
    h_q = torch.empty_like(q, device="cpu").pin_memory()
    h_gate = torch.empty_like(gate, device="cpu").pin_memory()
    h_kn = torch.empty_like(kn, device="cpu").pin_memory()
    h_vn = torch.empty_like(vn, device="cpu").pin_memory()
    h_outs = [(torch.empty(LAYERS, EMBD) if op_arr is not None else torch.empty(LAYERS, QH, HD) if world > 1
               else torch.empty_like(out, device="cpu")).pin_memory() for _ in range(2)]
    for t_ in (h_q, h_gate, h_kn, h_vn):
        t_.normal_()
    h2d = sum(t_.numel() * t_.element_size() for t_ in (h_q, h_gate, h_kn, h_vn))
    d2h = h_outs[0].numel() * h_outs[0].element_size()
    bufs = [dict(q=q, gate=gate, kn=kn, vn=vn, out=out, gathered=gathered)]
    bufs.append({k_: v_.clone() for k_, v_ in bufs[0].items()})
    op_arrs = None
    if op_arr is not None:
        from sf37_b200 import _lib
        for B in bufs:
            B["op_out"] = torch.empty(LAYERS, EMBD, device=dev)
        op_arrs = [(_lib.OprojLayer * LAYERS)(*[_lib.OprojLayer(op_w[l].data_ptr(), B["out"][l].data_ptr(),
                                                                B["op_out"][l].data_ptr()) for l in range(LAYERS)])
                   for B in bufs]

    def descs_b(pos, B):
        return kv.decode_layers_desc([
            dict(k_cache=kc[l], v_cache=vc[l], cap=caps[l], sliding=sliding[l], window=512, pos=pos,
                 q=B["q"][l], gate=B["gate"][l], out=B["out"][l], k_new=B["kn"][l], v_new=B["vn"][l])
            for l in range(LAYERS)])

    e2e_desc = [[descs_b(ctx + warm + steps + (i % 4), bufs[bb]) for bb in range(2)] for i in range(4)]
    copy_s = torch.cuda.Stream(dev)   # host -> device
    out_s = torch.cuda.Stream(dev)    # device -> host
    ev_done = [torch.cuda.Event(), torch.cuda.Event()]
    ev_out = [torch.cuda.Event(), torch.cuda.Event()]
    ev_in = [torch.cuda.Event(), torch.cuda.Event()]

    def e2e_step(i):
        bb = i & 1
        B = bufs[bb]
        copy_s.wait_event(ev_done[bb])  # step i-2 is done with these inputs
        with torch.cuda.stream(copy_s):
            B["q"].copy_(h_q, non_blocking=True)
            B["gate"].copy_(h_gate, non_blocking=True)
            B["kn"].copy_(h_kn, non_blocking=True)
            B["vn"].copy_(h_vn, non_blocking=True)
        ev_in[bb].record(copy_s)
        stream.wait_event(ev_in[bb])
        stream.wait_event(ev_out[bb])   # step i-2's outputs have been read out
        if pg is not None:
            # the peer buffer half is rewritten two steps later by the other
            # ranks, so take a device copy on the decode stream first
            pg.step(e2e_desc[i % 4][bb], kv.F16, stream)
            B["gathered"].copy_(pg.gathered[pg.epoch & 1])
        else:
            if prep_arr is not None:
                kv.decode_prep(e2e_desc[i % 4][bb], prep_arr, qh_l, kvh_l, HD, kv.F16, stream)
            else:
                kv.decode(e2e_desc[i % 4][bb], qh_l, kvh_l, HD, kv.F16, stream)
            if op_arrs is not None:
                run_oproj(op_arrs[bb], B["op_out"])
            elif world > 1:
                dist.all_gather_into_tensor(B["gathered"], B["out"])
        ev_done[bb].record(stream)
        out_s.wait_event(ev_done[bb])
        with torch.cuda.stream(out_s):
            if op_arrs is not None:
                h_outs[bb].copy_(B["op_out"], non_blocking=True)
            elif world > 1:
                h_outs[bb].view(LAYERS, world, qh_l, HD).copy_(B["gathered"].permute(1, 0, 2, 3), non_blocking=True)
            else:
                h_outs[bb].copy_(B["out"], non_blocking=True)
        ev_out[bb].record(out_s)

    for i in range(3):
        e2e_step(i)
    _barrier(world, dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(steps):
        e2e_step(i)
    stream.wait_stream(copy_s)
    stream.wait_stream(out_s)
    e1.record(stream)
    _barrier(world, dev)
    e2e_ms = _max_over_ranks(e0.elapsed_time(e1) / steps, world, dev)
    clk.__exit__()

    # Parity of the gathered (or reduced) outputs, after the timed regions.
    parity = None
    if not prep_on and not oproj_on:
        pgen = torch.Generator(device=dev)
        pgen.manual_seed(4321 + rank)
        parity = decode_parity(rank, world, dev, stream, kc, vc, caps, sliding, ctx + warm + steps + 2,
                               qh_l, kvh_l, pg, pgen)
    elif pr is not None:
        parity = oproj_reduce_parity(world, dev, stream, pr, op_arr, op_w, out, op_out, in_local)
    for peer in (pg, pr):
        if peer is not None:
            if kv.device_error(1):
                raise RuntimeError("peer gather/reduce: a bounded wait timed out")
            dist.barrier()
            torch.cuda.synchronize(dev)
            peer.close()

    line = {
        "metric": METRIC, "value": tok_s, "unit": "tokens/s", "n_gpus": world, "steps": steps,
        "warmup": warm, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f16",
        "data": "synthetic: N(0,1) f16 K/V caches and fp32 q/gate/new rows from torch's seeded CUDA "
                "generator",
        "config": decode_config(wl, world, prep_on, oproj_on, gather),
        "kv_read_GBps": kv_bytes_step / (ms * 1e-3) / 1e9,
        "kv_read_frac_of_8TBps": kv_bytes_step / (ms * 1e-3) / 8e12,
        "roofline": {"bound": "hbm", "kernel": "decode_f16_pipe_kernel", "achieved": achieved,
                     "peak": peak, "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": traffic, "launch_ms": att_ms,
                     "algorithmic_bytes_per_launch": att_bytes},
        "e2e": {"value": 1000.0 / e2e_ms, "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms},
        "gpu_launches": launches,
        "clocks": clk.summary(),
    }
    if parity is not None:
        line["parity"] = parity
    if world > 1:
        # max over ranks of each: the whole step, and the decode kernel timed
        # alone (no append, no gather); the rest is the output gather and
        # rank skew
        line["phases"] = {"step_ms": ms, "decode_kernel_ms": att_ms, "gather_and_skew_ms": ms - att_ms}
    if op_line:
        line["oproj"] = op_line
    del kc, vc, all_desc, e2e_desc, bufs
    torch.cuda.empty_cache()
    return line


def oproj_reduce_parity(world, dev, stream, pr, op_arr, op_w, out, op_out, in_local):
    """Row-parallel o_proj: the peer-memory reduce of the ranks' partial
    products equals an NCCL all-reduce of the same partials (computed by the
    plain sf37kv_oproj_q8_0 on this rank's column slice), up to the float
    summation order."""
    import torch
    import torch.distributed as dist
    from sf37_b200 import _lib, kv
    out.normal_()
    pr.step(op_arr, in_local, (in_local // 32) * 34, op_out, stream)
    got = op_out.clone()
    part = torch.empty_like(op_out)
    arr = (_lib.OprojLayer * LAYERS)(*[_lib.OprojLayer(op_w[l].data_ptr(), out[l].data_ptr(), part[l].data_ptr())
                                       for l in range(LAYERS)])
    kv.oproj(arr, in_local, EMBD, stream)
    dist.all_reduce(part)
    scale = float(part.abs().max())
    err = float((got - part).abs().max())
    t = torch.tensor([err / max(scale, 1e-30)], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    rel = float(t.item())
    return {"max_rel_to_max": rel, "checked": "peer-memory reduce vs NCCL all-reduce of the ranks' partials",
            "ok": rel <= 1e-5}


def oproj_leg(dev, stream, op_arr, op_w, x, op_out, steps, peak):
    """The o_proj kernel alone over all layers (one launch), timed with CUDA
    events per launch; and the reference's own quantize + matvec kernels
    (sf37_cuda_matvec_q8_0 of oracle/_ref/libsf37ref_cuda.so), one call per
    layer, on the same weights and inputs."""
    import torch
    from sf37_b200 import kv
    n_layers = op_w.shape[0]
    wbytes = op_w.numel()
    for _ in range(3):
        kv.oproj(op_arr, QH * HD, EMBD, stream)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(max(steps, 20))]
    for a, b_ in evs:
        a.record(stream)
        kv.oproj(op_arr, QH * HD, EMBD, stream)
        b_.record(stream)
    torch.cuda.synchronize(dev)
    ms = sum(a.elapsed_time(b_) for a, b_ in evs) / len(evs)
    alg = wbytes + n_layers * (QH * HD * 4 + EMBD * 4)
    res = {"kernel": "oproj_q8_0_kernel", "layers": n_layers, "in_dim": QH * HD, "out_dim": EMBD,
           "launch_ms": ms, "algorithmic_bytes_per_launch": alg,
           "roofline": {"bound": "hbm", "achieved": alg / (ms * 1e-3) / 1e9, "peak": peak, "unit": "GB/s",
                        "frac": alg / (ms * 1e-3) / 1e9 / peak}}
    try:
        import oracle
        if not oracle.ref_cuda_available():
            raise RuntimeError("oracle/_ref/libsf37ref_cuda.so not built")
        R = oracle.ref_cuda()
        TP = ctypes.POINTER(oracle.RefTensor)
        R.sf37_cuda_matvec_q8_0.restype = ctypes.c_int
        R.sf37_cuda_matvec_q8_0.argtypes = [TP, TP, ctypes.c_uint64, ctypes.c_uint64, TP]
        refout = torch.empty(EMBD, device=dev)

        def rt(t):
            return oracle.ref_tensor(t.data_ptr(), t.numel() * t.element_size())
        ts = [(rt(refout), rt(op_w[l]), rt(x[l])) for l in range(n_layers)]
        for o, w, xx in ts[:3]:
            R.sf37_cuda_matvec_q8_0(o, w, QH * HD, EMBD, xx)
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        reps = 5
        for _ in range(reps):
            for o, w, xx in ts:
                if not R.sf37_cuda_matvec_q8_0(o, w, QH * HD, EMBD, xx):
                    raise RuntimeError("reference matvec failed")
        e1.record()
        torch.cuda.synchronize(dev)
        rms = e0.elapsed_time(e1) / reps
        res["reference_kernels"] = {"ms_all_layers": rms, "GBps": alg / (rms * 1e-3) / 1e9,
                                    "calls": f"{n_layers} x sf37_cuda_matvec_q8_0 (quantize + matvec kernels)"}
    except Exception as e:
        res["reference_kernels"] = {"unavailable": str(e)}
    return res


def reference_gpu_leg(dev, steps):
    """Config 2 with fp32 caches, one call per layer through the reference's
    own entry point sf37_cuda_attention_decode_heads_at: (a) the reference's
    CUDA kernels (oracle/_ref/libsf37ref_cuda.so, sm_100a build of its
    sources), (b) this library's drop-in of the same symbol.  Tokens/s of the
    48 per-layer calls per step (attention only, fp32 KV = 12.9 GB)."""
    import torch
    import oracle
    from sf37_b200 import kv
    if not oracle.ref_cuda_available():
        return None
    R = oracle.ref_cuda()
    cap = CTX + 1
    layers = []
    for _ in range(LAYERS):
        k = torch.empty(cap, KVH * HD, device=dev).normal_()
        v = torch.empty(cap, KVH * HD, device=dev).normal_()
        layers.append((k, v))
    q = torch.randn(QH, HD, device=dev)
    gate = torch.randn(QH, device=dev)
    out = torch.empty(QH, HD, device=dev)

    def rt(t):
        return oracle.ref_tensor(t.data_ptr(), t.numel() * t.element_size())

    def run(which, n):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for rep in range(2):
            torch.cuda.synchronize(dev)
            e0.record()
            for _ in range(n):
                for k, v in layers:
                    if which == "ref":
                        R.sf37_cuda_attention_decode_heads_at(rt(out), rt(q), rt(k), rt(v), rt(gate), CTX, cap,
                                                              QH, KVH, HD, 0, 512)
                    else:
                        kv.attention_decode_heads_at(out, q, k, v, gate, CTX, cap, QH, KVH, HD, 0, 512)
            e1.record()
            torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / n

    n = max(2, min(steps, 5))
    ms_ref = run("ref", n)
    ms_ours = run("ours", n)
    b = LAYERS * cap * KVH * HD * 4 * 2
    peak, _ = _peaks()
    del layers
    torch.cuda.empty_cache()
    return {"what": "cfg2 attention, fp32 caches, 48 per-layer calls of sf37_cuda_attention_decode_heads_at "
                    "issued from the host (no graph), as sf37.c issues them",
            "reference_kernels": {"tokens_per_s": 1000.0 / ms_ref, "kv_read_GBps": b / (ms_ref * 1e-3) / 1e9,
                                  "frac": b / (ms_ref * 1e-3) / 1e9 / peak},
            "dropin_f32": {"tokens_per_s": 1000.0 / ms_ours, "kv_read_GBps": b / (ms_ours * 1e-3) / 1e9,
                           "frac": b / (ms_ours * 1e-3) / 1e9 / peak}}


def per_layer_leg(args, dev):
    """The engine's call pattern: in sf37.c each layer's q depends on the
    previous layer's output, so a decode step is 48 SEQUENTIAL single-layer
    attention calls (sf37.c:3285-3437), not one batched launch.  Config 2
    caches (32768 + 1 rows), one step = 48 calls, each appending its row
    and attending over 32769 rows.  Timed as CUDA-graph replays of the 48
    calls (the reference engine captures its decode in a CUDA graph) for f16
    caches (sf37kv_decode) and fp32 caches (the drop-in's kernel)."""
    import torch
    from sf37_b200 import kv
    cap = CTX + 1
    pos = CTX
    peak, kind = _peaks()
    res = {"what": "48 sequential single-layer decode calls per step (append + attention over 32769 rows), "
                   "replayed from a CUDA graph"}
    s = torch.cuda.Stream(dev)
    for name, dt, tdt in (("f16", kv.F16, torch.float16), ("f32", kv.F32, torch.float32)):
        g = torch.Generator(device=dev)
        g.manual_seed(55)
        ks = [torch.randn(cap, KVH * HD, device=dev, generator=g).to(tdt) for _ in range(LAYERS)]
        vs = [torch.randn(cap, KVH * HD, device=dev, generator=g).to(tdt) for _ in range(LAYERS)]
        q = torch.randn(LAYERS, QH, HD, device=dev, generator=g)
        gate = torch.randn(LAYERS, QH, device=dev, generator=g)
        kn = torch.randn(LAYERS, KVH * HD, device=dev, generator=g)
        vn = torch.randn(LAYERS, KVH * HD, device=dev, generator=g)
        out = torch.empty(LAYERS, QH, HD, device=dev)
        descs = [kv.decode_layers_desc([dict(k_cache=ks[l], v_cache=vs[l], cap=cap, pos=pos, q=q[l], gate=gate[l],
                                             out=out[l], k_new=kn[l], v_new=vn[l])]) for l in range(LAYERS)]
        with torch.cuda.stream(s):
            for _ in range(3):
                for d in descs:
                    kv.decode(d, QH, KVH, HD, dt, s)
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            for d in descs:
                kv.decode(d, QH, KVH, HD, dt, s)
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize(dev)
        n = max(args.steps, 20)
        clk = ClockSampler(dev.index).__enter__()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        with torch.cuda.stream(s):
            for _ in range(n):
                graph.replay()
        e1.record(s)
        torch.cuda.synchronize(dev)
        clk.__exit__()
        ms = e0.elapsed_time(e1) / n
        alg = LAYERS * (cap * KVH * HD * 2 * (2 if dt == kv.F16 else 4) + QH * HD * 8 + QH * 4)
        ach = alg / (ms * 1e-3) / 1e9
        res[name] = {"tokens_per_s": 1000.0 / ms, "ms_per_step": ms, "us_per_layer_call": ms * 1e3 / LAYERS,
                     "roofline": {"bound": "hbm", "achieved": ach, "peak": peak, "peak_kind": kind, "unit": "GB/s",
                                  "frac": ach / peak, "algorithmic_bytes_per_step": alg},
                     "clocks": clk.summary()}
        del ks, vs, graph, descs
        torch.cuda.empty_cache()
    return res


def cfg1_leg(args, dev):
    """one layer, 2048 cached f16 rows + the appended row
    at position 2048, 64 Q / 8 KV heads, d 128.  One step = one
    sf37kv_decode (append + attention, one launch).  The 8.4 MB of K/V would
    sit in the 126 MB L2, so steps rotate over 16 independent cache copies
    (134 MB); the rotation is captured once in a CUDA graph."""
    import torch
    from sf37_b200 import kv
    cap, ncopy = 2049, 16
    g = torch.Generator(device=dev)
    g.manual_seed(3)
    copies = []
    for _ in range(ncopy):
        k = torch.randn(cap, KVH * HD, device=dev, generator=g).half()
        v = torch.randn(cap, KVH * HD, device=dev, generator=g).half()
        q = torch.randn(QH, HD, device=dev, generator=g)
        gate = torch.randn(QH, device=dev, generator=g)
        kn = torch.randn(KVH * HD, device=dev, generator=g)
        vn = torch.randn(KVH * HD, device=dev, generator=g)
        out = torch.empty(QH, HD, device=dev)
        copies.append((kv.decode_layers_desc([dict(k_cache=k, v_cache=v, cap=cap, pos=2048, q=q, gate=gate,
                                                   out=out, k_new=kn, v_new=vn)]), k, v, q, gate, kn, vn, out))
    gs = torch.cuda.Stream(dev)
    with torch.cuda.stream(gs):
        for i in range(args.warmup * ncopy):
            kv.decode(copies[i % ncopy][0], QH, KVH, HD, kv.F16, gs)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=gs):
        for i in range(ncopy):
            kv.decode(copies[i][0], QH, KVH, HD, kv.F16, gs)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize(dev)
    reps = max(args.steps, 50)
    clk = ClockSampler(dev.index).__enter__()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(gs)
    with torch.cuda.stream(gs):
        for _ in range(reps):
            graph.replay()
    e1.record(gs)
    torch.cuda.synchronize(dev)
    clk.__exit__()
    us = e0.elapsed_time(e1) * 1e3 / (reps * ncopy)
    cpu = None
    import oracle
    if oracle.ref_available() and not args.no_cpu:
        from sf37_b200 import synth
        k, v, k_new, v_new, q, gate = synth.cfg1_inputs(0)
        kc = np.zeros((cap, 1024), np.float32)
        vc = np.zeros((cap, 1024), np.float32)
        ts = []
        for _ in range(5):
            kc[:2048] = k
            vc[:2048] = v
            t0 = time.perf_counter()
            n = oracle.ref_kv_cache_push(kc, vc, cap, 2048, k_new[None], v_new[None])
            oracle.ref_attention_decode(q, kc, vc, n, cap, QH, 0, gate)
            ts.append(time.perf_counter() - t0)
        cpu = {"us_per_step": min(ts) * 1e6, "cores": 1, "kind": "reference",
               "sample": "one config-1 step (kv_cache_push + attention_decode + gate), best of 5"}
    alg = cap * KVH * HD * 2 * 2 + QH * HD * 8 + QH * 4 + KVH * HD * 8
    peak, kind = _peaks()
    ach = alg / (us * 1e-6) / 1e9
    del copies, graph
    torch.cuda.empty_cache()
    return {"workload": "cfg1: 1 layer, 2048 cached rows + 1 appended, one sf37kv_decode per step",
            "us_per_step": us, "steps_per_s": 1e6 / us, "launches_per_step": 1,
            "l2": "16 rotating cache copies (134 MB > 126 MB L2), CUDA-graph replay",
            "roofline": {"bound": "hbm", "kernel": "decode_f16_pipe_kernel", "achieved": ach, "peak": peak,
                         "peak_kind": kind, "unit": "GB/s", "frac": ach / peak, "algorithmic_bytes_per_step": alg},
            "cpu_baseline": cpu, "clocks": clk.summary()}


def prefill_leg(args, rank, world, dev, steps):
    """per layer, append an 8192-token chunk onto a
    24576-token f16 prefix and run causal chunk attention (bf16 queries,
    64 Q / 8 KV heads, d 128); one step = all layers.  Tensor-core bound."""
    import torch
    from sf37_b200 import kv
    kvh_l, qh_l = KVH // world, QH // world
    kd = kvh_l * HD
    prefix, chunk, cap = 24576, 8192, 32768
    g = torch.Generator(device=dev)
    g.manual_seed(99 + rank)
    kc = [torch.randn(cap, kd, device=dev, generator=g).half() for _ in range(LAYERS)]
    vc = [torch.randn(cap, kd, device=dev, generator=g).half() for _ in range(LAYERS)]
    kn = torch.randn(chunk, kd, device=dev, generator=g)
    vn = torch.randn(chunk, kd, device=dev, generator=g)
    q = torch.randn(chunk, qh_l, HD, device=dev, generator=g).to(torch.bfloat16)
    gate = torch.randn(chunk, qh_l, device=dev, generator=g)
    out = torch.empty(chunk, qh_l, HD, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        for l in range(LAYERS):
            kv.append([dict(k_cache=kc[l], v_cache=vc[l], cap=cap, pos0=prefix, n_tok=chunk, k=kn, v=vn)],
                      kd, kv.F16, stream)
            kv.prefill(kc[l], vc[l], cap, q, gate, out, prefix, chunk, qh_l, kvh_l, HD, kv.F16,
                       stream=stream)

    for _ in range(args.warmup):
        step()
    _barrier(world, dev)
    n0 = kv.launch_count()
    clk = ClockSampler(dev.index).__enter__()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    _barrier(world, dev)
    ms = _max_over_ranks(e0.elapsed_time(e1) / steps, world, dev)
    launches = kv.launch_count() - n0
    # attention kernel alone, CUDA events per launch
    evs = []
    for _ in range(16):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        kv.prefill(kc[0], vc[0], cap, q, gate, out, prefix, chunk, qh_l, kvh_l, HD, kv.F16, stream=stream)
        b.record(stream)
        evs.append((a, b))
    torch.cuda.synchronize(dev)
    clk.__exit__()
    att_ms = _max_over_ranks(sum(a.elapsed_time(b) for a, b in evs) / len(evs), world, dev)
    pairs = chunk * prefix + chunk * (chunk + 1) // 2
    flops_layer = 4.0 * HD * pairs * qh_l
    peak, kind = _tensor_peak()
    ach = flops_layer / (att_ms * 1e-3) / 1e12
    del kc, vc
    torch.cuda.empty_cache()
    return {"workload": "cfg4: 8192-token chunk on a 24576-token prefix, 48 layers (append + causal chunk "
                        "attention per layer), f16 K/V, bf16 q, f32 accumulate",
            "tokens_per_s": chunk / (ms * 1e-3), "ms_per_step": ms, "steps": steps, "gpu_launches": launches,
            "roofline": {"bound": "tensor", "kernel": "prefill_tc05_kernel", "achieved": ach, "peak": peak,
                         "peak_kind": kind, "unit": "TFLOP/s", "frac": ach / peak, "launch_ms": att_ms,
                         "algorithmic_flops_per_launch": flops_layer},
            "clocks": clk.summary()}


def prefill_f32_leg(dev):
    """The call the reference engine makes for chunked prefill
    (sf37.c:5919): sf37_cuda_attention_prefill_heads with fp32 caches and
    fp32 q, one layer, a 2048-token chunk on a 24576-token prefix (64 Q /
    8 KV heads, d 128).  Timed through this library's drop-in of the symbol
    (tensor-core tiles, bf16 hi/lo operand split) and through the
    reference's own CUDA kernel (oracle/_ref/libsf37ref_cuda.so, a warp per
    (token, head), sf37_cuda.cu:3163-3317) on the same inputs; the two
    outputs are compared at the north-star tolerance."""
    import torch
    import oracle
    from sf37_b200 import kv
    prefix, chunk = 24576, 2048
    cap = prefix + chunk
    g = torch.Generator(device=dev)
    g.manual_seed(21)
    k = torch.randn(cap, KVH * HD, device=dev, generator=g)
    v = torch.randn(cap, KVH * HD, device=dev, generator=g)
    q = torch.randn(chunk, QH, HD, device=dev, generator=g)
    gate = torch.randn(chunk, QH, device=dev, generator=g)
    out = torch.empty(chunk, QH, HD, device=dev)
    pairs = chunk * prefix + chunk * (chunk + 1) // 2
    flops = 4.0 * HD * pairs * QH
    peak, kind = _tensor_peak()

    def ours():
        if not kv.attention_prefill_heads(out, q, k, v, gate, prefix, chunk, cap, QH, KVH, HD, 0, 512):
            raise RuntimeError("drop-in prefill failed")

    for _ in range(3):
        ours()
    torch.cuda.synchronize(dev)
    clk = ClockSampler(dev.index).__enter__()
    reps = 10
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        ours()
    e1.record()
    torch.cuda.synchronize(dev)
    clk.__exit__()
    ms = e0.elapsed_time(e1) / reps
    ach = flops / (ms * 1e-3) / 1e12
    res = {"what": "sf37_cuda_attention_prefill_heads, fp32 caches + fp32 q, one layer: 2048-token chunk on a "
                   "24576-token prefix (the engine's prefill call, sf37.c:5919)",
           "dropin_ms": ms, "dropin_tokens_per_s": chunk / (ms * 1e-3),
           "roofline": {"bound": "tensor", "kernel": "prefill_tc32 (mma.sync bf16, 3-term hi/lo split)",
                        "achieved": ach, "peak": peak, "peak_kind": kind, "unit": "TFLOP/s", "frac": ach / peak,
                        "algorithmic_flops_per_launch": flops,
                        "note": "algorithmic flops count one fp32 product; the kernel issues three bf16 products"},
           "clocks": clk.summary()}
    try:
        if not oracle.ref_cuda_available():
            raise RuntimeError("oracle/_ref/libsf37ref_cuda.so not built")
        R = oracle.ref_cuda()

        def rt(t):
            return oracle.ref_tensor(t.data_ptr(), t.numel() * t.element_size())
        theirs = torch.empty_like(out)
        args = (rt(theirs), rt(q), rt(k), rt(v), rt(gate), prefix, chunk, cap, QH, KVH, HD, 0, 512)
        if not R.sf37_cuda_attention_prefill_heads(*args):
            raise RuntimeError("reference prefill failed")
        torch.cuda.synchronize(dev)
        e0.record()
        rreps = 2
        for _ in range(rreps):
            R.sf37_cuda_attention_prefill_heads(*args)
        e1.record()
        torch.cuda.synchronize(dev)
        rms = e0.elapsed_time(e1) / rreps
        ours()
        torch.cuda.synchronize(dev)
        d = (out - theirs).abs()
        ok = bool(((d <= ATOL) | (d <= RTOL * theirs.abs())).all())
        res["reference_kernel"] = {"ms": rms, "tokens_per_s": chunk / (rms * 1e-3),
                                   "TFLOPs": flops / (rms * 1e-3) / 1e12}
        res["speedup_vs_reference_kernel"] = rms / ms
        res["parity_vs_reference_kernel"] = {"max_abs": float(d.max()), "ok": ok,
                                             "tolerance": f"abs {ATOL} or rel {RTOL}"}
    except Exception as e:
        res["reference_kernel"] = {"unavailable": str(e)}
    del k, v, q, out
    torch.cuda.empty_cache()
    return res


def snapshot_leg(args, rank, world, dev):
    """BASELINE config 5b: pack the 32768-token prefix of 48 f16 layers into
    pinned host memory in both reference formats (raw f32 rows, int8-grouped
    payload rows), then restore it.  Reports the device-side pack kernel
    bandwidth (to a device buffer, HBM-bound) and the end-to-end host rates
    (sf37kv_pack_to_host / sf37kv_unpack_from_host, link-bound)."""
    import torch
    from sf37_b200 import _lib, kv
    kd = (KVH // world) * HD
    rows = 32768
    g = torch.Generator(device=dev)
    g.manual_seed(7 + rank)
    layers = []
    for _ in range(LAYERS):
        k = torch.empty(rows, kd, dtype=torch.float16, device=dev).normal_(generator=g)
        v = torch.empty(rows, kd, dtype=torch.float16, device=dev).normal_(generator=g)
        layers.append(dict(k_cache=k, v_cache=v, cap=rows, first_pos=0, rows=rows))
    res = {}
    stream = torch.cuda.current_stream(dev)
    peak, kind = _peaks()
    clk = ClockSampler(dev.index).__enter__()
    for fmt, name in ((kv.FMT_RAW, "raw_f32"), (kv.FMT_I8G, "i8_grouped")):
        arr, total = kv.pack_layers_desc(layers, kd, fmt)
        dbuf = torch.empty(total, dtype=torch.uint8, device=dev)
        for _ in range(args.warmup):
            kv.pack(dbuf, arr, kd, kv.F16, fmt, stream=stream)
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n = max(args.steps, 5)
        e0.record(stream)
        for _ in range(n):
            kv.pack(dbuf, arr, kd, kv.F16, fmt, stream=stream)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1) / n
        kv_read = LAYERS * rows * kd * 2 * 2
        del dbuf
        host = _lib.lib().sf37kv_host_alloc(total)
        assert host, _lib.last_error()
        kv.pack_to_host(host, arr, kd, kv.F16, fmt)  # warm (page-in)
        t0 = time.perf_counter()
        kv.pack_to_host(host, arr, kd, kv.F16, fmt)
        t_pack = time.perf_counter() - t0
        t0 = time.perf_counter()
        kv.unpack_from_host(host, arr, kd, kv.F16, fmt)
        t_unpack = time.perf_counter() - t0
        _lib.lib().sf37kv_host_free(host)
        dev_gbps = (kv_read + total) / (ms * 1e-3) / 1e9
        res[name] = {"bytes": total, "device_pack_ms": ms, "device_pack_GBps": dev_gbps,
                     "device_pack_frac": dev_gbps / peak,
                     "host_pack_s": t_pack, "host_pack_GBps": total / t_pack / 1e9,
                     "host_restore_s": t_unpack, "host_restore_GBps": total / t_unpack / 1e9}
    clk.__exit__()
    sess = session_leg(dev, layers, kd, rows) if (world == 1 and not args.no_session) else None
    del layers
    torch.cuda.empty_cache()
    r = res["raw_f32"]
    return {"workload": "cfg5b: pack/restore the 32768-token prefix x 48 f16 layers (raw f32 snapshot rows and "
                        "int8-grouped payload rows) to/from pinned host memory",
            "formats": res,
            "roofline": {"bound": "hbm", "kernel": "pack_kernel (raw, to a device buffer)",
                         "achieved": r["device_pack_GBps"], "peak": peak, "peak_kind": kind, "unit": "GB/s",
                         "frac": r["device_pack_GBps"] / peak},
            "session": sess, "clocks": clk.summary()}


def session_leg(dev, layers, kd, rows):
    """Whole session checkpoints through sf37kv_session_* (48 f16 layers of
    `rows` live rows): the payload written to a file and read back, and the
    raw snapshot written to pinned memory; beside it, the reference's own
    CUDA-backend per-row loops (two synchronous 4 KiB tensor reads per row,
    its own encoder and fwrite) timed on one fp32 layer and scaled to 48."""
    import shutil
    import tempfile
    import torch
    from sf37_b200.session import Session, default_layout
    L = default_layout()
    L.n_layers = len(layers)
    s = Session(rows, [(d["k_cache"], d["v_cache"]) for d in layers], layout=L)
    s.set_tokens(np.arange(rows) % L.vocab)
    out = {}
    d = "/dev/shm" if shutil.disk_usage("/dev/shm").free > 2 * s.payload_bytes() else tempfile.gettempdir()
    with tempfile.NamedTemporaryFile(dir=d) as f:
        t0 = time.perf_counter()
        nb = s.save_payload(f)
        os.fsync(f.fileno())
        out["payload_save_s"] = time.perf_counter() - t0
        f.seek(0)
        t0 = time.perf_counter()
        s.load_payload(f.fileno(), nb)
        out["payload_load_s"] = time.perf_counter() - t0
    out.update(payload_bytes=nb, file_dir=d, payload_save_GBps=nb / out["payload_save_s"] / 1e9,
               payload_load_GBps=nb / out["payload_load_s"] / 1e9)
    buf = torch.empty(s.snapshot_bytes(), dtype=torch.uint8, pin_memory=True)
    s.save_snapshot(buf)  # page-in
    t0 = time.perf_counter()
    s.save_snapshot(buf)
    out["snapshot_save_s"] = time.perf_counter() - t0
    t0 = time.perf_counter()
    s.load_snapshot(buf)
    out["snapshot_load_s"] = time.perf_counter() - t0
    out["snapshot_bytes"] = buf.numel()
    del buf
    try:
        import oracle
        if not (oracle.ref_available() and oracle.ref_cuda_available()):
            raise RuntimeError("oracle/_ref not built")
        R = oracle.ref()
        RC = oracle.ref_cuda()
        rd = ctypes.cast(RC.sf37_cuda_tensor_read, ctypes.c_void_p)
        R.sf37ref_payload_rows_cuda.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_uint32] * 3 + [ctypes.c_int]
        R.sf37ref_snapshot_rows_cuda.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_uint32] * 3 + [ctypes.c_void_p]
        k = layers[0]["k_cache"].float()
        v = layers[0]["v_cache"].float()
        kt = oracle.RefTensor(k.data_ptr(), k.numel() * 4)
        vt = oracle.RefTensor(v.data_ptr(), v.numel() * 4)
        torch.cuda.synchronize(dev)
        with open(os.devnull, "wb") as f:
            t0 = time.perf_counter()
            rc = R.sf37ref_payload_rows_cuda(rd, ctypes.addressof(kt), ctypes.addressof(vt), 0, rows, rows,
                                             f.fileno())
            t_pay = time.perf_counter() - t0
        host = np.empty(2 * rows * kd * 4, np.uint8)
        t0 = time.perf_counter()
        rc |= R.sf37ref_snapshot_rows_cuda(rd, ctypes.addressof(kt), ctypes.addressof(vt), 0, rows, rows,
                                           host.ctypes.data)
        t_snap = time.perf_counter() - t0
        if rc:
            raise RuntimeError("reference row loop failed")
        n = len(layers)
        out["reference_per_row"] = {
            "payload_save_s": t_pay * n, "snapshot_save_s": t_snap * n,
            "sample": f"1 of {n} layers ({rows} rows, fp32 cache: the reference's only type), x{n}",
            "payload_speedup": t_pay * n / out["payload_save_s"],
            "snapshot_speedup": t_snap * n / out["snapshot_save_s"]}
    except Exception as e:  # the reference library is test infrastructure
        out["reference_per_row"] = {"unavailable": str(e)}
    return out


# ---------------------------------------------------------------- drivers
def _compact_decode(line):
    keep = ("value", "unit", "ms_per_step", "kv_read_GBps", "roofline", "e2e", "parity", "phases", "gpu_launches",
            "clocks")
    d = {"workload": line["config"]["workload"], "ctx": line["config"]["ctx"]}
    d.update({k: line[k] for k in keep if k in line})
    return d


def run_default(args, rank, world):
    """The headline line (config 2) plus, after its timed region, the other
    configs and the per-layer pattern as compact sub-objects."""
    import torch
    dev = _dev()
    line = decode_leg(args, rank, world, "decode", headline=True)
    if line is None:
        return
    ok = line.get("parity", {}).get("ok", True)
    if not args.headline_only:
        configs = {}
        sub_steps = max(3, min(args.steps, 10))
        for wl, key in (("hybrid", "cfg3"), ("long", "cfg5a")):
            sub = decode_leg(args, rank, world, wl, headline=False)
            ok = ok and sub.get("parity", {}).get("ok", True)
            configs[key] = _compact_decode(sub)
        configs["cfg4"] = prefill_leg(args, rank, world, dev, max(2, min(args.steps, 3)))
        configs["cfg5b"] = snapshot_leg(args, rank, world, dev)
        if world == 1:
            configs["cfg1"] = cfg1_leg(args, dev)
            line["per_layer"] = per_layer_leg(args, dev)
            line["prefill_dropin"] = prefill_f32_leg(dev)
            ok = ok and line["prefill_dropin"].get("parity_vs_reference_kernel", {}).get("ok", True)
            if not args.no_ref_gpu:
                line["reference_gpu"] = reference_gpu_leg(dev, sub_steps)
        line["configs"] = configs
    if world == 1 and not args.no_cpu and rank == 0:
        line["cpu_baseline"] = cpu_baseline(CTX + 1)
    _barrier(world, dev)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if not ok:
        sys.stderr.write("bench: parity check FAILED (see the line's parity objects)\n")
        sys.exit(3)


def run_single(args, rank, world):
    """--workload X: one line for that config alone."""
    dev = _dev()
    wl = args.workload
    if wl in ("decode", "hybrid", "long"):
        line = decode_leg(args, rank, world, wl, headline=True)
        if line is None:
            return
    elif wl == "prefill":
        line = prefill_leg(args, rank, world, dev, args.steps)
    elif wl == "snapshot":
        line = snapshot_leg(args, rank, world, dev)
    elif wl == "cfg1":
        line = cfg1_leg(args, dev)
    elif wl == "per_layer":
        line = per_layer_leg(args, dev)
    elif wl == "prefill_dropin":
        line = prefill_f32_leg(dev)
    _barrier(world, dev)
    if rank == 0:
        line.setdefault("workload", wl)
        line.setdefault("n_gpus", world)
        print(json.dumps(line), flush=True)
    if not line.get("parity", {}).get("ok", True):
        sys.exit(3)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--gather", default="peer", choices=["peer", "nccl"],
                    help="multi-GPU output gather: decode-kernel stores into peer memory, or NCCL")
    ap.add_argument("--oproj", action="store_true",
                    help="decode workloads: add each layer's Q8_0 o_proj matvec to the step")
    ap.add_argument("--prep", action="store_true",
                    help="decode workloads: fuse the q/k head norm + RoPE into the step (sf37kv_decode_prep)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    ap.add_argument("--no-ref-gpu", action="store_true", help="skip the reference CUDA kernels leg")
    ap.add_argument("--no-session", action="store_true", help="skip the whole-session checkpoint leg")
    ap.add_argument("--headline-only", action="store_true", help="default workload: skip the other configs")
    ap.add_argument("--workload", default="all",
                    choices=["all", "decode", "prefill", "hybrid", "long", "snapshot", "cfg1", "per_layer", "prefill_dropin"],
                    help="all = config 2 headline + every other config (default); decode = config 2; "
                         "hybrid = config 3; prefill = config 4; long = config 5a; snapshot = config 5b")
    ap.add_argument("--quick", action="store_true",
                    help="timed steps only (no roofline/e2e/cpu legs): for profiler runs")
    ap.add_argument("--layers", type=int, default=48,
                    help="layers in the synthetic stack (48 = BASELINE config 2)")
    args = ap.parse_args()
    global LAYERS
    LAYERS = args.layers
    if args.warmup < 3:
        args.warmup = 3
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if world > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group("nccl")
    try:
        if args.workload == "all":
            if args.quick:
                decode_leg(args, rank, world, "decode", headline=True)
            else:
                run_default(args, rank, world)
        else:
            run_single(args, rank, world)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()

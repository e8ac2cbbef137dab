"""Benchmark of the HBA attention hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--config cfg1|cfg3|cfg2|cfg2-bwd|cfg2-aux|cfg3-shard|cfg4] [--no-secondary]

Headline (default): BASELINE config 1 -- one decode step (grouped-query
scoring of every candidate block summary, flat top-16, gather of the
selected 64-token blocks, one fused union softmax over sinks + RoPE window +
routed blocks) for a batch of 64 sequences with 32K cached tokens each
(14/2 heads, dh 64, bf16).  A step is one CUDA-graph replay of
hba_b200_decode with the cache resident in HBM; L2 is flushed (a 256 MB
write) before every timed step, outside the timed events.  `value` is decode
queries/s over all ranks (each rank decodes its own batch: weak scaling).
`e2e` is the same step through the C-ABI call with the query in pinned host
memory and the output + LSE delivered to pinned host memory inside the timed
region: the decode kernel reads and writes the mapped host buffers directly
(zero-copy, one graph node); `e2e.copy_variant` is the same step with an
explicit H2D copy of q and D2H copy of out + LSE around the kernel (three
graph nodes).  The secondary lines measure config 3 (hierarchical decode at
128K), config 2 (prefill at 32K), the backward of that prefill (cfg2-bwd:
dq, dk, dv and the QKNorm gains' gradients), the summarizer's aux-KL teacher
at that shape (cfg2-aux), and with N > 1 ranks config 3 with every
128K context sharded by token range over the N GPUs (one batch of 32
sequences, strong scaling; the fused kernel exchanges the per-rank top-k
lists and softmax partials over NVLink).  `--impl reference` times the CPU oracle port (the
reference algorithm restated in numpy) on the host cores instead.
"""

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "hierarchical-block-attention_b200"))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "HBA attn decode queries/s & prefill tok/s at 32K/128K; % HBM/tensor roofline"
FLUSH_BYTES = 256 << 20


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", default="cfg1", choices=["cfg1", "cfg2", "cfg2-bwd", "cfg2-aux", "cfg3", "cfg3-shard", "cfg4"])
    ap.add_argument("--no-secondary", action="store_true")
    ap.add_argument("--ncu-case", default=None, choices=["cfg1", "cfg3", "cfg2", "cfg2-bwd", "cfg2-aux"],
                    help="profiling target: build this decode workload (cfg3 at batch 4) and run 3 decodes, "
                         "or (cfg2) one prefill forward; no timing, no output")
    return ap.parse_args()


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return dict(hbm=d["hbm_gbs"], bf16=d["bf16_tflops"], bf16_sustained=d.get("bf16_tflops_sustained"),
                    source="measured")
    return dict(hbm=6650.0, bf16=1590.0, bf16_sustained=1400.0, source="fallback")


def traffic_of(key):
    """Per-launch DRAM bytes of a kernel from the committed ncu summary, or None."""
    p = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    if os.path.exists(p):
        return json.load(open(p)).get(key)
    return None


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons during a region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.rows = []
        if self.proc is None:
            return
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out = ""
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 8:
                self.rows.append(f)

    def summary(self):
        if not getattr(self, "rows", None):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[4 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


# ------------------------------------------------------------------ dist ----
def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x, world, dev):
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------- b200 arm ----
def timed_steps(fn, steps, warmup, flush, world, dev, clocks_index, marks=0):
    """Per-step device times (ms) of fn(), L2 flushed before each, outside the
    events.  With marks > 0 the library also records CUDA events at its kernel
    boundaries inside the same timed steps (hba_b200_set_profile_events, a
    fresh set per step): returns (times, clocks, per-kernel mean ms)."""
    from hba_b200 import _lib
    L = _lib.load()
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    kev = [[torch.cuda.Event(enable_timing=True) for _ in range(marks)] for _ in range(steps)]
    for ks in kev:  # torch creates an event's CUDA handle at its first record
        for e in ks:
            e.record()
    torch.cuda.synchronize()
    karr = [(ctypes.c_void_p * marks)(*[e.cuda_event for e in ks]) if marks else None for ks in kev]
    recorded = []
    barrier(world)
    torch.cuda.synchronize()
    try:
        with Clocks(clocks_index) as ck:
            for (e0, e1), arr in zip(evs, karr):
                if marks:
                    L.hba_b200_set_profile_events(arr, marks)
                flush.zero_()
                e0.record()
                fn()
                e1.record()
                if marks:
                    recorded.append(L.hba_b200_profile_events_recorded())
            torch.cuda.synchronize()
    finally:
        if marks:
            L.hba_b200_set_profile_events(None, 0)
    barrier(world)
    times = [a.elapsed_time(b) for a, b in evs]
    if not marks:
        return times, ck.summary()
    per = [[ks[i].elapsed_time(ks[i + 1]) for i in range(k - 1)] for ks, k in zip(kev, recorded)]
    return times, ck.summary(), [statistics.mean(x) for x in zip(*per)]


def kernel_times(call, steps, flush, n_events):
    """Durations (ms) between consecutive profile marks of the library, per step."""
    from hba_b200 import _lib
    L = _lib.load()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(n_events)]
    for e in evs:
        e.record()
    torch.cuda.synchronize()
    arr = (ctypes.c_void_p * n_events)(*[e.cuda_event for e in evs])
    L.hba_b200_set_profile_events(arr, n_events)
    per = []
    try:
        for _ in range(steps):
            flush.zero_()
            call()
            torch.cuda.synchronize()
            k = L.hba_b200_profile_events_recorded()
            per.append([evs[i].elapsed_time(evs[i + 1]) for i in range(k - 1)])
    finally:
        L.hba_b200_set_profile_events(None, 0)
    return [statistics.mean(x) for x in zip(*per)]


def shard_bench(name, steps, warmup, world, rank, local, pk):
    """KV-range sharded decode: one batch of `name`'s sequences whose contexts
    are split by token range over the `world` ranks (strong scaling: the
    batch is the whole job).  Timed with CUDA events, max over ranks."""
    from hba_b200 import baseline_config, synth
    from hba_b200.sharded import HBAShardedDecode
    dev = torch.device("cuda", local)
    cfg, B, n, hier = baseline_config(name)
    summ, qkn = synth.make_weights(cfg, dev, seed=0, gains=False)
    cos, sin = synth.rope_tables(n, cfg.head_dim, 1e6, dev)
    wl = synth.decode_workload(cfg, B, n, hier=hier, seed=1000, device=dev, qkn=qkn)
    sh = HBAShardedDecode(cfg, B, n, summ, qkn, cos, sin, device=dev, hier=hier)  # fused NVLink path
    sh.fill(wl["k"], wl["v"])
    del wl["k"], wl["v"]
    torch.cuda.empty_cache()
    q = wl["q"].contiguous()
    out = torch.empty_like(q)
    lse = torch.empty(B, cfg.n_heads, dtype=torch.float32, device=dev)
    flush = torch.empty(FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    sh.capture(q, out, lse)  # the step as one CUDA graph: epoch bump + the fused shard kernel
    times, clocks = timed_steps(sh.replay, steps, warmup, flush, world, dev, local)
    t_ms = max_over_ranks(statistics.mean(times), world, dev)
    torch.cuda.synchronize(dev)
    status = int(sh.status.item())  # sticky: 1 if any wait of any step gave up
    sh.close()
    res = dict(
        metric=METRIC, value=B / (t_ms * 1e-3), unit="decode queries/s", n_gpus=world, steps=steps, warmup=warmup,
        ms_per_step=t_ms, higher_is_better=True, scaling="strong", vs_baseline=None, dtype="bf16",
        data="synthetic (seeded N(0,1) q/k/v, 8 planted blocks per sequence and kv head)",
        config=dict(workload=f"{name} sharded: decode, batch {B} (whole job), context {n} split over {world} "
                             f"ranks by token range ({sh.n_loc} tokens each)", batch=B, context=n,
                    tokens_per_rank=sh.n_loc, hier=hier,
                    exchanges_per_step=(2 if hier else 1) + 1,
                    l2="flushed (256 MB write) before every timed step",
                    timing="CUDA graph replay of the step (epoch bump + fused kernel), CUDA events, max over ranks",
                    parallelism=f"kv-range shards x{world} (top-k lists and (O, l) partials exchanged inside the "
                                "decode kernel over NVLink peer memory; no collective library call)"),
        gpu_launches=steps * 2,
        device_status=status,
        clocks=clocks,
    )
    if status != 0:
        res["error"] = f"device status {status} on rank {rank}: a bounded wait gave up"
    del sh
    torch.cuda.empty_cache()
    return res


def ncu_case(name, local):
    """Profiling target: the decode workload `name` (cfg3 at batch 4, so that
    the device holds a few GB), decoded 3 times, or (cfg2) one prefill
    forward at full size (~3 GB on the device); no timing, no output."""
    from hba_b200 import HBADecodeCache, baseline_config, synth
    from hba_b200.attention import stream_of
    dev = torch.device("cuda", local)
    if name == "cfg2-aux":
        # one aux-KL teacher of one cfg2 sequence (batch 1: ~1 GB on the device)
        from hba_b200.attention import aux_teacher_b200
        cfg, B, n, hier = baseline_config("cfg2")
        summ, qkn = synth.make_weights(cfg, dev, seed=0, gains=True)
        cos, sin = synth.rope_tables(n, cfg.head_dim, 1e6, dev)
        wl = synth.prefill_workload(cfg, 1, n, seed=0, device=dev)
        aux_teacher_b200(wl["q"], wl["k"], cos, sin, cfg, qkn)
        torch.cuda.synchronize()
        return
    if name == "cfg2-bwd":
        # one forward + backward of one cfg2 sequence (batch 1: ~4 GB on the device)
        from hba_b200 import hba_attention_b200_fused
        cfg, B, n, hier = baseline_config("cfg2")
        summ, qkn = synth.make_weights(cfg, dev, seed=0, gains=True)
        cos, sin = synth.rope_tables(n, cfg.head_dim, 1e6, dev)
        wl = synth.prefill_workload(cfg, 1, n, seed=0, device=dev)
        q, k, v = (wl[x].requires_grad_(True) for x in ("q", "k", "v"))
        out, _ = hba_attention_b200_fused(q, k, v, cos, sin, cfg, summ, qkn)
        out.backward(torch.ones_like(out))
        torch.cuda.synchronize()
        return
    cfg, B, n, hier = baseline_config(name)
    if name == "cfg2":
        from hba_b200 import hba_attention_b200
        summ, qkn = synth.make_weights(cfg, dev, seed=0, gains=False)
        cos, sin = synth.rope_tables(n, cfg.head_dim, 1e6, dev)
        wl = synth.prefill_workload(cfg, B, n, seed=0, device=dev)
        with torch.no_grad():
            hba_attention_b200(wl["q"], wl["k"], wl["v"], cos, sin, cfg, summ, qkn, hier=hier)
        torch.cuda.synchronize()
        return
    if name == "cfg3":
        B = 4
        os.environ["HBA_B200_DECODE_PATH"] = "tc"  # the kernel the full-size bench runs (the default at every batch)
    summ, qkn = synth.make_weights(cfg, dev, seed=0, gains=False)
    cos, sin = synth.rope_tables(n, cfg.head_dim, 1e6, dev)
    wl = synth.decode_workload(cfg, B, n, hier=hier, seed=1000, device=dev, qkn=qkn)
    cache = HBADecodeCache(cfg, B, n, summ, qkn, cos, sin, device=dev, hier=hier)
    cache.append(wl["k"], wl["v"])
    del wl["k"], wl["v"]
    q = wl["q"].contiguous()
    out = torch.empty_like(q)
    lse = torch.empty(B, cfg.n_heads, dtype=torch.float32, device=dev)
    for _ in range(3):
        cache.decode_into(q, out, lse, stream=stream_of(dev))
    torch.cuda.synchronize()


DECODE_DATA = "synthetic (seeded N(0,1) q/k/v, 8 planted blocks per sequence and kv head)"


def decode_config(name, world):
    """The `config` of a decode line; the reference arm prints the same one."""
    from hba_b200.config import baseline_config
    cfg, B, n, hier = baseline_config(name)
    return dict(workload=f"{name}: decode, batch {B}/rank, context {n}, {cfg.n_heads}/{cfg.n_kv} heads, "
                         f"dh {cfg.head_dim}, {'hierarchical beam ' + str(cfg.beam) if hier else 'flat'} "
                         f"top-{cfg.k_blocks}",
                batch_per_rank=B, context=n, n_heads=cfg.n_heads, n_kv=cfg.n_kv, head_dim=cfg.head_dim,
                window=cfg.window, sinks=cfg.sinks, block=cfg.block, slots=cfg.slots, k_blocks=cfg.k_blocks,
                hier=hier, fanout=cfg.fanout if hier else None, beam=cfg.beam if hier else None,
                l2="flushed (256 MB write) before every timed step", timing="CUDA graph replay, CUDA events",
                parallelism=f"replicas x{world} (batch-sharded, no collective)")


def decode_bench(name, steps, warmup, world, rank, local, pk):
    from hba_b200 import HBADecodeCache, baseline_config, synth
    from hba_b200.attention import stream_of
    dev = torch.device("cuda", local)
    cfg, B, n, hier = baseline_config(name)
    G, dh, Hq, Hkv = cfg.G, cfg.head_dim, cfg.n_heads, cfg.n_kv
    summ, qkn = synth.make_weights(cfg, dev, seed=0, gains=False)
    cos, sin = synth.rope_tables(n, dh, 1e6, dev)
    wl = synth.decode_workload(cfg, B, n, hier=hier, seed=1000 + rank, device=dev, qkn=qkn)
    cache = HBADecodeCache(cfg, B, n, summ, qkn, cos, sin, device=dev, hier=hier)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    cache.append(wl["k"], wl["v"])
    torch.cuda.synchronize()
    build_s = time.perf_counter() - t0
    del wl["k"], wl["v"]
    q = wl["q"].contiguous()
    out = torch.empty_like(q)
    lse = torch.empty(B, Hq, dtype=torch.float32, device=dev)
    flush = torch.empty(FLUSH_BYTES // 4, dtype=torch.float32, device=dev)

    def step_direct():
        cache.decode_into(q, out, lse, stream=stream_of(dev))

    step_direct()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        cache.decode_into(q, out, lse, stream=stream_of(dev))
    times, clocks = timed_steps(graph.replay, steps, warmup, flush, world, dev, local)
    t_ms = statistics.mean(times)
    t_ms = max_over_ranks(t_ms, world, dev)

    # dominant kernel: the tcgen05 / fused paths' step IS one kernel launch,
    # so its time is the graph-replayed step measured above (the same timed
    # region as ms_per_step); the split path's attend kernel is timed between
    # the library's event marks.  The eager per-launch time is kept beside it.
    from hba_b200 import _lib
    nmarks = 4 if hier else 3          # begin | select (super, child) | attend
    kt = kernel_times(step_direct, max(3, min(steps, 10)), flush, nmarks)
    kernels = _lib.load().hba_b200_last_kernels().decode()
    single = "+" not in kernels
    attend_ms = t_ms if single else kt[-1]
    keys = cfg.sinks + cfg.window + cfg.k_blocks * cfg.block
    attend_bytes = B * Hkv * (keys * dh * 2 * 2 + G * dh * 2 * 2)
    if hier:
        ns = n // cfg.block // cfg.fanout
        summ_bytes = B * Hkv * (ns + cfg.beam * cfg.fanout) * cfg.slots * dh * 2
    else:
        n_cand = (n - 1 - cfg.window + 1) // cfg.block - 1
        summ_bytes = B * Hkv * n_cand * cfg.slots * dh * 2
    step_bytes = attend_bytes + summ_bytes
    dom_kernel = kernels if single else "decode_attend_kernel"
    dom_bytes = step_bytes if single else attend_bytes
    achieved = dom_bytes / (attend_ms * 1e-3) / 1e9
    traffic = traffic_of(f"{dom_kernel}_{name}")

    # e2e: the C-ABI call with the query copied from pinned host memory and
    # out + lse (one device buffer) copied back, captured as one CUDA graph as
    # a serving loop runs it
    q_host = q.cpu().pin_memory()
    ob, lb = out.numel() * out.element_size(), lse.numel() * lse.element_size()
    io = torch.empty(ob + lb, dtype=torch.uint8, device=dev)
    out_e = io[:ob].view(out.dtype).view(out.shape)
    lse_e = io[ob:].view(lse.dtype).view(lse.shape)
    io_host = torch.empty(ob + lb, dtype=torch.uint8).pin_memory()

    def step_e2e_body():
        q.copy_(q_host, non_blocking=True)
        cache.decode_into(q, out_e, lse_e, stream=stream_of(dev))
        io_host.copy_(io, non_blocking=True)

    step_e2e_body()
    torch.cuda.synchronize()
    g_e2e = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_e2e):
        step_e2e_body()
    e2e_times, _ = timed_steps(g_e2e.replay, steps, warmup, flush, world, dev, local)
    e2e_copy_ms = max_over_ranks(statistics.mean(e2e_times), world, dev)
    # the copied-back result is the device result
    assert torch.equal(io_host[:ob].view(out.dtype).view(out.shape), out_e.cpu())

    # e2e, zero-copy (the headline): q sits in mapped pinned host memory and
    # the decode kernel reads it from there and writes out + lse back into it
    # -- the step's host -> device and device -> host traffic with no copy
    # launch around the kernel (hba_b200_host_alloc)
    from hba_b200.hostio import MappedHostBuffer
    qbytes = q.numel() * q.element_size()
    hbuf = MappedHostBuffer(qbytes + ob + lb)
    hbuf.host_view(q.dtype, q.shape).copy_(q_host)
    out_z = hbuf.host_view(out.dtype, out.shape, offset=qbytes)
    q_d, out_d, lse_d = hbuf.device_view(0), hbuf.device_view(qbytes), hbuf.device_view(qbytes + ob)

    def step_zero_copy():
        cache.decode_into(q_d, out_d, lse_d, stream=stream_of(dev))

    step_zero_copy()
    torch.cuda.synchronize()
    g_zc = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_zc):
        step_zero_copy()
    zc_times, _ = timed_steps(g_zc.replay, steps, warmup, flush, world, dev, local)
    e2e_ms = max_over_ranks(statistics.mean(zc_times), world, dev)
    torch.cuda.synchronize()
    assert torch.equal(out_z, out_e.cpu())  # the host-written result is the device result
    del g_zc
    hbuf.close()

    res = dict(
        metric=METRIC, value=B * world / (t_ms * 1e-3), unit="decode queries/s", n_gpus=world, steps=steps,
        warmup=warmup, ms_per_step=t_ms, higher_is_better=True, scaling="weak", vs_baseline=None, dtype="bf16",
        data=DECODE_DATA,
        config=decode_config(name, world),
        roofline=dict(bound="hbm", kernel=dom_kernel, achieved=achieved, peak=pk["hbm"], unit="GB/s",
                      frac=achieved / pk["hbm"], peak_source=pk["source"], traffic=traffic,
                      algorithmic_bytes_per_launch=dom_bytes, kernel_ms=attend_ms,
                      kernel_timing=("the step's single kernel launch, graph-replayed in the timed steps "
                                     "(= ms_per_step)") if single else
                                    "eager launches between the library's event marks",
                      kernel_ms_eager=kt[-1]),
        step_effective_gbs=step_bytes / (t_ms * 1e-3) / 1e9,
        step_algorithmic_bytes=step_bytes,
        decode_kernels=kernels,
        kernel_ms={"select": kt[:-1], "attend": attend_ms} if not single else {kernels: attend_ms},
        cache_build_s=build_s,
        e2e=dict(value=B * world / (e2e_ms * 1e-3), unit="decode queries/s", ms_per_step=e2e_ms,
                 h2d_bytes_per_step=q.numel() * q.element_size(), d2h_bytes_per_step=ob + lb,
                 timing="one CUDA graph per step: hba_b200_decode reading q from and writing out + lse to "
                        "mapped pinned host memory (zero-copy; hba_b200_host_alloc)",
                 copy_variant=dict(value=B * world / (e2e_copy_ms * 1e-3), ms_per_step=e2e_copy_ms,
                                   timing="one CUDA graph per step: pinned H2D of q, hba_b200_decode, "
                                          "D2H of out + lse")),
        gpu_launches=steps * (len(kt) + 0),
        clocks=clocks,
    )
    sample = None
    if rank == 0:
        sample = cpu_decode_sample(cache, q, cfg, hier, n)
    res["cpu_baseline"] = sample
    del cache
    torch.cuda.empty_cache()
    return res


def cpu_decode_sample(cache, q, cfg, hier, n, seqs=2):
    """Oracle (numpy port, one thread) decode of `seqs` sequences of the same
    workload, copied from the device cache."""
    from oracle import hba_oracle as orc
    from hba_b200.ops import qknorm_b200
    try:
        from threadpoolctl import threadpool_limits
    except Exception:  # pragma: no cover
        threadpool_limits = None
    qc = qknorm_b200(q[:seqs], cache.q_gain).float().cpu().numpy()
    nb = n // cfg.block
    data = []
    for b in range(seqs):
        kc = cache.tokens("k")[b:b + 1, :n].float().cpu().numpy()
        v = cache.tokens("v")[b:b + 1, :n].float().cpu().numpy()
        S0 = cache.summaries[b:b + 1, :, :nb].float().cpu().numpy()
        S1 = cache.supers[b:b + 1, :, :-(-nb // cfg.fanout)].float().cpu().numpy() if hier else None
        data.append((kc, v, S0, S1))
    cos, sin = cache.cos.cpu().numpy(), cache.sin.cpu().numpy()
    ocfg = dict(block=cfg.block, window=cfg.window, sinks=cfg.sinks, k_blocks=cfg.k_blocks, fanout=cfg.fanout,
                beam=cfg.beam, qknorm=cfg.qknorm, content_scale_mode=cfg.content_scale_mode, temp_c=cfg.temp_c,
                n_cal=cfg.n_cal, native_ctx=cfg.native_ctx)
    scale = orc.union_scale(cfg.qknorm, cfg.content_scale_mode, cfg.temp_c, cfg.n_cal, cfg.native_ctx,
                            cfg.head_dim, n)
    ctx = threadpool_limits(limits=1) if threadpool_limits else None
    if ctx:
        ctx.__enter__()
    t0 = time.perf_counter()
    for b in range(seqs):
        kc, v, S0, S1 = data[b]
        orc.decode(qc[b:b + 1], kc, v, cos, sin, S0, S1, ocfg, scale, None, hier=hier, bf16=True, qknorm_q=False)
    dt = time.perf_counter() - t0
    if ctx:
        ctx.__exit__(None, None, None)
    return dict(value=seqs / dt, unit="decode queries/s", cores=1, kind="port",
                sample=f"{seqs} sequences of the same workload (one query each, cache contents copied "
                       f"from the device), numpy oracle, 1 thread")


def prefill_attended_keys(cfg, n):
    """Sum over query positions i < n of the union's keys: sinks min(S, i+1),
    window, routed valid picks (min(k, candidates) blocks)."""
    i = np.arange(n)
    win = np.maximum(0, i - np.maximum(cfg.sinks, i - cfg.window + 1) + 1)
    sink = np.minimum(cfg.sinks, i + 1)
    lim = i - cfg.window + 1
    ncand = np.where(lim >= 2 * cfg.block, lim // cfg.block - 1, 0)
    routed = np.minimum(cfg.k_blocks, ncand) * cfg.block
    return float((win + sink + routed).sum())


def cpu_prefill_sample(q, k, v, cos, sin, cfg, summ, qkn, n, B, rows=32):
    """The oracle (numpy port, one thread) on a bounded sample of the same
    prefill workload: the summaries of one whole sequence (every kv head),
    then the selection and union of `rows` query positions of it (all heads),
    spread over the sequence.  Projected to the whole batch: B x (summary time
    + n x the mean per-row time); the value is tokens/s of that projection."""
    from oracle import hba_oracle as orc
    try:
        from threadpoolctl import threadpool_limits
    except Exception:  # pragma: no cover
        threadpool_limits = None
    r = np.random.default_rng(0)
    rws = np.sort(r.choice(np.arange(cfg.window, n), size=rows, replace=False))
    qs = q[0, torch.as_tensor(rws, device=q.device)].float().cpu().numpy()[None]   # [1, rows, Hq, dh]
    ks, vs = k[:1].float().cpu().numpy(), v[:1].float().cpu().numpy()
    cosn, sinn = cos.float().cpu().numpy(), sin.float().cpu().numpy()
    probes, proj = summ.probes.float().cpu().numpy(), summ.proj.float().cpu().numpy()
    qg, kg = qkn.q.gain.float().cpu().numpy(), qkn.k.gain.float().cpu().numpy()
    ocfg = dict(block=cfg.block, window=cfg.window, sinks=cfg.sinks, k_blocks=cfg.k_blocks, fanout=cfg.fanout,
                beam=cfg.beam, qknorm=cfg.qknorm, content_scale_mode=cfg.content_scale_mode, temp_c=cfg.temp_c,
                n_cal=cfg.n_cal, native_ctx=cfg.native_ctx)
    scale = orc.union_scale(cfg.qknorm, cfg.content_scale_mode, cfg.temp_c, cfg.n_cal, cfg.native_ctx,
                            cfg.head_dim, n)
    Hkv, G = cfg.n_kv, cfg.n_heads // cfg.n_kv
    ctx = threadpool_limits(limits=1) if threadpool_limits else None
    if ctx:
        ctx.__enter__()
    try:
        t0 = time.perf_counter()
        kc = orc.head_rmsnorm(ks, kg, bf16=True)
        S0 = orc.summarize(kc, probes, proj, cfg.block)
        t_summ = time.perf_counter() - t0
        qc = orc.head_rmsnorm(qs, qg, bf16=True)
        qgr = orc.grouped_query(qc, Hkv, bf16=True)                                   # [1, Hkv, rows, dh]
        t1 = time.perf_counter()
        for g in range(Hkv):
            idx, val, ok = orc.select_rows(rws, qgr[0, g], S0[0, g], None, ocfg, scale, False)
            orc.union_attention_rows(rws, qc[0, :, g * G:(g + 1) * G], kc[0, :, g], vs[0, :, g], cosn, sinn, idx,
                                     ok, cfg.sinks, cfg.window, cfg.block, scale, bf16=True)
        t_rows = time.perf_counter() - t1
    finally:
        if ctx:
            ctx.__exit__(None, None, None)
    t_full = B * (t_summ + n * t_rows / rows)
    return dict(value=B * n / t_full, unit="prefill tokens/s", cores=1, kind="port",
                sample=f"numpy oracle, 1 thread: summaries of 1 whole sequence ({t_summ:.2f} s) + selection and "
                       f"union of {rows} query rows of it, all {cfg.n_heads} heads ({t_rows:.2f} s); projected "
                       f"linearly to {B} x {n} tokens (rows spread over positions >= the window, where each "
                       f"row attends its full ~2.1K keys)",
                measured_s=t_summ + t_rows, projected_s=t_full)


def prefill_bench(name, steps, warmup, world, rank, local, pk):
    from hba_b200 import baseline_config, synth
    from hba_b200.attention import (as_f32, c_config, gains, ptr, stream_of, summarizer_weights, union_scale)
    from hba_b200 import _lib
    dev = torch.device("cuda", local)
    cfg, B, n, hier = baseline_config(name)
    dh, Hq, Hkv = cfg.head_dim, cfg.n_heads, cfg.n_kv
    summ, qkn = synth.make_weights(cfg, dev, seed=0, gains=False)
    cos, sin = synth.rope_tables(n, dh, 1e6, dev)
    wl = synth.prefill_workload(cfg, B, n, seed=2000 + rank, device=dev)
    q, k, v = wl["q"], wl["k"], wl["v"]
    out = torch.empty_like(q)
    lse = torch.empty(B, Hq, n, dtype=torch.float32, device=dev)
    c = c_config(cfg, hier)
    L = _lib.load()
    ws_bytes = L.hba_b200_prefill_workspace_size(ctypes.byref(c), B, n)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    qg, kg = gains(qkn, dev)
    probes, proj = summarizer_weights(summ, dev)
    scale = union_scale(cfg, dh, n)
    flush = torch.empty(FLUSH_BYTES // 4, dtype=torch.float32, device=dev)

    def call(qq, kk, vv, oo):
        st = L.hba_b200_prefill(ctypes.byref(c), B, n, ctypes.c_float(scale), ptr(qq), ptr(kk), ptr(vv), ptr(cos),
                                ptr(sin), ptr(qg), ptr(kg), ptr(probes), ptr(proj), ptr(oo), ptr(lse), None, None,
                                ptr(ws), ws_bytes, stream_of(dev))
        _lib.check(st, "hba_b200_prefill")

    def step():
        call(q, k, v, out)

    # the step's kernels are timed between the library's marks inside the same timed steps
    nmarks = 5 if not hier else 7
    times, clocks, kt = timed_steps(step, steps, warmup, flush, world, dev, local, marks=nmarks)
    t_ms = max_over_ranks(statistics.mean(times), world, dev)
    kernels = _lib.load().hba_b200_last_kernels().decode().split("+")
    attend_ms = kt[-1]
    keys = prefill_attended_keys(cfg, n)
    flops = 4.0 * dh * Hq * B * keys
    achieved = flops / (attend_ms * 1e-3) / 1e12
    status = L.hba_b200_device_status(ptr(ws), 0, stream_of(dev))

    # e2e: the C-ABI call with q/k/v copied in from pinned host memory and the
    # output copied back to pinned host memory, every step, inside the timed
    # region (one stream: H2D, the prefill kernels, D2H)
    qh, kh, vh = (t.cpu().pin_memory() for t in (q, k, v))
    oh = torch.empty(out.shape, dtype=out.dtype).pin_memory()

    def step_e2e():
        q.copy_(qh, non_blocking=True)
        k.copy_(kh, non_blocking=True)
        v.copy_(vh, non_blocking=True)
        call(q, k, v, out)
        oh.copy_(out, non_blocking=True)

    e2e_times, _ = timed_steps(step_e2e, max(2, min(steps, 3)), 1, flush, world, dev, local)
    e2e_ms = max_over_ranks(statistics.mean(e2e_times), world, dev)
    torch.cuda.synchronize()
    assert torch.equal(oh, out.cpu())  # the copied-back result is the device result
    h2d = sum(t.numel() * t.element_size() for t in (q, k, v))
    d2h = out.numel() * out.element_size()
    res = dict(
        metric=METRIC, value=B * n * world / (t_ms * 1e-3), unit="prefill tokens/s", n_gpus=world, steps=steps,
        warmup=warmup, ms_per_step=t_ms, higher_is_better=True, scaling="weak", vs_baseline=None, dtype="bf16",
        data="synthetic (seeded N(0,1) q/k/v; 64-query tiles share a topic with 8 planted blocks)",
        config=dict(workload=f"{name}: prefill, batch {B}/rank, seq {n}, {Hq}/{Hkv} heads, dh {dh}, flat top-16",
                    batch_per_rank=B, seq_len=n, n_heads=Hq, n_kv=Hkv, head_dim=dh,
                    l2="flushed (256 MB write) before every timed step",
                    timing="eager C-ABI call per step, CUDA events; kernel times between the library's event "
                           "marks in the same steps"),
        roofline=dict(bound="tensor", kernel=kernels[-1], achieved=achieved, peak=pk["bf16"], unit="TFLOP/s",
                      frac=achieved / pk["bf16"], peak_source=pk["source"],
                      traffic=traffic_of(f"{kernels[-1]}_{name}"), attended_flops=flops, kernel_ms=attend_ms),
        kernel_ms={f"{i}:{k_}": t for i, (k_, t) in enumerate(zip(kernels, kt))},
        e2e=dict(value=B * n * world / (e2e_ms * 1e-3), unit="prefill tokens/s", ms_per_step=e2e_ms,
                 h2d_bytes_per_step=h2d, d2h_bytes_per_step=d2h,
                 timing="per step: pinned H2D of q, k, v, hba_b200_prefill, pinned D2H of out, one stream"),
        gpu_launches=steps * len(kernels), device_status=status, clocks=clocks,
    )
    if rank == 0:
        res["cpu_baseline"] = cpu_prefill_sample(q, k, v, cos, sin, cfg, summ, qkn, n, B)
    del q, k, v, ws, wl, qh, kh, vh, oh
    torch.cuda.empty_cache()
    return res


def cpu_prefill_bwd_sample(q, k, v, cos, sin, cfg, qkn, sel, dout, n, B, rows=16):
    """The oracle's union-softmax backward (numpy port, one thread) on a
    bounded sample of the same workload: `rows` query positions (>= the
    window) of one (sequence, kv head), all its query heads, with the GPU
    forward's picks.  Projected linearly to every row of the batch (B x Hkv x
    n rows of the same per-row work); the value is tokens/s of that projection."""
    from oracle import hba_oracle as orc
    try:
        from threadpoolctl import threadpool_limits
    except Exception:  # pragma: no cover
        threadpool_limits = None
    r = np.random.default_rng(1)
    rws = np.sort(r.choice(np.arange(cfg.window, n), size=rows, replace=False))
    G = cfg.n_heads // cfg.n_kv
    idx = torch.as_tensor(rws, device=q.device)
    qs = q[0, idx, :G].float().cpu().numpy()                   # [rows, G, dh], kv head 0
    dos = dout[0, idx, :G].float().cpu().numpy()
    ks, vs = k[0, :, 0].float().cpu().numpy(), v[0, :, 0].float().cpu().numpy()
    cosn, sinn = cos.float().cpu().numpy(), sin.float().cpu().numpy()
    qg, kg = qkn.q.gain.float().cpu().numpy(), qkn.k.gain.float().cpu().numpy()
    si = sel[0, 0, idx].cpu().numpy()
    scale = orc.union_scale(cfg.qknorm, cfg.content_scale_mode, cfg.temp_c, cfg.n_cal, cfg.native_ctx,
                            cfg.head_dim, n)
    ctx = threadpool_limits(limits=1) if threadpool_limits else None
    if ctx:
        ctx.__enter__()
    try:
        t0 = time.perf_counter()
        qc = orc.head_rmsnorm(qs, qg[:G], bf16=True)
        kc = orc.head_rmsnorm(ks[:, None], kg[:1], bf16=True)[:, 0]
        dq, dk, dv = orc.union_backward_rows(rws, qc, kc, vs, cosn, sinn, np.maximum(si, 0), si >= 0, cfg.sinks,
                                             cfg.window, cfg.block, scale, dos, bf16=True)
        orc.head_rmsnorm_backward(qs, qg[:G], dq)
        t_rows = time.perf_counter() - t0
    finally:
        if ctx:
            ctx.__exit__(None, None, None)
    t_full = B * cfg.n_kv * n * t_rows / rows
    return dict(value=B * n / t_full, unit="prefill backward tokens/s", cores=1, kind="port",
                sample=f"numpy oracle backward, 1 thread: {rows} query rows (all {G} heads of one kv head, positions "
                       f">= the window) of one sequence ({t_rows:.2f} s); projected linearly to {B} x {cfg.n_kv} "
                       f"kv heads x {n} rows",
                measured_s=t_rows, projected_s=t_full)


def prefill_bwd_bench(name, steps, warmup, world, rank, local, pk):
    """The backward of the cfg2 prefill (hba_b200_prefill_backward): dq, dk,
    dv and the QKNorm gains' gradients for a seeded output gradient, the
    forward's outputs and picks computed once before the timed steps."""
    from hba_b200 import baseline_config, synth
    from hba_b200.attention import as_f32, c_config, gains, ptr, stream_of, summarizer_weights, union_scale
    from hba_b200 import _lib
    dev = torch.device("cuda", local)
    cfg, B, n, hier = baseline_config(name)
    dh, Hq, Hkv = cfg.head_dim, cfg.n_heads, cfg.n_kv
    summ, qkn = synth.make_weights(cfg, dev, seed=0, gains=True)
    cos, sin = synth.rope_tables(n, dh, 1e6, dev)
    wl = synth.prefill_workload(cfg, B, n, seed=2000 + rank, device=dev)
    q, k, v = wl["q"], wl["k"], wl["v"]
    c = c_config(cfg, False)
    L = _lib.load()
    qg, kg = gains(qkn, dev)
    probes, proj = summarizer_weights(summ, dev)
    scale = union_scale(cfg, dh, n)
    out = torch.empty_like(q)
    lse = torch.empty(B, Hq, n, dtype=torch.float32, device=dev)
    sel_i = torch.empty(B, Hkv, n, cfg.k_blocks, dtype=torch.int32, device=dev)
    sel_s = torch.empty(B, Hkv, n, cfg.k_blocks, dtype=torch.float32, device=dev)
    fws_bytes = L.hba_b200_prefill_workspace_size(ctypes.byref(c), B, n)
    fws = torch.empty(fws_bytes, dtype=torch.uint8, device=dev)
    _lib.check(L.hba_b200_prefill(ctypes.byref(c), B, n, ctypes.c_float(scale), ptr(q), ptr(k), ptr(v), ptr(cos),
                                  ptr(sin), ptr(qg), ptr(kg), ptr(probes), ptr(proj), ptr(out), ptr(lse), ptr(sel_i),
                                  ptr(sel_s), ptr(fws), fws_bytes, stream_of(dev)), "hba_b200_prefill")
    del fws
    g = torch.Generator(device="cpu").manual_seed(3000 + rank)
    dout = torch.randn(q.shape, generator=g).to(dev, torch.bfloat16)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    dqg = torch.empty(Hq, dtype=torch.float32, device=dev)
    dkg = torch.empty(Hkv, dtype=torch.float32, device=dev)
    ws_bytes = L.hba_b200_prefill_backward_workspace_size(ctypes.byref(c), B, n)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    flush = torch.empty(FLUSH_BYTES // 4, dtype=torch.float32, device=dev)

    def call(qq, kk, vv, gg):
        st = L.hba_b200_prefill_backward(ctypes.byref(c), B, n, ctypes.c_float(scale), ptr(qq), ptr(kk), ptr(vv),
                                         ptr(cos), ptr(sin), ptr(qg), ptr(kg), ptr(out), ptr(lse), ptr(sel_i),
                                         ptr(gg), ptr(dq), ptr(dk), ptr(dv), ptr(dqg), ptr(dkg), ptr(ws), ws_bytes,
                                         stream_of(dev))
        _lib.check(st, "hba_b200_prefill_backward")

    def step():
        call(q, k, v, dout)

    times, clocks, kt = timed_steps(step, steps, warmup, flush, world, dev, local, marks=4)
    t_ms = max_over_ranks(statistics.mean(times), world, dev)
    kernels = _lib.load().hba_b200_last_kernels().decode().split("+")
    status = L.hba_b200_device_status(ptr(ws), 0, stream_of(dev))
    main_ms = kt[1]
    keys = prefill_attended_keys(cfg, n)
    flops = 10.0 * dh * Hq * B * keys  # 5 products of the forward's 2 per attended (row, key)

    # e2e: q, k, v, dout in from pinned host memory, dq / dk / dv back, every step
    qh, kh, vh, gh = (t.cpu().pin_memory() for t in (q, k, v, dout))
    dqh, dkh, dvh = (torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in (dq, dk, dv))

    def step_e2e():
        q.copy_(qh, non_blocking=True)
        k.copy_(kh, non_blocking=True)
        v.copy_(vh, non_blocking=True)
        dout.copy_(gh, non_blocking=True)
        call(q, k, v, dout)
        dqh.copy_(dq, non_blocking=True)
        dkh.copy_(dk, non_blocking=True)
        dvh.copy_(dv, non_blocking=True)

    e2e_times, _ = timed_steps(step_e2e, max(2, min(steps, 3)), 1, flush, world, dev, local)
    e2e_ms = max_over_ranks(statistics.mean(e2e_times), world, dev)
    torch.cuda.synchronize()
    h2d = sum(t.numel() * t.element_size() for t in (q, k, v, dout))
    d2h = sum(t.numel() * t.element_size() for t in (dq, dk, dv))
    achieved = flops / (main_ms * 1e-3) / 1e12
    res = dict(
        metric="prefill backward tokens/s", value=B * n * world / (t_ms * 1e-3), unit="prefill backward tokens/s",
        n_gpus=world, steps=steps, warmup=warmup, ms_per_step=t_ms, higher_is_better=True, scaling="weak",
        vs_baseline=None, dtype="bf16",
        data="synthetic (the cfg2 prefill workload, seeded N(0,1) output gradient, gains ~U(0.6, 1.6))",
        config=dict(workload=f"{name}-bwd: backward of the prefill, batch {B}/rank, seq {n}, {Hq}/{Hkv} heads, "
                             f"dh {dh}, flat top-16 (the forward's picks)",
                    batch_per_rank=B, seq_len=n, n_heads=Hq, n_kv=Hkv, head_dim=dh,
                    l2="flushed (256 MB write) before every timed step",
                    timing="eager C-ABI call per step, CUDA events; kernel times between the library's event "
                           "marks in the same steps"),
        roofline=dict(bound="tensor", kernel="prefill_bwd_kernel", achieved=achieved, peak=pk["bf16"],
                      unit="TFLOP/s", frac=achieved / pk["bf16"], peak_source=pk["source"],
                      traffic=traffic_of(f"prefill_bwd_kernel_{name}"), algorithmic_flops=flops, kernel_ms=main_ms),
        kernel_ms={"pre-pass+delta": kt[0], "prefill_bwd_kernel": kt[1], "bwd_norm_kernel x3": kt[2]},
        e2e=dict(value=B * n * world / (e2e_ms * 1e-3), unit="prefill backward tokens/s", ms_per_step=e2e_ms,
                 h2d_bytes_per_step=h2d, d2h_bytes_per_step=d2h,
                 timing="per step: pinned H2D of q, k, v, dout, hba_b200_prefill_backward, pinned D2H of dq, dk, dv"),
        gpu_launches=steps * 7,  # qknorm_rope x2, bwd_delta, prefill_bwd, bwd_norm x3
        device_status=status, clocks=clocks,
    )
    if rank == 0:
        res["cpu_baseline"] = cpu_prefill_bwd_sample(q, k, v, cos, sin, cfg, qkn, sel_i, dout, n, B)
    del q, k, v, ws, wl, qh, kh, vh, gh, dqh, dkh, dvh, dq, dk, dv, dout
    torch.cuda.empty_cache()
    return res


def aux_candidate_keys(cfg, n):
    """Sum over query positions of the candidate keys the aux teacher scores
    (every key of blocks 1 .. last_candidate(i))."""
    i = np.arange(n)
    lim = i - cfg.window + 1
    bmax = np.where(lim >= 2 * cfg.block, lim // cfg.block - 1, 0)
    return float((np.minimum(bmax, n // cfg.block - 1) * cfg.block).sum())


def aux_teacher_bench(name, steps, warmup, world, rank, local, pk):
    """The summarizer's aux-KL teacher (hba_b200_aux_teacher) at the cfg2
    prefill shape: pstar [B, Hkv, n, nb] from q, k (O(n^2): two passes of
    QK^T over every query's candidate keys)."""
    from hba_b200 import baseline_config, synth
    from hba_b200.attention import as_f32, c_config, gains, ptr, stream_of, union_scale
    from hba_b200 import _lib
    dev = torch.device("cuda", local)
    cfg, B, n, hier = baseline_config(name)
    dh, Hq, Hkv = cfg.head_dim, cfg.n_heads, cfg.n_kv
    nb = n // cfg.block
    summ, qkn = synth.make_weights(cfg, dev, seed=0, gains=True)
    cos, sin = synth.rope_tables(n, dh, 1e6, dev)
    wl = synth.prefill_workload(cfg, B, n, seed=4000 + rank, device=dev)
    q, k = wl["q"], wl["k"]
    del wl
    c = c_config(cfg, False)
    L = _lib.load()
    qg, kg = gains(qkn, dev)
    scale = union_scale(cfg, dh, n)
    pstar = torch.empty(B, Hkv, n, nb, dtype=torch.float32, device=dev)
    ws_bytes = L.hba_b200_aux_teacher_workspace_size(ctypes.byref(c), B, n)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    flush = torch.empty(FLUSH_BYTES // 4, dtype=torch.float32, device=dev)

    def call(qq, kk):
        st = L.hba_b200_aux_teacher(ctypes.byref(c), B, n, ctypes.c_float(scale), ptr(qq), ptr(kk), ptr(cos),
                                    ptr(sin), ptr(qg), ptr(kg), ptr(pstar), ptr(ws), ws_bytes, stream_of(dev))
        _lib.check(st, "hba_b200_aux_teacher")

    def step():
        call(q, k)

    times, clocks, kt = timed_steps(step, steps, warmup, flush, world, dev, local, marks=3)
    t_ms = max_over_ranks(statistics.mean(times), world, dev)
    status = L.hba_b200_device_status(ptr(ws), 0, stream_of(dev))
    keys = aux_candidate_keys(cfg, n)
    flops = 2.0 * dh * Hq * B * keys  # the reference's one QK^T over the candidate keys (the kernel runs it twice)
    main_ms = kt[1]
    achieved = flops / (main_ms * 1e-3) / 1e12
    qh, kh = q.cpu().pin_memory(), k.cpu().pin_memory()
    ph = torch.empty(pstar.shape, dtype=pstar.dtype).pin_memory()

    def step_e2e():
        q.copy_(qh, non_blocking=True)
        k.copy_(kh, non_blocking=True)
        call(q, k)
        ph.copy_(pstar, non_blocking=True)

    e2e_times, _ = timed_steps(step_e2e, 2, 1, flush, world, dev, local)
    e2e_ms = max_over_ranks(statistics.mean(e2e_times), world, dev)
    res = dict(
        metric="aux-KL teacher tokens/s", value=B * n * world / (t_ms * 1e-3), unit="aux teacher tokens/s",
        n_gpus=world, steps=steps, warmup=warmup, ms_per_step=t_ms, higher_is_better=True, scaling="weak",
        vs_baseline=None, dtype="bf16", data="synthetic (the cfg2 prefill workload's q, k; gains ~U(0.6, 1.6))",
        config=dict(workload=f"{name}-aux: the summarizer's aux-KL teacher, batch {B}/rank, seq {n}, {Hq}/{Hkv} "
                             f"heads, dh {dh}", batch_per_rank=B, seq_len=n, n_heads=Hq, n_kv=Hkv, head_dim=dh,
                    l2="flushed (256 MB write) before every timed step",
                    timing="eager C-ABI call per step, CUDA events; kernel times between the library's event marks"),
        roofline=dict(bound="tensor", kernel="aux_teacher_kernel", achieved=achieved, peak=pk["bf16"], unit="TFLOP/s",
                      frac=achieved / pk["bf16"], peak_source=pk["source"], traffic=traffic_of(f"aux_teacher_kernel_{name}"),
                      algorithmic_flops=flops, kernel_ms=main_ms),
        kernel_ms={"pre-pass": kt[0], "aux_teacher_kernel": kt[1]},
        e2e=dict(value=B * n * world / (e2e_ms * 1e-3), unit="aux teacher tokens/s", ms_per_step=e2e_ms,
                 h2d_bytes_per_step=q.numel() * 2 + k.numel() * 2, d2h_bytes_per_step=pstar.numel() * 4,
                 timing="per step: pinned H2D of q, k, hba_b200_aux_teacher, pinned D2H of pstar"),
        gpu_launches=steps * 3, device_status=status, clocks=clocks,
    )
    if rank == 0:
        res["cpu_baseline"] = cpu_aux_sample(q, k, cfg, qkn, n, B, scale)
    del q, k, ws, pstar, qh, kh, ph
    torch.cuda.empty_cache()
    return res


def cpu_aux_sample(q, k, cfg, qkn, n, B, scale, rows=8):
    """The oracle's teacher (numpy, one thread) for `rows` query positions of
    one (sequence, kv head) (all its heads, scoring every key), projected
    linearly to every row of the batch."""
    from oracle import hba_oracle as orc
    try:
        from threadpoolctl import threadpool_limits
    except Exception:  # pragma: no cover
        threadpool_limits = None
    G = cfg.n_heads // cfg.n_kv
    r = np.random.default_rng(2)
    rws = np.sort(r.choice(np.arange(cfg.window + 2 * cfg.block, n), size=rows, replace=False))
    idx = torch.as_tensor(rws, device=q.device)
    qg, kg = qkn.q.gain.float().cpu().numpy(), qkn.k.gain.float().cpu().numpy()
    qs = q[0, idx, :G].float().cpu().numpy()
    ks = k[0, :, :1].float().cpu().numpy()
    ctx = threadpool_limits(limits=1) if threadpool_limits else None
    if ctx:
        ctx.__enter__()
    try:
        t0 = time.perf_counter()
        qc = orc.head_rmsnorm(qs, qg[:G], bf16=True)
        kc = orc.head_rmsnorm(ks, kg[:1], bf16=True)[:, 0]
        orc.aux_teacher_rows(rws, qc, kc, dict(block=cfg.block, window=cfg.window), scale)
        t_rows = time.perf_counter() - t0
    finally:
        if ctx:
            ctx.__exit__(None, None, None)
    t_full = B * cfg.n_kv * n * t_rows / rows
    return dict(value=B * n / t_full, unit="aux teacher tokens/s", cores=1, kind="port",
                sample=f"numpy oracle teacher, 1 thread: {rows} query rows (all {G} heads of one kv head, positions "
                       f"past the window, every key scored as the reference does) of one sequence ({t_rows:.2f} s); "
                       f"projected linearly to {B} x {cfg.n_kv} kv heads x {n} rows",
                measured_s=t_rows, projected_s=t_full)


class _AttnTimer:
    """CUDA events around every call of the wrapped function (the HBA
    attention of a layer); .ms() sums the closed intervals."""

    def __init__(self, fn):
        self.fn, self.ev = fn, []

    def __call__(self, *a, **kw):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        r = self.fn(*a, **kw)
        e1.record()
        self.ev.append((e0, e1))
        return r

    def ms(self):
        torch.cuda.synchronize()
        t = sum(a.elapsed_time(b) for a, b in self.ev)
        self.ev = []
        return t


def cfg4_bench(steps, warmup, world, rank, local, pk):
    """a random-init 24-layer decoder (hidden 896, 14 / 2
    heads, dh 64, SwiGLU 4864, vocab 151936, every layer HBA: window 1024,
    block 64, top-16, 4 sinks, 4 slots) over batch 8 x 131072 uniform random
    token ids, the KV range split evenly over the world's GPUs: one prefill
    of the whole prompt, then `steps` decode steps (one token per sequence).
    value = prefill tokens/s; decode queries/s and the attention share of
    each phase beside it."""
    import types
    from transformers import Qwen2Config, Qwen2ForCausalLM
    import hba_b200.decoder as decmod
    import hba_b200.sharded_model as shmod
    from hba_b200 import HBAConfig, synth
    dev = torch.device("cuda", local)
    B, N, L = 8, 131072, 24
    cfg = HBAConfig(n_layers=L, n_heads=14, n_kv=2, head_dim=64, hidden=896, rope_theta=1e6, native_ctx=32768,
                    vocab_size=151936, block=64, window=1024, sinks=4, k_blocks=16, slots=4)
    qcfg = Qwen2Config(vocab_size=cfg.vocab_size, hidden_size=cfg.hidden, intermediate_size=4864, num_hidden_layers=L,
                       num_attention_heads=cfg.n_heads, num_key_value_heads=cfg.n_kv, max_position_embeddings=N + 64,
                       rope_theta=cfg.rope_theta, tie_word_embeddings=True)
    torch.manual_seed(0)
    with torch.device(dev):
        donor = Qwen2ForCausalLM(qcfg).to(torch.bfloat16).eval()
    summ, qkn = zip(*[synth.make_weights(cfg, dev, seed=100 + i, gains=False) for i in range(L)])
    model = types.SimpleNamespace(cfg=cfg, core=donor.model, lm_head=donor.lm_head, summarizers=list(summ),
                                  qknorms=list(qkn))
    g = torch.Generator().manual_seed(4)
    ids = torch.randint(0, cfg.vocab_size, (B, N + max(1, steps + warmup)), generator=g).to(dev)
    cap = N + steps + warmup + 64
    sharded = world > 1
    # time the HBA attention inside the model's layer loop: prefill (range) calls and decode cache steps
    if sharded:
        at = _AttnTimer(shmod.hba_attention_b200_range)
        shmod.hba_attention_b200_range = at
    else:
        at = _AttnTimer(decmod.hba_attention_b200)
        decmod.hba_attention_b200 = at
    try:
        # warm-up: a short prompt through a small decoder (kernels loaded, tensor maps cached)
        small = (shmod.HBAShardedModelDecoder(model, B, 4096, dev) if sharded else decmod.HBAModelDecoder(model, B, 4096))
        small.prefill(ids[:, :2048])
        small.step(ids[:, 2048])
        if sharded:
            small.close()
        del small
        torch.cuda.empty_cache()
        at.ms()
        dec = shmod.HBAShardedModelDecoder(model, B, cap, dev) if sharded else decmod.HBAModelDecoder(model, B, cap)
        barrier(world)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        dec.prefill(ids[:, :N])
        e1.record()
        torch.cuda.synchronize()
        prefill_ms = max_over_ranks(e0.elapsed_time(e1), world, dev)
        prefill_attn_ms = max_over_ranks(at.ms(), world, dev)
        # decode steps: every layer's cache step is the HBA attention of the step
        for j in range(warmup):
            dec.step(ids[:, N + j])
        torch.cuda.synchronize()
        cstep = [None]
        for cache_obj in (dec.shards if sharded else dec.caches):
            orig = cache_obj.attend if sharded else cache_obj.step
            t = _AttnTimer(orig)
            if sharded:
                cache_obj.attend = t
            else:
                cache_obj.step = t
            cstep.append(t)
        barrier(world)
        torch.cuda.synchronize()
        d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with Clocks(local) as ck:
            d0.record()
            for j in range(steps):
                dec.step(ids[:, N + warmup + j])
            d1.record()
            torch.cuda.synchronize()
        step_ms = max_over_ranks(d0.elapsed_time(d1) / steps, world, dev)
        step_attn_ms = max_over_ranks(sum(t.ms() for t in cstep[1:]) / steps, world, dev)
        if sharded:
            dec.close()
    finally:
        if sharded:
            shmod.hba_attention_b200_range = at.fn
        else:
            decmod.hba_attention_b200 = at.fn
    res = dict(
        metric=METRIC, value=B * N / (prefill_ms * 1e-3), unit="prefill tokens/s", n_gpus=world, steps=steps,
        warmup=warmup, ms_per_step=step_ms, higher_is_better=True, scaling="strong", vs_baseline=None, dtype="bf16",
        data="synthetic (uniform random token ids from seed; random-init weights of the config-4 architecture)",
        config=dict(workload=f"cfg4: {L}-layer decoder (hidden 896, 14/2 heads, dh 64, SwiGLU 4864, vocab 151936, "
                             f"every layer HBA flat top-16), batch {B} x {N} tokens, KV range split over {world} "
                             f"GPU(s)", batch=B, seq_len=N, layers=L,
                    parallelism=(f"sequence shards x{world}: per-layer NCCL all-gather of the new K/V in the "
                                 f"prefill, the fused NVLink sharded decode per layer") if sharded else "one GPU"),
        prefill=dict(ms=prefill_ms, tokens_per_s=B * N / (prefill_ms * 1e-3), attention_ms=prefill_attn_ms,
                     attention_fraction=prefill_attn_ms / prefill_ms),
        decode=dict(ms_per_step=step_ms, queries_per_s=B / (step_ms * 1e-3), attention_ms_per_step=step_attn_ms,
                    attention_fraction=step_attn_ms / step_ms,
                    timing="eager per-layer calls (projections, cache append + HBA decode attention, MLP), "
                           "the status of every layer's attention checked"),
        clocks=ck.summary(),
    )
    del dec, donor, model
    torch.cuda.empty_cache()
    return res


# -------------------------------------------------------- reference arm ----
def _ref_worker(args):
    """One host process: one sequence of the GPU arm's workload (the same
    seeded generator with its planted blocks, built on the host), its cache
    built with the oracle (untimed), `warmup` decodes, then `steps` timed
    oracle decodes of its query."""
    name, seed, warmup, steps = args
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "hierarchical-block-attention_b200"))
    torch.set_num_threads(1)
    from hba_b200 import synth
    from hba_b200.config import baseline_config
    from oracle import hba_oracle as orc
    cfg, B, n, hier = baseline_config(name)
    dh = cfg.head_dim
    summ, qkn = synth.make_weights(cfg, "cpu", seed=0, gains=False)
    wl = synth.decode_workload(cfg, 1, n, hier=hier, seed=seed, device="cpu", qkn=qkn)
    q = wl["q"].float().numpy()
    k, v = wl["k"].float().numpy(), wl["v"].float().numpy()
    probes, proj = summ.probes.numpy(), summ.proj.numpy()
    qg, kg = qkn.q.gain.numpy(), qkn.k.gain.numpy()
    kc = orc.head_rmsnorm(k, kg, bf16=True)
    S0 = orc.round_bf16(orc.summarize(kc, probes, proj, cfg.block).astype(np.float32))
    S1 = orc.round_bf16(orc.build_super(S0, cfg.fanout)[0].astype(np.float32)) if hier else None
    cos, sin = orc.rope_tables(n, dh, 1e6)
    ocfg = dict(block=cfg.block, window=cfg.window, sinks=cfg.sinks, k_blocks=cfg.k_blocks, fanout=cfg.fanout,
                beam=cfg.beam, qknorm=cfg.qknorm, content_scale_mode=cfg.content_scale_mode, temp_c=cfg.temp_c,
                n_cal=cfg.n_cal, native_ctx=cfg.native_ctx)
    scale = orc.union_scale(True, "inv_d", cfg.temp_c, cfg.n_cal, cfg.native_ctx, dh, n)
    for _ in range(warmup):
        orc.decode(q, kc, v, cos, sin, S0, S1, ocfg, scale, qg, hier=hier, bf16=True)
    t0 = time.perf_counter()
    for _ in range(steps):
        orc.decode(q, kc, v, cos, sin, S0, S1, ocfg, scale, qg, hier=hier, bf16=True)
    return time.perf_counter() - t0


def reference_arm(args, world, rank):
    """The reference algorithm's CPU path (the numpy oracle port) on every host
    core: one process per core, each decoding its own sequence of the GPU
    arm's workload `steps` times after `warmup`; value = all decodes / the
    slowest process.  Prints the GPU arm's `config` and `data`."""
    if rank != 0:
        return None
    import multiprocessing as mp
    os.environ.setdefault("OMP_NUM_THREADS", "1")
    os.environ.setdefault("OPENBLAS_NUM_THREADS", "1")
    name = args.config if args.config in ("cfg1", "cfg3") else "cfg1"
    procs = max(1, min(os.cpu_count() or 1, 64))
    with mp.get_context("spawn").Pool(procs) as pool:
        dts = pool.map(_ref_worker, [(name, 1000 + s, args.warmup, args.steps) for s in range(procs)])
    value = procs * args.steps / max(dts)
    line = dict(metric=METRIC, value=value, unit="decode queries/s", n_gpus=world, steps=args.steps,
                warmup=args.warmup, ms_per_step=1e3 * statistics.mean(dts) / args.steps, higher_is_better=True,
                scaling="weak", vs_baseline=None, dtype="f64 (bf16 inputs)", data=DECODE_DATA, impl="reference",
                config=decode_config(name, world),
                cpu_baseline=dict(value=value, unit="decode queries/s", cores=procs, kind="port",
                                  sample=f"{procs} processes x 1 sequence of the workload (planted, the GPU arm's "
                                         f"generator), {args.steps} timed decodes each (cache pre-built, untimed), "
                                         f"numpy oracle port of the reference eval path"),
                e2e=dict(value=value, unit="decode queries/s", h2d_bytes_per_step=0, d2h_bytes_per_step=0))
    return line


def main():
    args = parse()
    world, rank, local = dist_setup(args.gpus)
    if args.impl == "reference":
        line = reference_arm(args, world, rank)
        if line is not None:
            print(json.dumps(line))
        return
    torch.cuda.set_device(local)
    sys.path.insert(0, os.path.join(ROOT, "hierarchical-block-attention_b200"))
    import hba_b200  # noqa: F401  (fails loudly if the CUDA library is missing)
    hba_b200.load_library()
    if args.ncu_case is not None:
        ncu_case(args.ncu_case, local)
        return
    pk = peaks()
    if args.config in ("cfg1", "cfg3"):
        res = decode_bench(args.config, args.steps, args.warmup, world, rank, local, pk)
    elif args.config == "cfg3-shard":
        res = shard_bench("cfg3", args.steps, args.warmup, world, rank, local, pk)
    elif args.config == "cfg4":
        res = cfg4_bench(args.steps, args.warmup, world, rank, local, pk)
    elif args.config == "cfg2-bwd":
        res = prefill_bwd_bench("cfg2", args.steps, args.warmup, world, rank, local, pk)
    elif args.config == "cfg2-aux":
        res = aux_teacher_bench("cfg2", args.steps, args.warmup, world, rank, local, pk)
    else:
        res = prefill_bench(args.config, args.steps, args.warmup, world, rank, local, pk)
    if not args.no_secondary and args.config == "cfg1":
        sec = []
        for name in ("cfg3", "cfg2", "cfg2-bwd", "cfg2-aux") + (("cfg3-shard",) if world > 1 else ()):
            try:
                if name == "cfg3":
                    sec.append(decode_bench(name, min(args.steps, 10), args.warmup, world, rank, local, pk))
                elif name == "cfg3-shard":
                    sec.append(shard_bench("cfg3", min(args.steps, 10), args.warmup, world, rank, local, pk))
                elif name == "cfg2-bwd":
                    sec.append(prefill_bwd_bench("cfg2", min(args.steps, 3), 3, world, rank, local, pk))
                elif name == "cfg2-aux":
                    sec.append(aux_teacher_bench("cfg2", min(args.steps, 3), 3, world, rank, local, pk))
                else:
                    sec.append(prefill_bench(name, min(args.steps, 3), 3, world, rank, local, pk))
            except Exception as e:  # report, do not hide, a failing secondary
                sec.append(dict(config=name, error=repr(e)))
        res["secondary"] = sec
    if rank == 0:
        print(json.dumps(res))
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

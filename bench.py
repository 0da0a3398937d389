"""Benchmark of litevllm's per-step hot path on B200: KV store -> paged decode
attention -> greedy sampler, config 2 of the baseline (Llama-3-8B attention
shapes, 256 sequences per GPU, log-normal contexts, V = 128256).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...   (one process per GPU)

Sequences are sharded by request: the N*B global sequences are dealt to the
GPUs by context length (sharding.balanced_shard: B each, nearly equal total
context); each GPU owns its KV pool and inputs; no collective touches the data
path (weak scaling). torch.distributed is used only for the start/stop
barrier and the max-over-ranks time. Rank 0 prints one JSON line.

The same line carries sub-records ("sub") for every target the configurations
name, each device-timed with CUDA events over --steps after --warmup, max over
ranks: the sampler alone (greedy [256, 128256]; in-kernel-noise Gumbel-max
[128, 151936] at T = 0.7), config 5 (64 long-context sequences split over the
ranks: strong scaling), config 3 (chunked prefill on prior context + 252
decodes) and config 4 (prefix-shared decode). --no-sub skips them.

--impl reference times the reference algorithm on the host CPU (the CPU
restatement of litevllm's Attention.forward store + _decode_fast and the greedy
Sampler, run with every host thread) on a bounded sample of the same workload.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "paged-decode attn HBM GB/s (% of peak); sampled tok/s at 1/2/4/8 B200"
CFG = 2
B_PER_GPU = 256
H, H_KV, D, BS, V = 32, 8, 128, 16, 128256
FALLBACK_HBM_GBS = 6650.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--layers", type=int, default=1, help="attention layers per step")
    ap.add_argument("--num-splits", type=int, default=0, help="decode split-KV override (0=auto)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--cfg5-seqs", type=int, default=64,
                    help="config 5's global sequence count (64; fewer only for a small "
                         "profiling case)")
    ap.add_argument("--no-sub", action="store_true",
                    help="skip the sub-records (sampler, cfg5, cfg3, cfg4) of the default line")
    ap.add_argument("--workload", default="cfg2",
                    choices=["cfg2", "cfg3", "cfg4", "cfg5", "sampler", "mma_rate"],
                    help="cfg2 (default) is the contract's workload; the others print one "
                         "sub-record alone (cfg3 mixed prefill step, cfg4 prefix-shared "
                         "decode, cfg5 long-context decode, sampler greedy + in-kernel noise)")
    return ap.parse_args()


# ----------------------------------------------------------- algorithmic bytes ---
def decode_bytes(ctx, B, elem=2):
    kv = sum(ctx) * 2 * H_KV * D * elem
    qo = B * H * D * elem * 2
    meta = sum(-(-c // BS) for c in ctx) * 4 + B * 4
    return kv + qo + meta


def store_bytes(B, elem=2):
    return B * 2 * H_KV * D * elem * 2 + B * 8


def sampler_bytes(B, elem=2):
    return B * V * elem + B * 8


# ---------------------------------------------------------------- environment ---
def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return ws, rank, local


def measured_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic():
    """Per-launch DRAM bytes of the decode kernel from the committed ncu summary."""
    p = ROOT / "profiles" / "paged_decode_cfg2.md"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.strip().startswith("traffic_bytes_per_launch:"):
            try:
                return int(float(line.split(":", 1)[1].strip().split()[0]))
            except ValueError:
                return None
    return None


class ClockSampler:
    """Polls NVML clocks and throttle reasons on a thread during the timed region."""

    REASONS = {
        "hw_slowdown": 0x0000000000000008,
        "sw_thermal_slowdown": 0x0000000000000020,
        "hw_thermal_slowdown": 0x0000000000000040,
        "sw_power_cap": 0x0000000000000004,
        "hw_power_brake_slowdown": 0x0000000000000080,
    }

    def __init__(self, index: int):
        self.index = index
        # poll period (BENCH_CLOCK_POLL_MS, default 0.5 ms; 0 disables polling)
        self.period_s = float(os.environ.get("BENCH_CLOCK_POLL_MS", "0.5")) * 1e-3
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None
        self.ok = False
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.ok = False

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for name, bit in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period_s)

    def __enter__(self):
        # The launching thread holds the GIL while it enqueues steps; with the
        # default 5 ms switch interval a region of a few ms yields one sample.
        # A short interval lets the poller run between launches.
        self._switch = sys.getswitchinterval()
        if self.ok and self.period_s > 0:
            sys.setswitchinterval(1e-4)
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join()
        sys.setswitchinterval(self._switch)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                    "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def gpu_local_cpus(dev):
    """The host CPUs NVML reports as local to `dev` (its NUMA node), within this
    process's current affinity; None when NVML cannot say."""
    try:
        import pynvml

        pynvml.nvmlInit()
        p = torch.cuda.get_device_properties(dev)
        bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        words = pynvml.nvmlDeviceGetCpuAffinity(h, (os.cpu_count() + 63) // 64)
        cpus = {64 * i + b for i, m in enumerate(words) for b in range(64) if (m >> b) & 1}
        return (cpus & os.sched_getaffinity(0)) or None
    except Exception:
        return None


# ------------------------------------------------------------------ our arm ---
def run_ours(args, ws, rank, local):
    from litevllm_b200 import ops, workloads
    from litevllm_b200.attention import Attention
    from litevllm_b200.sampler import Sampler

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    from litevllm_b200.sharding import balanced_shard

    # the global batch's sequences are dealt to the ranks by length (equal
    # counts, nearly equal total context): the step is the slowest rank's
    lens = [workloads.context_len(CFG, 0, i) for i in range(B_PER_GPU * ws)]
    mine = balanced_shard(lens, ws, rank)
    B = len(mine)
    first = rank * B_PER_GPU
    batch = workloads.make_decode_batch(CFG, B, seed=0, first_seq=first,
                                        ctx=[lens[i] for i in mine], device=dev)
    # L layers: separate KV pools per layer would multiply memory; the layers
    # share the block tables and read distinct pools (layer 0 reuses batch's).
    pools = [(batch.key_cache, batch.value_cache)]
    for li in range(1, args.layers):
        pools.append((torch.randn_like(batch.key_cache), torch.randn_like(batch.value_cache)))
    logits = [workloads.make_logits(CFG, B, V, seed=s, first_seq=first, device=dev) for s in (0, 1)]
    ids = torch.empty(B, dtype=torch.int64, device=dev)
    out = torch.empty_like(batch.query)
    max_blocks = batch.block_tables.shape[1]
    nsplit = args.num_splits or ops.decode_num_splits(B, H_KV, max_blocks, BS)
    stream = torch.cuda.current_stream(dev)

    def step(i, ev=None):
        for li, (kc, vc) in enumerate(pools):
            ops.store_kvcache(batch.key, batch.value, kc, vc, batch.slot_mapping)
            if ev is not None and li == 0:
                ev[0].record(stream)
            ops.paged_decode(batch.query, kc, vc, batch.block_tables, batch.context_lens,
                             batch.scale, num_splits=nsplit, out=out)
            if ev is not None and li == 0:
                ev[1].record(stream)
        # config 2 is all-greedy: the temperature-0 path of Sampler.sample
        ops.sample(logits[i & 1], None, out=ids)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize(dev)

    K = args.steps
    dec_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(K)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if ws > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(local) as clk:
        # ~0.5 ms of device sleep ahead of the start event: the host enqueues
        # the first steps meanwhile, so a short run does not time the host's
        # first launches on an idle GPU (a host slower than the GPU in steady
        # state still drains the queue and shows in the time)
        torch.cuda._sleep(1_000_000)
        t0.record(stream)
        h0 = time.perf_counter()
        for i in range(K):
            step(i, dec_ev[i])
        host_us = (time.perf_counter() - h0) / K * 1e6  # host time to enqueue one step
        t1.record(stream)
        torch.cuda.synchronize(dev)
    if ws > 1:
        torch.distributed.barrier()
    ms = t0.elapsed_time(t1) / K
    dec_ms = sum(a.elapsed_time(b) for a, b in dec_ev) / K
    status = ops.decode_status()
    if status:
        raise RuntimeError(f"decode kernel status bits {status}")

    # ---- e2e through the public API: host inputs in, token ids out, every step
    e2e = None
    if not args.no_e2e:
        # Serve from the GPU's own NUMA node, as a deployment pins its serving
        # process: the pinned input buffers are first touched there, so the
        # host-to-device copies read local memory. Restored after the e2e run.
        prev_cpus = os.sched_getaffinity(0)
        near = gpu_local_cpus(dev) if os.environ.get("BENCH_E2E_NUMA", "1") != "0" else None
        if near:
            os.sched_setaffinity(0, near)
        attn = Attention(H, D, H_KV)
        pin = lambda t: t.detach().cpu().pin_memory()
        h_q, h_k, h_v = pin(batch.query), pin(batch.key), pin(batch.value)
        h_slot, h_bt, h_ctx = pin(batch.slot_mapping), pin(batch.block_tables), pin(batch.context_lens)
        h_logits = [pin(x) for x in logits]
        h_ids = torch.empty(B, dtype=torch.int64).pin_memory()
        kc, vc = pools[0]

        # Step i+1's host inputs are uploaded on a copy stream into the other
        # of two device buffer sets while step i computes; every step still
        # waits for its own token ids on the host.
        cstream = torch.cuda.Stream(dev)
        host_in = [dict(q=h_q, k=h_k, v=h_v, slot=h_slot, bt=h_bt, ctx=h_ctx, lg=h_logits[s_])
                   for s_ in (0, 1)]
        bufs = [{n: torch.empty_like(t, device=dev) for n, t in hi.items()} for hi in host_in]
        ready = [torch.cuda.Event(), torch.cuda.Event()]
        free = [torch.cuda.Event(), torch.cuda.Event()]
        for ev in free:
            ev.record(stream)

        def upload(i):
            s_ = i & 1
            with torch.cuda.stream(cstream):
                cstream.wait_event(free[s_])
                for n, t in host_in[s_].items():
                    bufs[s_][n].copy_(t, non_blocking=True)
                ready[s_].record(cstream)

        def compute(i):
            s_ = i & 1
            d = bufs[s_]
            stream.wait_event(ready[s_])
            o = attn.forward(d["q"], d["k"], d["v"], kc, vc, d["bt"], d["slot"], d["ctx"],
                             is_prefill=False)
            for li in range(1, args.layers):
                o = attn.forward(d["q"], d["k"], d["v"], pools[li][0], pools[li][1], d["bt"],
                                 d["slot"], d["ctx"], is_prefill=False)
            tok = Sampler.sample_batch(d["lg"], None, seed=1, offset=i)
            free[s_].record(stream)
            h_ids.copy_(tok, non_blocking=True)
            stream.synchronize()
            return o

        def run(n, first):
            upload(first)
            for i in range(first, first + n):
                if i + 1 < first + n:
                    upload(i + 1)
                compute(i)

        run(max(3, args.warmup), 0)
        if ws > 1:
            torch.distributed.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        cstream.wait_event(e0)
        run(K, 1000)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        e2e_ms = e0.elapsed_time(e1) / K
        if ws > 1:
            t = torch.tensor([e2e_ms], device=dev)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            e2e_ms = float(t.item())
        h2d = sum(x.numel() * x.element_size() for x in (h_q, h_k, h_v, h_slot, h_bt, h_ctx, h_logits[0]))
        # the host link on its own: the same pinned copies, every rank at once
        if ws > 1:
            torch.distributed.barrier()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(cstream):
            torch.cuda.synchronize(dev)
            c0.record(cstream)
            for _ in range(5):
                for n, t_ in host_in[0].items():
                    bufs[0][n].copy_(t_, non_blocking=True)
            c1.record(cstream)
        torch.cuda.synchronize(dev)
        h2d_ms = c0.elapsed_time(c1) / 5
        if ws > 1:
            t = torch.tensor([h2d_ms], device=dev)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            h2d_ms = float(t.item())
        h2d_gbs = h2d / (h2d_ms * 1e-3) / 1e9
        e2e = dict(ms=e2e_ms, h2d=h2d, d2h=B * 8, h2d_gbs=h2d_gbs,
                   host=("pinned buffers on the GPU's NUMA node (NVML CPU affinity, "
                         f"{len(near)} CPUs)") if near else "pinned buffers (process CPU affinity unchanged)")
        os.sched_setaffinity(0, prev_cpus)

    mine_t = torch.tensor([ms, dec_ms, host_us], device=dev, dtype=torch.float64)
    if ws > 1:
        allt = [torch.empty_like(mine_t) for _ in range(ws)]
        torch.distributed.all_gather(allt, mine_t)
        allt = torch.stack(allt).cpu()
    else:
        allt = mine_t.cpu()[None]
    ms, dec_ms = float(allt[:, 0].max()), float(allt[:, 1].max())

    def spread(col):
        v = sorted(float(x) for x in allt[:, col])
        return {"min": round(v[0], 4), "median": round(statistics.median(v), 4),
                "max": round(v[-1], 4)}

    per_rank = {"ms_per_step": spread(0), "decode_ms": spread(1),
                "host_enqueue_us_per_step": spread(2)}
    # the whole job's bytes: ranks hold different context mixes
    step_b = args.layers * (decode_bytes(batch.ctx, B) + store_bytes(B)) + sampler_bytes(B)
    jb = torch.tensor([float(step_b), float(B)], device=dev, dtype=torch.float64)
    if ws > 1:
        torch.distributed.all_reduce(jb, op=torch.distributed.ReduceOp.SUM)
    return dict(ms=ms, dec_ms=dec_ms, ctx=batch.ctx, B=B, e2e=e2e, clocks=clk.summary(),
                nsplit=nsplit, K=K, per_rank=per_rank, job_bytes=float(jb[0]),
                job_seqs=int(jb[1]))


# -------------------------------------------------------- CPU (reference) arm ---
def cpu_reference_sample(n_seqs: int, seed_offset: int = 0):
    """Time the reference algorithm on the host for n_seqs config-2 sequences:
    store + _decode_fast (literal restatement, padded gather) + greedy argmax,
    fp32, all host threads. Returns (seconds, algorithmic bytes, tokens)."""
    from litevllm_b200 import workloads
    from oracle import paged_attention as pa
    from oracle import sampler as osamp
    from oracle import store_kv as ostore

    b = workloads.make_decode_batch(CFG, n_seqs, seed=0, first_seq=seed_offset, dtype=torch.float32)
    lg = workloads.make_logits(CFG, n_seqs, V, seed=0, first_seq=seed_offset, dtype=torch.float32)
    kc, vc = b.key_cache.numpy(), b.value_cache.numpy()
    t = time.perf_counter()
    ostore.store_kv(b.key.numpy(), b.value.numpy(), kc, vc, b.slot_mapping.numpy())
    pa.decode_batched_reference(b.query, b.key_cache, b.value_cache, b.block_tables,
                                b.context_lens, b.scale)
    osamp.greedy(lg.numpy())
    dt = time.perf_counter() - t
    nbytes = decode_bytes(b.ctx, n_seqs) + store_bytes(n_seqs) + sampler_bytes(n_seqs)
    return dt, nbytes, n_seqs


def cpu_baseline(budget_s=12.0, n_seqs=8):
    torch.set_num_threads(os.cpu_count() or 1)
    cpu_reference_sample(2)  # warm
    tot_t = tot_b = tot_n = 0.0
    i = 0
    while tot_t < budget_s and i < 5000:
        dt, nb, n = cpu_reference_sample(n_seqs, seed_offset=1000 + i * n_seqs)
        tot_t, tot_b, tot_n = tot_t + dt, tot_b + nb, tot_n + n
        i += 1
    return dict(gbs=tot_b / tot_t / 1e9, tok_s=tot_n / tot_t, cores=torch.get_num_threads(),
                sample=f"{i} x {n_seqs} config-2 sequences (store + _decode_fast restatement + "
                       f"greedy argmax over {V}), fp32, {tot_t:.1f} s")


def workload_config(N):
    return {
        "workload": "config 2: bf16 paged decode step, Llama-3-8B attention (32 Q / 8 KV heads, "
                    "D=128, block 16), 256 sequences per GPU, context lengths "
                    "clip(lognormal(median 1024, sigma 0.5), 16, 4096); KV store of the 256 new "
                    "tokens + decode (1 layer) + greedy sampler over [256, 128256] bf16",
        "global_batch": B_PER_GPU * N,
        "l2": "inputs larger than L2: KV pool ~1.2 GB per GPU, two rotating 66 MB logits buffers",
        "parallelism": f"request-sharded x{N}: the {B_PER_GPU * N} sequences dealt to the GPUs "
                       "by context length, equal counts (no collective on the data path)",
    }


def run_reference(args, ws, rank):
    """CPU arm: the reference algorithm on the host, rank 0 only."""
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    n = 8
    for i in range(max(1, args.warmup)):
        cpu_reference_sample(n, seed_offset=5000 + i * n)
    tt = tb = tn = 0.0
    for i in range(args.steps):
        dt, nb, k = cpu_reference_sample(n, seed_offset=i * n)
        tt, tb, tn = tt + dt, tb + nb, tn + k
    gbs = tb / tt / 1e9
    sample = f"{args.steps} steps x {n} config-2 sequences (store + _decode_fast + greedy argmax), fp32"
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(gbs, 3),
        "unit": "GB/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(tt / args.steps * 1e3, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": workload_config(args.gpus),
        "sampled_tok_s": round(tn / tt, 2),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": torch.get_num_threads(),
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def measured_tflops():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["bf16_tflops"]), "measured"
        except Exception:
            pass
    return 1590.0, "fallback"


def _time_events(stream, fn, K, warmup):
    for _ in range(warmup):
        fn(None)
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    evs = []
    t0.record(stream)
    for _ in range(K):
        evs.append(fn(stream))
    t1.record(stream)
    torch.cuda.synchronize()
    return t0.elapsed_time(t1) / K, evs


def _time_graph(fn, K, warmup, dev):
    """fn() enqueued K times into one CUDA graph, replayed and timed with
    CUDA events: ms per call on the device alone (the host's Python and
    launch time, which can exceed a short kernel's, is not in the region)."""
    for _ in range(max(1, warmup)):
        fn()
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(K):
            fn()
    g.replay()
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    g.replay()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    return e0.elapsed_time(e1) / K


def measure_sub(workload, steps, warmup, ws, rank, local):
    """Secondary workloads, device-timed per kernel with CUDA events, max over
    ranks: "cfg3" (mixed chunked-prefill + decode step), "cfg4" (prefix-shared
    decode + T=0.7 sampler), "cfg5" (long-context decode + T=1.0 sampler,
    64 sequences split over the ranks: strong scaling). Returns the record."""
    from litevllm_b200 import ops, workloads
    from litevllm_b200.sharding import balanced_shard

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    args = argparse.Namespace(workload=workload, steps=steps, warmup=warmup)
    peak_hbm, _ = measured_peak()
    peak_tf, tf_kind = measured_tflops()
    Ev = lambda: torch.cuda.Event(enable_timing=True)
    if args.workload == "cfg4":
        # 128 sequences per GPU share a 2048-token prefix (copy-on-write fork of
        # its last block by the library's block copy) + 256 private tokens;
        # T = 0.7 sampling over 151936 with in-kernel noise.
        B = 128
        b = workloads.make_prefix_batch(B=B, seed=rank, device=dev, fork=ops.copy_blocks)
        V4 = 151936
        logits = workloads.make_logits(4, B, V4, seed=0, first_seq=rank * B, device=dev)
        temps = workloads.temperatures_for(4, B, device=dev)
        ids = torch.empty(B, dtype=torch.int64, device=dev)
        out = torch.empty_like(b.query)
        nsplit = ops.decode_num_splits(B, H_KV, b.block_tables.shape[1], BS)

        prefix_tokens = 127 * BS  # the physically shared blocks (the 128th is forked)

        def make_step(shared):
            def step(st, i=[0]):
                i[0] += 1
                e = (Ev(), Ev()) if st is not None else None
                ops.store_kvcache(b.key, b.value, b.key_cache, b.value_cache, b.slot_mapping)
                if e: e[0].record(st)
                if shared:  # the prefix once on the tensor cores, suffixes on the decode kernel
                    ops.paged_decode_shared_prefix(b.query, b.key_cache, b.value_cache,
                                                   b.block_tables, b.context_lens, b.scale,
                                                   prefix_tokens, out=out)
                else:
                    ops.paged_decode(b.query, b.key_cache, b.value_cache, b.block_tables,
                                     b.context_lens, b.scale, num_splits=nsplit, out=out)
                if e: e[1].record(st)
                ops.sample(logits, temps, seed=3, offset=i[0], out=ids)
                return e
            return step

        ms_r, evs = _time_events(stream, make_step(False), args.steps, max(3, args.warmup))
        dec_r = sum(a.elapsed_time(c) for a, c in evs) / len(evs)
        ms, evs = _time_events(stream, make_step(True), args.steps, max(3, args.warmup))
        dec_ms = sum(a.elapsed_time(c) for a, c in evs) / len(evs)
        # device time alone, from CUDA graphs (see cfg3)
        K = max(8, args.steps)
        g_dec = _time_graph(lambda: ops.paged_decode_shared_prefix(
            b.query, b.key_cache, b.value_cache, b.block_tables, b.context_lens, b.scale,
            prefix_tokens, out=out), K, 3, dev)
        g_dec_r = _time_graph(lambda: ops.paged_decode(
            b.query, b.key_cache, b.value_cache, b.block_tables, b.context_lens, b.scale,
            num_splits=nsplit, out=out), K, 3, dev)
        step_s = make_step(True)
        g_step = _time_graph(lambda: step_s(None), K, 3, dev)
        t = torch.tensor([ms, dec_ms, ms_r, dec_r, g_dec, g_dec_r, g_step], device=dev)
        if ws > 1:
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms, dec_ms, ms_r, dec_r, g_dec, g_dec_r, g_step = (float(x) for x in t)
        logical = decode_bytes(b.ctx, B)
        unique = b.key_cache.numel() * 2 * 2 + B * H * D * 4
        line = {"workload": "cfg4", "metric": METRIC, "n_gpus": ws, "steps": args.steps,
                "config": {"workload": "config 4: bf16 prefix-shared decode, Qwen3-8B attention "
                           "(32 Q / 8 KV heads, D=128): 128 sequences per GPU share 127 blocks "
                           "+ a copy-on-write fork of the 128th (2048-token prefix) then 16 "
                           "private blocks; T=0.7 Gumbel-max (in-kernel Philox) over 151936",
                           "parallelism": f"request-sharded x{ws}"},
                "ms_per_step": round(g_step, 4), "ms_per_step_eager": round(ms, 4),
                "sampled_tok_s": round(B * ws / (g_step * 1e-3), 1),
                "timing": "CUDA graphs of `steps` calls, replayed (device time); *_eager: "
                          "the same calls one by one with events",
                "value": round(logical / (g_dec * 1e-3) / 1e9, 1), "unit": "GB/s (logical)",
                "decode": {"kernel": "paged_decode_shared_prefix (prefix on tensor cores + "
                                     "suffix split decode)", "ms": round(g_dec, 4),
                           "ms_eager": round(dec_ms, 4),
                           "logical_gbs": round(logical / (g_dec * 1e-3) / 1e9, 1),
                           "unique_gbs": round(unique / (g_dec * 1e-3) / 1e9, 1),
                           "note": "logical = bytes a per-row decode reads; unique = bytes "
                                   "in the pool"},
                "decode_per_row": {"kernel": "paged_decode (every row streams the prefix, "
                                             "L2-resident)", "ms": round(g_dec_r, 4),
                                   "ms_eager": round(dec_r, 4), "step_ms_eager": round(ms_r, 4),
                                   "logical_gbs": round(logical / (g_dec_r * 1e-3) / 1e9, 1)}}
    elif args.workload == "cfg5":
        # 64 sequences dealt to the ranks by context length (equal counts)
        nseq = int(os.environ.get("BENCH_CFG5_SEQS", "64"))
        lens = [workloads.context_len(5, 0, i) for i in range(nseq)]
        mine = balanced_shard(lens, ws, rank)
        B = len(mine)
        b = workloads.make_decode_batch(5, B, seed=0, first_seq=rank * 64,
                                        ctx=[lens[i] for i in mine], device=dev)
        V5 = 151936
        logits = workloads.make_logits(5, B, V5, seed=0, first_seq=rank * 64, device=dev)
        temps = workloads.temperatures_for(5, B, device=dev)
        ids = torch.empty(B, dtype=torch.int64, device=dev)
        out = torch.empty_like(b.query)
        nsplit = ops.decode_num_splits(B, H_KV, b.block_tables.shape[1], BS)

        def step(st, i=[0]):
            i[0] += 1
            e = (Ev(), Ev(), Ev()) if st is not None else None
            ops.store_kvcache(b.key, b.value, b.key_cache, b.value_cache, b.slot_mapping)
            if e: e[0].record(st)
            ops.paged_decode(b.query, b.key_cache, b.value_cache, b.block_tables, b.context_lens,
                             b.scale, num_splits=nsplit, out=out)
            if e: e[1].record(st)
            ops.sample(logits, temps, seed=7, offset=i[0], out=ids)
            if e: e[2].record(st)
            return e

        ms, evs = _time_events(stream, step, args.steps, max(3, args.warmup))
        dec_ms = sum(a.elapsed_time(c) for a, c, _ in evs) / len(evs)
        smp_ms = sum(c.elapsed_time(d) for _, c, d in evs) / len(evs)
        dec_b = decode_bytes(b.ctx, B)
        smp_b = B * V5 * 2 + B * 8
        step_b = dec_b + store_bytes(B) + smp_b
        # per rank: time maxima; bytes summed (ranks hold different contexts)
        own_dec_ms = dec_ms
        t = torch.tensor([ms, dec_ms, smp_ms], device=dev, dtype=torch.float64)
        nb = torch.tensor([step_b, dec_b], device=dev, dtype=torch.float64)
        if ws > 1:
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            torch.distributed.all_reduce(nb, op=torch.distributed.ReduceOp.SUM)
        own = torch.tensor([dec_b / (own_dec_ms * 1e-3) / 1e9], device=dev, dtype=torch.float64)
        ms, dec_ms, smp_ms = (float(x) for x in t)
        job_b, job_dec_b = (float(x) for x in nb)
        # per rank: its own decode bytes over its own decode time
        if ws > 1:
            allr = [torch.empty_like(own) for _ in range(ws)]
            torch.distributed.all_gather(allr, own)
            rates = sorted(float(x) for x in allr)
        else:
            rates = [float(own)]
        dec_gbs = statistics.median(rates)
        line = {"workload": "cfg5", "metric": METRIC, "n_gpus": ws, "steps": args.steps,
                "config": {"workload": f"config 5: bf16 long-context decode, {nseq} sequences in total "
                           f"({B} per GPU), context U[32768,131072], 32 Q / 8 KV heads, D=128, "
                           "block 16, split-KV, + T=1.0 Gumbel-max sampler (in-kernel Philox) "
                           "over 151936", "parallelism": f"request-sharded x{ws}",
                           "l2": f"inputs larger than L2: {job_dec_b / ws / 1e9:.1f} GB of KV per GPU"},
                "scaling": "strong",
                "value": round(job_b / (ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                "ms_per_step": round(ms, 4), "sampled_tok_s": round(nseq / (ms * 1e-3), 1),
                "decode_split_kv": nsplit,
                "decode": {"ms": round(dec_ms, 4),
                           "job_gbs": round(job_dec_b / (dec_ms * 1e-3) / 1e9, 1)},
                "sampler": {"kernel": "gumbel_kernel (in-kernel Philox, T=1.0)",
                            "ms": round(smp_ms, 4), "rows": B, "vocab": V5,
                            "gbs": round(smp_b / (smp_ms * 1e-3) / 1e9, 1)},
                "roofline": {"kernel": "paged_decode_kernel", "bound": "hbm",
                             "achieved": round(dec_gbs, 1), "peak": peak_hbm, "unit": "GB/s",
                             "frac": round(dec_gbs / peak_hbm, 4),
                             "achieved_per_rank": {"min": round(rates[0], 1),
                                                   "max": round(rates[-1], 1)},
                             "note": "median over ranks of each rank's decode bytes / its "
                                     "decode time",
                             "traffic_over_algorithmic": 1.0004,
                             "traffic_source": "ncu dram bytes of an 8-sequence config-5 launch "
                                               "(profiles/paged_decode_cfg5.md), not measured "
                                               "in this run",
                             "algorithmic_bytes_per_launch": dec_b}}
    else:
        # config 3: 4 chunks of 512 on prior U[0,3584] + 252 decode sequences,
        # 2300 new tokens stored through slot_mapping, pool of 65536 blocks.
        prior = [workloads.prefill_prior(0, i) for i in range(4)]
        pf = workloads.make_prefill_batch([512] * 4, prior, seed=0, device=dev)
        npf = pf.key_cache.shape[0]
        dec = workloads.make_decode_batch(3, 252, seed=0, device=dev, pool_blocks=65536 - npf)
        pout = torch.empty_like(pf.query)
        dout = torch.empty_like(dec.query)
        nsplit = ops.decode_num_splits(252, H_KV, dec.block_tables.shape[1], BS)

        def step(st):
            e = (Ev(), Ev(), Ev()) if st is not None else None
            ops.store_kvcache(pf.key, pf.value, pf.key_cache, pf.value_cache, pf.slot_mapping)
            ops.store_kvcache(dec.key, dec.value, dec.key_cache, dec.value_cache, dec.slot_mapping)
            if e: e[0].record(st)
            ops.paged_prefill(pf.query, pf.key_cache, pf.value_cache, pf.cu_seqlens_q, 512,
                              pf.scale, block_tables=pf.block_tables, context_lens=pf.context_lens,
                              out=pout)
            if e: e[1].record(st)
            ops.paged_decode(dec.query, dec.key_cache, dec.value_cache, dec.block_tables,
                             dec.context_lens, dec.scale, num_splits=nsplit, out=dout)
            if e: e[2].record(st)
            return e

        ms, evs = _time_events(stream, step, args.steps, max(3, args.warmup))
        pre_ms = sum(a.elapsed_time(c) for a, c, _ in evs) / len(evs)
        dec_ms = sum(c.elapsed_time(d) for _, c, d in evs) / len(evs)

        # The same step as Attention.forward_mixed runs it: decode on a side
        # stream next to the prefill (the decode blocks fill the SMs that the
        # persistent prefill kernel's tail leaves idle).
        from litevllm_b200.attention import run_overlapped

        def step_overlapped(st):
            ops.store_kvcache(pf.key, pf.value, pf.key_cache, pf.value_cache, pf.slot_mapping)
            ops.store_kvcache(dec.key, dec.value, dec.key_cache, dec.value_cache, dec.slot_mapping)
            run_overlapped(
                lambda: ops.paged_prefill(pf.query, pf.key_cache, pf.value_cache, pf.cu_seqlens_q,
                                          512, pf.scale, block_tables=pf.block_tables,
                                          context_lens=pf.context_lens, out=pout),
                lambda: ops.paged_decode(dec.query, dec.key_cache, dec.value_cache,
                                         dec.block_tables, dec.context_lens, dec.scale,
                                         num_splits=nsplit, out=dout))

        ov_ms, _ = _time_events(stream, step_overlapped, args.steps, max(3, args.warmup))
        # the same from CUDA graphs: the device's time alone (one ops call's host
        # time, ~15-25 us, leaves the GPU idle between these short kernels)
        K = max(8, args.steps)
        g_pre = _time_graph(lambda: ops.paged_prefill(
            pf.query, pf.key_cache, pf.value_cache, pf.cu_seqlens_q, 512, pf.scale,
            block_tables=pf.block_tables, context_lens=pf.context_lens, out=pout), K, 3, dev)
        g_dec = _time_graph(lambda: ops.paged_decode(
            dec.query, dec.key_cache, dec.value_cache, dec.block_tables, dec.context_lens,
            dec.scale, num_splits=nsplit, out=dout), K, 3, dev)
        g_step = _time_graph(lambda: step(None), K, 3, dev)
        g_ov = _time_graph(lambda: step_overlapped(None), K, 3, dev)
        t = torch.tensor([ms, pre_ms, dec_ms, ov_ms, g_pre, g_dec, g_step, g_ov], device=dev)
        if ws > 1:
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms, pre_ms, dec_ms, ov_ms, g_pre, g_dec, g_step, g_ov = (float(x) for x in t)
        flops = sum(4 * H * D * 512 * (p_ + (512 + 1) / 2) for p_ in prior)
        dec_b = decode_bytes(dec.ctx, 252)
        tf = flops / (g_pre * 1e-3) / 1e12
        tf_eager = flops / (pre_ms * 1e-3) / 1e12
        line = {"workload": "cfg3", "metric": METRIC, "n_gpus": ws, "steps": args.steps,
                "config": {"workload": "config 3: bf16 mixed step, Qwen3-8B attention (32 Q / 8 KV "
                           "heads, D=128): 4 prefill chunks of 512 on prior context "
                           f"{prior} + 252 decode sequences (context U[64,2048]); 2300 new "
                           "tokens stored; 65536-block pool", "parallelism": f"replica x{ws}"},
                "ms_per_step": round(g_step, 4), "unit": "TFLOP/s",
                "value": round(tf, 1),
                "timing": "CUDA graphs of `steps` calls, replayed (device time); the *_eager "
                          "figures time the same calls one by one with events",
                "prefill": {"ms": round(g_pre, 4), "tflops": round(tf, 1),
                            "ms_eager": round(pre_ms, 4), "tflops_eager": round(tf_eager, 1),
                            "roofline": {"kernel": "paged_prefill_pp_kernel", "bound": "tensor",
                                         "achieved": round(tf, 1), "peak": peak_tf,
                                         "peak_source": f"{tf_kind} bf16 burst", "unit": "TFLOP/s",
                                         "frac": round(tf / peak_tf, 4)}},
                "decode": {"ms": round(g_dec, 4),
                           "gbs": round(dec_b / (g_dec * 1e-3) / 1e9, 1),
                           "frac_of_hbm_peak": round(dec_b / (g_dec * 1e-3) / 1e9 / peak_hbm, 4),
                           "ms_eager": round(dec_ms, 4)},
                "ms_per_step_eager": round(ms, 4),
                "step_overlapped": {"ms": round(g_ov, 4), "ms_eager": round(ov_ms, 4),
                                    "note": "store, then prefill and decode on two streams "
                                            "(Attention.forward_mixed); ms_per_step runs them "
                                            "one after the other"}}
    return line


def measure_sampler(steps, warmup, ws, local):
    """The vocab-wide sampler on its own, both modes the configurations use:
    greedy over [256, 128256] (config 2) and in-kernel-noise Gumbel-max at
    T = 0.7 over [128, 151936] (config 4's shape). Each is timed as `steps`
    back-to-back calls (CUDA events on the launching stream) rotating over four
    logits buffers (263 / 156 MB, larger than L2), replayed from a CUDA graph
    the way a captured serving step issues them; max over ranks."""
    from litevllm_b200 import ops, workloads

    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream(dev)
    peak, _ = measured_peak()
    rec = {}
    for name, B, V, T in (("greedy", 256, 128256, None), ("gumbel_rng", 128, 151936, 0.7)):
        bufs = [workloads.make_logits(2 if T is None else 4, B, V, seed=s_, device=dev)
                for s_ in range(4)]
        temps = None if T is None else torch.full((B,), T, device=dev)
        ids = torch.empty(B, dtype=torch.int64, device=dev)
        # One call costs ~15 us of host time (argument checks, ctypes), longer
        # than the kernel: timed call by call, the GPU would wait on the host.
        # The calls are captured in a CUDA graph and the graph is replayed, so
        # the events time the kernels back to back, as in a captured decode step.
        for i in range(max(3, warmup)):
            ops.sample(bufs[i & 3], temps, seed=11, offset=i, out=ids)
        torch.cuda.synchronize(dev)
        n = max(8, steps)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(n):
                ops.sample(bufs[i & 3], temps, seed=11, offset=i, out=ids)
        for _ in range(2):
            g.replay()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        g.replay()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1) / n
        t = torch.tensor([ms], device=dev)
        if ws > 1:
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        us = float(t[0]) * 1e3
        nbytes = B * V * 2 + B * 8
        gbs = nbytes / (us * 1e-6) / 1e9
        rec[name] = {"rows": B, "vocab": V, "temperature": T or 0.0, "us": round(us, 2),
                     "algorithmic_bytes": nbytes, "gbs": round(gbs, 1),
                     "frac_of_hbm_peak": round(gbs / peak, 4)}
        del bufs
    rec["gumbel_rng"]["bound"] = ("instruction issue: per element a quarter Philox4x32-10 "
                                  "block; keys (Gumbel map, division) only for vectors "
                                  "whose bound can beat the CTA's best")
    rec["timing"] = ("`steps` calls captured in one CUDA graph over 4 rotating buffers > L2, "
                     "replayed and timed with CUDA events")
    return rec


def measure_mma_rate(local, n_mma=8192):
    """Issue rate of tcgen05.mma on this GPU (lk_selftest_mma_rate): one CTA per
    SM issues n_mma back-to-back M = 128, K = 16 bf16 MMAs of one shape; the
    per-instruction cycles and the implied whole-GPU TFLOP/s (CUDA events)."""
    from litevllm_b200 import _lib

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    nsm = torch.cuda.get_device_properties(dev).multi_processor_count
    cycles = torch.zeros(nsm, dtype=torch.int64, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    peak_tf, kind = measured_tflops()
    rec = {"n_mma": n_mma, "ctas": nsm}
    for shape, name, N in ((0, "ss_128x128x16", 128), (1, "ss_128x256x16", 256),
                           (2, "ts_128x128x16", 128), (3, "ts_128x128x16_b_mn_major", 128),
                           (4, "ss_128x128x16_b_mn_major", 128), (5, "ss_128x128x16_b_sw32", 128),
                           (6, "ss_128x128x16_ab_sw32", 128), (7, "ss_128x256x16_b_sw32", 256),
                           (8, "rot_ss_128x128x16", 128), (9, "rot_ss_128x256x16", 256),
                           (10, "rot_ts_128x128x16", 128), (11, "rot_ts_128x128x16_b_mn_major", 128),
                           (12, "rot_ss_128x128x16_b_mn_major", 128),
                           (13, "rot_ss_128x128x16_b_sw32", 128)):
        run = lambda: _lib.check(_lib.lib().lk_selftest_mma_rate(
            n_mma, shape, cycles.data_ptr(), status.data_ptr(), stream.cuda_stream))
        for _ in range(3):
            run()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        run()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        c = cycles.double()
        flops = nsm * n_mma * 2.0 * 128 * N * 16
        tf = flops / (e0.elapsed_time(e1) * 1e-3) / 1e12
        rec[name] = {"cycles_per_mma": round(float(c.median()) / n_mma, 1),
                     "tflops": round(tf, 1), "frac_of_bf16_peak": round(tf / peak_tf, 4)}
    rec["status"] = int(status.item())
    rec["peak"] = f"{peak_tf} TFLOP/s ({kind} bf16 burst)"
    return rec


def _decode_launches(num_splits: int) -> int:
    """Kernels one ops.paged_decode call launches (mirrors the library's
    LITEKERN_DECODE_ORDER switch: the longest-first ordering kernel runs before
    the split kernel unless it is set to 0; the persistent kernel is one)."""
    if num_splits < 0 or os.environ.get("LITEKERN_DECODE_ORDER", "1").strip() == "0":
        return 1
    return 2


def main():
    args = parse()
    os.environ["BENCH_CFG5_SEQS"] = str(args.cfg5_seqs)
    ws, rank, local = dist_env()
    if args.impl == "reference":
        run_reference(args, ws, rank)
        return
    if ws > 1:
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", device_id=torch.device("cuda", local))
    if args.workload != "cfg2":
        if args.workload == "sampler":
            torch.cuda.set_device(local)
            rec = {"workload": "sampler", **measure_sampler(args.steps, args.warmup, ws, local)}
        elif args.workload == "mma_rate":
            rec = {"workload": "mma_rate", **measure_mma_rate(local)}
        else:
            rec = measure_sub(args.workload, args.steps, args.warmup, ws, rank, local)
        if rank == 0:
            print(json.dumps(rec), flush=True)
        if ws > 1:
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()
        return
    r = run_ours(args, ws, rank, local)
    N = ws
    ms = r["ms"]
    B = r["B"]
    # value: whole-job hot-path bytes (summed over ranks) per second of the slowest rank
    job_bytes = r["job_bytes"]
    value = job_bytes / (ms * 1e-3) / 1e9
    dec_b = decode_bytes(r["ctx"], B)
    dec_gbs = dec_b / (r["dec_ms"] * 1e-3) / 1e9
    peak, peak_kind = measured_peak()
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": N,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": workload_config(N),
        "sampled_tok_s": round(r["job_seqs"] / (ms * 1e-3), 1),
        "decode_split_kv": r["nsplit"],
        "roofline": {
            "kernel": "paged_decode_kernel",
            "bound": "hbm",
            "achieved": round(dec_gbs, 1),
            "peak": peak,
            "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback 6.65 TB/s",
            "unit": "GB/s",
            "frac": round(dec_gbs / peak, 4),
            "traffic": profiled_traffic(),
            "traffic_source": "ncu dram bytes of one config-2 launch (profiles/paged_decode_cfg2.md), "
                              "not measured in this run",
            "algorithmic_bytes_per_launch": dec_b,
        },
        # per layer: store, decode ordering + decode (one launch when the
        # ordering kernel is switched off or the persistent kernel runs); sampler
        "gpu_launches": r["K"] * ((1 + _decode_launches(r["nsplit"])) * args.layers + 1),
        "clocks": r["clocks"],
        "per_rank": r["per_rank"],
    }
    if r["e2e"]:
        e = r["e2e"]
        line["e2e"] = {
            "value": round(job_bytes / (e["ms"] * 1e-3) / 1e9, 2),
            "unit": "GB/s",
            "h2d_bytes_per_step": e["h2d"],
            "d2h_bytes_per_step": e["d2h"],
            "ms_per_step": round(e["ms"], 4),
            "sampled_tok_s": round(r["job_seqs"] / (e["ms"] * 1e-3), 1),
            "host": e["host"],
            # the e2e step moves h2d_bytes_per_step over the host link: its own
            # roofline is that copy alone, measured with every rank copying
            "h2d_link_gbs_measured": round(e["h2d_gbs"], 1),
            "frac_of_h2d_link": round(e["h2d"] / (e["ms"] * 1e-3) / 1e9 / e["h2d_gbs"], 4),
        }
    if not args.no_sub:
        # every north-star target measured in the same run, after the headline
        torch.cuda.empty_cache()
        sub = {"sampler": measure_sampler(args.steps, args.warmup, ws, local)}
        for w in ("cfg5", "cfg3", "cfg4"):
            torch.cuda.empty_cache()
            rec = measure_sub(w, args.steps, args.warmup, ws, rank, local)
            for k_ in ("metric", "n_gpus", "steps", "workload"):
                rec.pop(k_, None)
            sub[w] = rec
        line["sub"] = sub
    if rank == 0 and N == 1 and not args.no_cpu_baseline:
        cb = cpu_baseline()
        line["cpu_baseline"] = {"value": round(cb["gbs"], 3), "unit": "GB/s", "cores": cb["cores"],
                                "kind": "port", "sample": cb["sample"],
                                "sampled_tok_s": round(cb["tok_s"], 2)}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if ws > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()

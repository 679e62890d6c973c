"""Benchmark: paged GQA decode attention + KV append, 760M decode shape.

One step = one decode step of the 760M model: for each of 24 layers, a KV
append of the new token followed by paged attention over that layer's own
cache (24 independent per-layer caches, ~7 GB, so L2 never holds a layer's K/V
between uses). Workload: batch 64, context ~ U[512, 2048], GQA 16/8, head_dim
112, page 16, bf16, values N(0,1)*0.5, randomly permuted pages.

``value`` is HBM GB/s of algorithmic bytes (K/V rows once per (sequence, KV
head), q, out, block-table rows, context lengths, append rows) with all inputs
resident in HBM; ``e2e`` is the same metric through the public API with the
step's per-token inputs (q, new K/V rows, block table, context lengths) copied
from pinned host memory and the outputs copied back inside the timed region.

``--impl reference`` times the CPU oracle (the reference algorithm restated in
C, OpenMP over all host cores) on one layer-call of the same workload per step.

Multi-GPU (torchrun): every rank runs its own batch of 64 sequences (requests
partitioned across GPUs, no collective on the data path); value = all ranks'
bytes / the slowest rank's time.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode-attn HBM GB/s (% of peak) and layer-calls/s at 1/2/4/8 B200 vs CPU ref"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="decode_760m")
    ap.add_argument("--layers", type=int, default=24)
    ap.add_argument("--schedule", default="auto", choices=["auto", "balanced", "split"])
    ap.add_argument("--split-pages", type=int, default=0)
    ap.add_argument("--no-graph", dest="graph", action="store_false",
                    help="launch every op from Python instead of replaying the step as one CUDA graph")
    ap.add_argument("--separate", action="store_true",
                    help="KV append as its own launch before attention (default: fused into one launch)")
    ap.add_argument("--no-overlap", dest="overlap", action="store_false",
                    help="no programmatic dependent launch between consecutive layer-calls")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    return ap.parse_args()


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profiled_traffic(workload: str):
    """DRAM bytes per attention launch from the committed ncu summary (or None)."""
    path = os.path.join(ROOT, "profiles", f"paged_decode_{workload}.md")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return int(float(line.split(":", 1)[1].strip()))
    except OSError:
        pass
    return None


class ClockSampler:
    """NVML samples of SM clock and throttle reasons while the timed region runs."""

    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4, "hw_slowdown": 0x8,
        "sync_boost": 0x10, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
        "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, index: int):
        self.samples, self.reasons = [], set()
        self.max_mhz = None
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for name, bit in self.REASONS.items():
                    if r & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.005)

    def __enter__(self):
        if self.nv is not None:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self.nv is not None:
            self.t.join()

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": len(self.samples)}


def cpu_oracle_run(lay, host, seconds: float, nthreads: int = 0):
    """Time the C oracle (append + attention, one layer) for about `seconds`."""
    from oracle import oracle
    oracle.build()
    kc, vc = host["k_cache"], host["v_cache"]
    calls, t0 = 0, time.perf_counter()
    while True:
        oracle.kv_append(host["k_new"], host["v_new"], kc, vc, host["slot_mapping"])
        _, st = oracle.paged_decode_attention(host["q"], kc, vc, host["block_table"], host["context_lens"],
                                              nthreads=nthreads)
        calls += 1
        el = time.perf_counter() - t0
        if el >= seconds or calls >= 1000:
            break
    return calls, el, oracle.num_threads() if nthreads <= 0 else nthreads


def host_layer(dev, layer):
    return {"q": dev["q"][layer].cpu(), "k_cache": dev["k_caches"][layer].cpu(),
            "v_cache": dev["v_caches"][layer].cpu(), "k_new": dev["k_new"][layer].cpu(),
            "v_new": dev["v_new"][layer].cpu(), "block_table": dev["block_table"].cpu(),
            "context_lens": dev["context_lens"].cpu(), "slot_mapping": dev["slot_mapping"].cpu()}


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    import torch
    import torch.distributed as dist
    from __graft_entry__ import load_package

    pkg = load_package()
    wl = pkg.workloads
    spec = wl.NAMED[args.workload]
    lay = wl.named_layout(args.workload, seed=1000 + rank)
    ebytes = {"float32": 4, "bfloat16": 2, "float16": 2}[spec["dtype"]]
    ab = wl.algorithmic_bytes(lay, ebytes)
    dtype_tag = {"float32": "f32", "bfloat16": "bf16", "float16": "f16"}[spec["dtype"]]
    config = {"workload": args.workload, "batch_per_gpu": lay.batch, "ctx_mean": float(lay.context_lens.mean()),
              "heads": [lay.num_heads, lay.num_kv_heads, lay.head_dim], "page": lay.block_size,
              "layers": args.layers, "kv_bytes_per_layer": int(2 * lay.num_blocks * lay.block_size *
                                                                lay.num_kv_heads * lay.head_dim * ebytes),
              "l2": "inputs > L2: 24 rotating per-layer caches",
              "parallelism": f"requests sharded, {world} GPU(s), no collective"}

    if args.impl == "reference":
        if rank != 0:
            return
        dev = wl.materialize_device(lay, 7, spec["dtype"], spec["scale_values"], 1, device="cpu") \
            if not torch.cuda.is_available() else None
        if dev is None:
            torch.cuda.set_device(local)
            dev = wl.materialize_device(lay, 7, spec["dtype"], spec["scale_values"], 1)
        host = host_layer(dev, 0)
        del dev
        from oracle import oracle
        oracle.build()
        times = []
        for i in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            oracle.kv_append(host["k_new"], host["v_new"], host["k_cache"], host["v_cache"], host["slot_mapping"])
            oracle.paged_decode_attention(host["q"], host["k_cache"], host["v_cache"], host["block_table"],
                                          host["context_lens"])
            if i >= args.warmup:
                times.append(time.perf_counter() - t0)
        tot = sum(times)
        gbs = ab["layer_call"] * len(times) / tot / 1e9
        cores = oracle.num_threads()
        sample = f"one layer-call (append + attention) of the {lay.batch}-sequence batch per step, host cores"
        print(json.dumps({
            "metric": METRIC, "value": round(gbs, 4), "unit": "GB/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * tot / len(times),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": dtype_tag,
            "data": "synthetic", "config": config, "layer_calls_per_s": len(times) / tot,
            "cpu_baseline": {"value": round(gbs, 4), "unit": "GB/s", "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(gbs, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }))
        return

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)

    L = args.layers
    dev = wl.materialize_device(lay, 7 + rank, spec["dtype"], spec["scale_values"], L)
    outs = [torch.empty_like(dev["q"][l]) for l in range(L)]
    bt, cl, sm = dev["block_table"], dev["context_lens"], dev["slot_mapping"]
    kw = dict(schedule=args.schedule, split_pages=args.split_pages)
    launches_per_layer = (2 if args.separate else 1) + (1 if args.schedule == "split" else 0)

    def layer(l, q, k_new, v_new, block_table, context_lens, out, slots=None, timer=None):
        """One layer-call: the new token's K/V append, then attention (engine.py:213-224)."""
        if args.separate:
            pkg.kv_append(k_new, v_new, dev["k_caches"][l], dev["v_caches"][l], slots)
        if timer is not None:
            timer[0].record()
        if args.separate:
            pkg.paged_attention(q, dev["k_caches"][l], dev["v_caches"][l], block_table, context_lens, out=out, **kw)
        else:
            # the previous kernel on the stream is another layer's attention (or a copy):
            # it writes neither this layer's pool nor the block table / context lengths
            pkg.paged_attention(q, dev["k_caches"][l], dev["v_caches"][l], block_table, context_lens, out=out,
                                k_new=k_new, v_new=v_new, overlap_previous=args.overlap, **kw)
        if timer is not None:
            timer[1].record()

    def step(timers=None):
        for l in range(L):
            layer(l, dev["q"][l], dev["k_new"][l], dev["v_new"][l], bt, cl, outs[l], sm,
                  None if timers is None else timers[l])

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def capture(fn):
        """CUDA graph of fn (warmed up on a side stream first, as graph capture needs)."""
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            fn()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        return g

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    pkg.check_device_errors(device)
    graph = capture(step) if args.graph else None
    if graph is not None:
        for _ in range(max(3, args.warmup)):
            graph.replay()

    # ---- device-resident timing (value)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    timers = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(L)]
              for _ in range(args.steps)]
    barrier()
    with ClockSampler(local) as clocks:
        ev0.record()
        for k in range(args.steps):
            if graph is not None:
                graph.replay()
            else:
                step(timers[k])
        ev1.record()
        torch.cuda.synchronize()
    barrier()
    ms = ev0.elapsed_time(ev1)
    ms_max = max_over_ranks(ms)
    pkg.check_device_errors(device)

    # ---- dominant kernel: average launch time on its own stream
    if graph is None:
        attn_ms = [a.elapsed_time(b) for row in timers for (a, b) in row]
        kernel_avg_ms = sum(attn_ms) / len(attn_ms)
    elif not args.separate and args.schedule != "split":
        kernel_avg_ms = ms / (args.steps * L)   # the step is exactly L launches of the fused kernel
    else:
        def attn_only():
            for l in range(L):
                pkg.paged_attention(dev["q"][l], dev["k_caches"][l], dev["v_caches"][l], bt, cl, out=outs[l], **kw)
        ga = capture(attn_only)
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a0.record()
        for _ in range(args.steps):
            ga.replay()
        a1.record()
        torch.cuda.synchronize()
        kernel_avg_ms = a0.elapsed_time(a1) / (args.steps * L)
        del ga
    kernel_bytes = ab["attention"] if args.separate else ab["layer_call"]

    # ---- end to end through the public API with host buffers
    qh = torch.stack([x.cpu() for x in dev["q"]]).pin_memory()
    knh = torch.stack([x.cpu() for x in dev["k_new"]]).pin_memory()
    vnh = torch.stack([x.cpu() for x in dev["v_new"]]).pin_memory()
    bth, clh = bt.cpu().pin_memory(), cl.cpu().pin_memory()
    outh = torch.empty((L,) + tuple(outs[0].shape), dtype=outs[0].dtype).pin_memory()
    qd, knd, vnd = torch.empty_like(qh, device=device), torch.empty_like(knh, device=device), \
        torch.empty_like(vnh, device=device)
    btd, cld = torch.empty_like(bth, device=device), torch.empty_like(clh, device=device)
    posd = torch.empty_like(clh, device=device)
    smd = torch.empty(lay.batch, dtype=torch.int64, device=device)
    outd = torch.empty_like(outh, device=device)

    def e2e_step():
        btd.copy_(bth, non_blocking=True)
        cld.copy_(clh, non_blocking=True)
        qd.copy_(qh, non_blocking=True)
        knd.copy_(knh, non_blocking=True)
        vnd.copy_(vnh, non_blocking=True)
        if args.separate:
            torch.sub(cld, 1, out=posd)
            pkg.slot_mapping(btd, posd, lay.block_size, out=smd)
        for l in range(L):
            layer(l, qd[l], knd[l], vnd[l], btd, cld, outd[l], smd)
        outh.copy_(outd, non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    eg = capture(e2e_step) if args.graph else None
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        if eg is not None:
            eg.replay()
        else:
            e2e_step()
    e1.record()
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    h2d = sum(t.numel() * t.element_size() for t in (bth, clh, qh, knh, vnh))
    d2h = outh.numel() * outh.element_size()
    assert torch.equal(outh[0].to(device), outs[0]), "end-to-end output differs from the device-resident step"
    del eg

    total_bytes_step = ab["layer_call"] * L * world
    value = total_bytes_step * args.steps / (ms_max / 1e3) / 1e9
    e2e_val = total_bytes_step * args.steps / (e2e_ms / 1e3) / 1e9
    peak, peak_kind = peaks()

    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": dtype_tag, "data": "synthetic", "config": config,
        "layer_calls_per_s": round(L * world * args.steps / (ms_max / 1e3), 1),
        "frac_of_hbm_peak": round(value / world / peak, 4),
        "gpu_launches": args.steps * L * launches_per_layer,
        "e2e": {"value": round(e2e_val, 2), "unit": "GB/s", "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h), "ms_per_step": round(e2e_ms / args.steps, 4)},
        "clocks": clocks.summary(),
        "graph": bool(graph is not None), "append": "separate launch" if args.separate else "fused",
        "overlap_previous": bool(args.overlap and not args.separate),
    }
    achieved = kernel_bytes / (kernel_avg_ms / 1e3) / 1e9
    traffic = profiled_traffic(args.workload)
    line["roofline"] = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                        "frac": round(achieved / peak, 4), "traffic": traffic,
                        "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                        else "fallback 6650 GB/s",
                        "kernel": "paged_decode_mma_kernel" + ("" if args.separate else " (KV append fused)"),
                        "algorithmic_bytes_per_launch": kernel_bytes, "avg_launch_us": round(kernel_avg_ms * 1e3, 2),
                        "timing": "per-launch CUDA events" if graph is None else "graph replay / launches"}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        host = host_layer(dev, 0)
        calls, el, thr = cpu_oracle_run(lay, host, args.cpu_seconds)
        cpu_gbs = ab["layer_call"] * calls / el / 1e9
        line["cpu_baseline"] = {"value": round(cpu_gbs, 4), "unit": "GB/s", "cores": thr, "kind": "port",
                                "sample": f"{calls} layer-call(s) (append + attention) of layer 0 of this "
                                          f"workload, C oracle with OpenMP, {el:.1f} s"}
    if rank == 0:
        print(json.dumps(line))
    del graph
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

"""Benchmark: paged GQA decode attention + KV append, 760M decode shape.

One step = one decode step of the 760M model: for each of 24 layers, the new
token's K/V append and paged attention over that layer's own cache, fused in
one launch (24 independent per-layer caches, ~7 GB, so L2 never holds a
layer's K/V between uses). Default workload (decode_760m): batch 64, context
~ U[512, 2048], GQA 16/8, head_dim 112, page 16, bf16, values N(0,1)*0.5,
randomly permuted pages. The step is replayed as one CUDA graph, and
consecutive layer-calls overlap through programmatic dependent launch.

``value`` is HBM GB/s of algorithmic bytes (K/V rows once per (sequence, KV
head), q, out, block-table rows, context lengths, append rows) with all inputs
resident in HBM; ``e2e`` is the same metric through the public API with the
step's per-token inputs (q, new K/V rows, block table, context lengths) copied
from pinned host memory and the outputs copied back inside the timed region, on
copy streams that overlap the layer-calls (layer l waits for its own inputs).

``e2e_eager`` is the same end-to-end step launched from Python every step,
with no CUDA graph and no events between launches, as the engine's eager
decode loop calls the ops.

``--impl reference`` times the CPU oracle (the reference algorithm restated in
C, OpenMP over all host cores) on one layer-call of the same workload per step.
``cpu_baseline_ref`` reports the reference's own Python path
(paged_decode_attention_ref + PagedKVCache.write_kv), timed where the
reference is importable on a subsample and extrapolated
(oracle/reference_cpu_path.json, made by oracle/time_reference_cpu.py).

``--op handoff`` and ``--op prefill`` measure the rows either side of the step
(the KV page hand-off between workers, a prefill chunk's KV write); see
bench_handoff and bench_prefill.

Multi-GPU (torchrun): decode_760m runs one batch of 64 per GPU (weak scaling:
requests partitioned across GPUs, no collective on the data path);
``--workload box_scale`` splits one batch of 1024 requests over the GPUs
(strong scaling, LPT placement, KV-head split of contexts over 2048 tokens).
value = all ranks' bytes / the slowest rank's time. Every default line also
carries ``box_scale``: that strong-scaling split measured in the same run at
this N, with the whole batch timed on rank 0's GPU alone for its efficiency.

The default 200 timed steps keep the timed region long enough (about 0.25 s
on one GPU) for a few dozen NVML clock samples.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode-attn HBM GB/s (% of peak) and layer-calls/s at 1/2/4/8 B200 vs CPU ref"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="decode_760m",
                    choices=["decode_760m", "correctness", "long_context", "radix_prefix", "box_scale"])
    ap.add_argument("--layers", type=int, default=24)
    ap.add_argument("--schedule", default="auto", choices=["auto", "balanced", "split"])
    ap.add_argument("--split-pages", type=int, default=0)
    ap.add_argument("--no-graph", dest="graph", action="store_false",
                    help="launch every op from Python instead of replaying the step as one CUDA graph")
    ap.add_argument("--separate", action="store_true",
                    help="KV append as its own launch before attention (default: fused into one launch)")
    ap.add_argument("--no-overlap", dest="overlap", action="store_false",
                    help="no programmatic dependent launch between consecutive layer-calls")
    ap.add_argument("--op", choices=["decode", "handoff", "prefill"], default="decode",
                    help="decode: the decode layer-call (default); handoff: KV page hand-off between workers; "
                         "prefill: the KV write of a 2048-token prompt chunk into every layer's pool")
    ap.add_argument("--prep", action="store_true",
                    help="layer-call = q/k RMSNorm + rotary embedding + KV append + attention in one launch "
                         "(the attention block between the QKV projection and o_proj)")
    ap.add_argument("--cascade", action="store_true",
                    help="read pages shared by several requests (radix prefix) once per layer-call: suffix and "
                         "shared-prefix passes in one launch, then a merge (plan built on the host once per step)")
    ap.add_argument("--prefix-ctas", type=int, default=None,
                    help="--cascade: CTAs of the one launch given to the shared-prefix pass (default: the plan's "
                         "cost model; 0: the two passes as two launches)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-box-scale", dest="box_scale", action="store_false",
                    help="skip the box-scale strong-scaling sub-record of the default decode_760m line")
    ap.add_argument("--box-scale-layers", type=int, default=12,
                    help="per-layer caches of the box-scale sub-record (4.5 GB each on one GPU, > L2)")
    return ap.parse_args()


def host_info():
    """The host the CPU baseline ran on: logical CPUs, the ones this process may
    use, and the CPU model."""
    model = None
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    usable = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    return {"cpu_count": os.cpu_count(), "usable_cpus": usable, "cpu_model": model}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profiled_traffic(summary: str):
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary
    profiles/<summary>.md (or None)."""
    path = os.path.join(ROOT, "profiles", f"{summary}.md")
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


class Staging:
    """A pinned host buffer and a device buffer with the same layout of named,
    256-byte aligned sections; copy_range moves sections first..last (in
    layout order) host -> device in one copy."""

    def __init__(self, specs, device):
        import torch
        self.layout, off = {}, 0
        for name, shape, dtype in specs:
            n = torch.Size(shape).numel() * torch.empty((), dtype=dtype).element_size()
            self.layout[name] = (off, n, tuple(shape), dtype)
            off = (off + n + 255) // 256 * 256
        self.host = torch.empty(off, dtype=torch.uint8).pin_memory()
        self.dev = torch.empty(off, dtype=torch.uint8, device=device)
        self.nbytes = sum(n for _, n, _, _ in self.layout.values())  # payload, without the alignment gaps

    def view(self, buf, name):
        off, n, shape, dtype = self.layout[name]
        return buf[off:off + n].view(dtype).view(shape)

    def copy_range(self, first, last):
        a = self.layout[first][0]
        off, n, _, _ = self.layout[last]
        self.dev[a:off + n].copy_(self.host[a:off + n], non_blocking=True)


def build_parts(pkg, workload: str, rank: int, world: int):
    """The (name, Layout) parts this rank attends over each layer, the scaling
    mode, and the whole workload's layout."""
    wl, sh = pkg.workloads, pkg.sharding
    if workload == "box_scale":
        glay = wl.named_layout("box_scale", seed=0)
        shard = sh.plan_shards(glay.context_lens, world)[rank]
        parts = []
        if len(shard.whole):
            parts.append(("whole", sh.local_layout(glay.context_lens, shard.whole, 1000 + rank, 16, 8)))
        if shard.kv_head_count:
            G = glay.num_heads // glay.num_kv_heads
            parts.append(("kv_head_slice", sh.local_layout(glay.context_lens, shard.head_split, 2000 + rank,
                                                           G * shard.kv_head_count, shard.kv_head_count)))
        return parts, "strong", glay
    lay = wl.named_layout(workload, seed=1000 + rank)
    return [("batch", lay)], "weak", lay


def host_layer(dev, layer):
    return {"q": dev["q"][layer].cpu(), "k_cache": dev["k_caches"][layer].cpu(),
            "v_cache": dev["v_caches"][layer].cpu(), "k_new": dev["k_new"][layer].cpu(),
            "v_new": dev["v_new"][layer].cpu(), "block_table": dev["block_table"].cpu(),
            "context_lens": dev["context_lens"].cpu(), "slot_mapping": dev["slot_mapping"].cpu()}


def cpu_layer_call(oracle, host):
    """The oracle's KV append then attention: one layer-call of the reference algorithm
    (with ``prep`` in host: the q/k RMSNorm and rotary embedding first)."""
    if "prep" in host:
        import torch
        pr = host["prep"]
        q, k, _ = oracle.qk_norm_rope(host["q"], host["k_new"], pr["q_w"], pr["k_w"], pr["rope"],
                                      host["context_lens"].numpy() - 1, 1e-6)
        host = dict(host, q=torch.from_numpy(q).to(host["q"].dtype), k_new=torch.from_numpy(k).to(host["q"].dtype))
    oracle.kv_append(host["k_new"], host["v_new"], host["k_cache"], host["v_cache"], host["slot_mapping"])
    _, st = oracle.paged_decode_attention(host["q"], host["k_cache"], host["v_cache"], host["block_table"],
                                          host["context_lens"])
    return st


PLAN_FIELDS = ("suffix_block_table", "suffix_context_lens", "page_list", "member_list", "work", "merge_items")
HANDOFF_METRIC = "KV hand-off GB/s of page payload (prefill pool -> decode pool)"
PREFILL_METRIC = "prefill KV write GB/s of algorithmic bytes (chunk rows -> paged pool)"


def bench_handoff(args):
    """One step = hand one finished 2048-token prompt of the 760M model (24 layers,
    128 pages of 16 x 8 x 112 bf16, K and V: 176 MB) from a prefill worker's pool
    to a decode worker's pool, at other page ids (worker.py:175-183 -> :217-223).
    N=1: both pools on one GPU, one page-copy kernel (HBM read + write).
    N>=2: ranks pair up (2k -> 2k+1), the decode worker's pool is mapped into the
    prefill worker over CUDA IPC and written over NVLink by one kernel.
    e2e: the reference's host path through this package's drop-ins,
    serialize_blocks -> host bytes -> deserialize_blocks."""
    import torch
    import torch.distributed as dist
    from __graft_entry__ import load_package

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    pkg = load_package()
    ho = pkg.handoff
    L, KVH, D, bs, npg, NB = 24, 8, 112, 16, 128, 1536
    payload = L * 2 * npg * bs * KVH * D * 2
    config = {"workload": "handoff_760m_prompt2048", "layers": L, "pages": npg, "page_bytes": bs * KVH * D * 2,
              "pool_pages": NB, "dtype": "bf16",
              "l2": "inputs > L2: 176 MB payload per step, 8 rotating page sets",
              "parallelism": "single GPU" if world == 1 else f"{world // 2} prefill->decode pair(s) over NVLink"}

    def pool(seed):
        g = torch.Generator(device="cuda")
        g.manual_seed(seed)
        t = torch.empty((L, 2, NB, bs, KVH, D), dtype=torch.bfloat16, device="cuda")
        for l in range(L):
            t[l].copy_(torch.randn((2, NB, bs, KVH, D), generator=g, device="cuda"))
        return t

    def page_sets(seed):
        g = torch.Generator(device="cuda")
        g.manual_seed(seed)
        return [torch.randperm(NB, generator=g, device="cuda")[:npg].to(torch.int32) for _ in range(8)]

    if args.impl == "reference":
        if rank != 0:
            return
        from oracle import oracle
        src = torch.randn((L, 2, 256, bs, KVH, D)).to(torch.bfloat16)
        dst = torch.zeros_like(src)
        sp = list(range(0, 256, 2))
        dp = list(range(1, 256, 2))
        times = []
        for i in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            oracle.scatter_pages(oracle.gather_pages(src, sp), dst, dp)
            if i >= args.warmup:
                times.append(time.perf_counter() - t0)
        v = payload * len(times) / sum(times) / 1e9
        print(json.dumps({
            "metric": HANDOFF_METRIC, "value": round(v, 3), "unit": "GB/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * sum(times) / len(times),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": config,
            "cpu_baseline": {"value": round(v, 3), "unit": "GB/s", "cores": 1, "kind": "port", **host_info(),
                             "sample": "one prompt's pages per step: numpy gather + scatter (the reference's "
                                       "serialize_blocks / deserialize_blocks without the socket)"},
            "e2e": {"value": round(v, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))
        return

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    sender = world == 1 or (rank % 2 == 0 and rank + 1 < world)
    receiver = world > 1 and rank % 2 == 1
    src = pool(100 + rank) if sender else None
    dst = pool(200 + rank) if (receiver or world == 1) else None
    sps, dps = page_sets(300 + rank), page_sets(400 + rank)
    mapping = None
    if world > 1:
        tokens = [None] * world
        dist.all_gather_object(tokens, ho.ipc_export(dst) if receiver else None)
        if sender:
            mapping = ho.ipc_import(tokens[rank + 1], device)

    def step(k):
        if not sender:
            return
        if mapping is None:
            ho.transfer_pages(src, sps[k % 8], dst, dps[k % 8])
        else:
            ho.transfer_pages_to_ipc(src, sps[k % 8], mapping, (L, 2, NB, bs, KVH, D), dps[k % 8])

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()

    for k in range(max(3, args.warmup)):
        step(k)
    barrier()
    # one CUDA graph per page set (one copy kernel each), so host-side argument
    # handling stays out of the timed device timeline
    graphs = []
    if sender:
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for k in range(8):
                step(k)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        for k in range(8):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                step(k)
            graphs.append(g)
        for g in graphs:
            g.replay()
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        ev0.record()
        for k in range(args.steps):
            if graphs:
                graphs[k % 8].replay()
        ev1.record()
        torch.cuda.synchronize()
    barrier()
    del graphs
    ms = ev0.elapsed_time(ev1) if sender else 0.0
    ms_max, pairs = ms, 1
    if world > 1:
        t = torch.tensor([ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_max, pairs = float(t.item()), world // 2
    value = pairs * payload * args.steps / (ms_max / 1e3) / 1e9
    pkg.check_device_errors(device)

    # e2e: the reference's host path (device gather -> host bytes -> device scatter)
    e2e = None
    if world == 1:
        sp_l = [sps[0].tolist(), sps[1].tolist()]
        dp_l = [dps[0].tolist(), dps[1].tolist()]
        for k in range(2):
            ho.deserialize_blocks(dst, ho.serialize_blocks(src, sp_l[k]), dp_l[k])
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        n_e2e = max(3, args.steps // 4)
        for k in range(n_e2e):
            ho.deserialize_blocks(dst, ho.serialize_blocks(src, sp_l[k % 2]), dp_l[k % 2])
        e1.record()
        torch.cuda.synchronize()
        e_ms = e0.elapsed_time(e1) / n_e2e
        e2e = {"value": round(payload / (e_ms / 1e3) / 1e9, 2), "unit": "GB/s", "h2d_bytes_per_step": payload + 64,
               "d2h_bytes_per_step": payload + 64, "ms_per_step": round(e_ms, 4),
               "path": "serialize_blocks -> host bytes -> deserialize_blocks (checksum verified)"}
    if world > 1:
        if mapping is not None:
            mapping.close()
        dist.barrier()

    peak, kind = peaks()
    per_step_ms = ms_max / args.steps
    line = {"metric": HANDOFF_METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per_step_ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic", "config": config, "gpu_launches": args.steps * (1 if sender else 0),
            "clocks": clocks.summary(), "e2e": e2e}
    if world == 1:
        ach = 2 * payload / (per_step_ms / 1e3) / 1e9
        line["roofline"] = {"bound": "hbm", "achieved": round(ach, 1), "peak": peak, "unit": "GB/s",
                            "frac": round(ach / peak, 4), "traffic": None,
                            "kernel": "kv_pages_bulk_kernel (TMA bulk load/store ring)",
                            "algorithmic_bytes_per_launch": 2 * payload, "avg_launch_us": round(per_step_ms * 1e3, 2),
                            "peak_source": f"{kind} (MEASURED_PEAKS.json hbm_gbs, read + write bytes)"}
    else:
        ach = payload / (per_step_ms / 1e3) / 1e9
        line["roofline"] = {"bound": "nvlink", "achieved": round(ach, 1), "peak": 770.0, "unit": "GB/s",
                            "frac": round(ach / 770.0, 4), "traffic": None,
                            "kernel": "kv_pages_copy_kernel (16-byte stores into the peer's pool)",
                            "algorithmic_bytes_per_launch": payload, "avg_launch_us": round(per_step_ms * 1e3, 2),
                            "peak_source": "measured peer copy per direction on this pool (770 GB/s)"}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import oracle
        hs = src[:, :, :256].cpu()
        hd = torch.zeros_like(hs)
        t0, n = time.perf_counter(), 0
        while time.perf_counter() - t0 < min(args.cpu_seconds, 5.0) or n == 0:
            oracle.scatter_pages(oracle.gather_pages(hs, list(range(0, 256, 2))), hd, list(range(1, 256, 2)))
            n += 1
        el = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": round(payload * n / el / 1e9, 3), "unit": "GB/s", "cores": 1,
                                "kind": "port", **host_info(), "sample": f"{n} prompt(s): numpy gather + scatter of 128 pages x 24 "
                                                          f"layers, {el:.1f} s"}
    if rank == 0:
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def bench_prefill(args):
    """One step = the KV write of one 2048-token prompt chunk of the 760M model into
    all 24 layers' pools (prefill_step, engine.py:121-128): per layer the slot
    computation over the chunk's positions and one append launch
    (``ops.prefill_kv_write``), or with ``--prep`` the q/k RMSNorm + rotary + append
    launch (``ops.prefill_prep``). Inputs > L2: 24 layers' chunk rows (352 MB with
    q) and 24 pools of 1536 pages. N GPUs: each rank writes its own prompt (weak
    scaling, no collective on the data path); value = all ranks' bytes / the
    slowest rank's time."""
    import torch
    import torch.distributed as dist
    from __graft_entry__ import load_package

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    L, T, H, KVH, D, bs, NB = args.layers, 2048, 16, 8, 112, 16, 1536
    npg = T // bs
    row_b = KVH * D * 2                      # one token's K (or V) row, bf16
    # algorithmic bytes per layer: the chunk's K/V rows read and written into the
    # pool, the slots written (and, with --prep, read back), the block-table row
    lay_b = 2 * T * row_b * 2 + T * 8 * (2 if args.prep else 1) + npg * 4
    if args.prep:  # + q read and written, k written out, rotary rows, weights, positions
        lay_b += 2 * T * H * D * 2 + T * row_b + T * (D // 2) * 8 + 2 * D * 2 + T * 4
    config = {"workload": "prefill_760m_chunk2048", "layers": L, "tokens": T, "heads": [H, KVH, D], "page": bs,
              "pool_pages": NB, "dtype": "bf16",
              "layer_call": "q/k RMSNorm + rotary + KV write" if args.prep else "slot mapping + KV write",
              "l2": "inputs > L2: per-layer chunk rows and pools",
              "parallelism": f"{world} GPU(s), one prompt each, no collective"}

    def host_chunk(seed):
        g = torch.Generator()
        g.manual_seed(seed)
        c = {"k": torch.randn((L, T, KVH, D), generator=g).to(torch.bfloat16),
             "v": torch.randn((L, T, KVH, D), generator=g).to(torch.bfloat16),
             "row": torch.randperm(NB, generator=g)[:npg].to(torch.int32)}
        if args.prep:
            c["q"] = torch.randn((L, T, H, D), generator=g).to(torch.bfloat16)
            c["q_w"] = (1 + 0.1 * torch.randn((L, D), generator=g)).to(torch.bfloat16)
            c["k_w"] = (1 + 0.1 * torch.randn((L, D), generator=g)).to(torch.bfloat16)
        return c

    if args.impl == "reference":
        if rank != 0:
            return
        from oracle import oracle
        oracle.build()
        cores = oracle.use_all_cores()
        c = host_chunk(1000)
        kc = torch.zeros((NB, bs, KVH, D), dtype=torch.bfloat16)
        vc = torch.zeros_like(kc)
        pkg = load_package()
        rope = pkg.rope_table(D, 2 * T, 500000.0, device="cpu") if args.prep else None
        slots = (c["row"].long()[torch.arange(T) // bs] * bs + torch.arange(T) % bs)
        times = []
        for i in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            k, v = c["k"][0], c["v"][0]
            if args.prep:
                _, k_r, _ = oracle.qk_norm_rope(c["q"][0], k, c["q_w"][0], c["k_w"][0], rope,
                                                torch.arange(T).numpy(), 1e-6)
                k = torch.from_numpy(k_r).to(torch.bfloat16)
            oracle.kv_append(k, v, kc, vc, slots)
            if i >= args.warmup:
                times.append(time.perf_counter() - t0)
        v = lay_b * len(times) / sum(times) / 1e9
        print(json.dumps({
            "metric": PREFILL_METRIC, "value": round(v, 4), "unit": "GB/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * sum(times) / len(times),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": config,
            "cpu_baseline": {"value": round(v, 4), "unit": "GB/s", "cores": cores, "kind": "port", **host_info(),
                             "sample": "one layer of the 2048-token chunk per step: "
                                       + ("numpy q/k norm + rotary, then " if args.prep else "")
                                       + "the C oracle's slot write"},
            "e2e": {"value": round(v, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))
        return

    pkg = load_package()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    c = host_chunk(1000 + rank)
    g = torch.Generator(device=device)
    g.manual_seed(2000 + rank)
    kcs = [torch.randn((NB, bs, KVH, D), generator=g, device=device).to(torch.bfloat16) for _ in range(L)]
    vcs = [torch.randn((NB, bs, KVH, D), generator=g, device=device).to(torch.bfloat16) for _ in range(L)]
    dk, dv, drow = c["k"].to(device), c["v"].to(device), c["row"].to(device)
    rope = pkg.rope_table(D, 2 * T, 500000.0, device=device) if args.prep else None
    if args.prep:
        dq, dqw, dkw = c["q"].to(device), c["q_w"].to(device), c["k_w"].to(device)
    outs = {}

    pre = {}

    def step_inputs(row):
        # positions and slots of the chunk: the same for every layer, once per step
        if args.prep:
            pre["ps"] = pkg.prefill_positions_and_slots(row, 0, T, bs)

    def layer(l, k, v, row, q=None):
        if args.prep:
            outs[l] = pkg.prefill_prep(q, k, v, dqw[l], dkw[l], rope, kcs[l], vcs[l], row, 0,
                                       positions_and_slots=pre["ps"])
        else:
            outs[l] = pkg.prefill_kv_write(k, v, kcs[l], vcs[l], row, 0, overlap_previous=args.overlap)

    def step():
        step_inputs(drow)
        for l in range(L):
            layer(l, dk[l], dv[l], drow, dq[l] if args.prep else None)

    def capture(fn):
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            fn()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            fn()
        return gr

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()

    def reduce_max(x):
        if world == 1:
            return x
        t = torch.tensor([x], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    pkg.check_device_errors(device)
    # the pool rows equal the chunk rows (K after the norm and rotary with --prep)
    slots = outs[0] if not args.prep else pkg.prefill_slots(drow, 0, T, bs)
    if not args.prep:
        got = kcs[0].view(-1, KVH, D)[slots]
        assert torch.equal(got, dk[0]), "pool rows differ from the chunk's K rows"
    graph = capture(step)
    for _ in range(max(3, args.warmup)):
        graph.replay()
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        ev0.record()
        for _ in range(args.steps):
            graph.replay()
        ev1.record()
        torch.cuda.synchronize()
    barrier()
    ms = reduce_max(ev0.elapsed_time(ev1))
    del graph
    step_b = L * lay_b

    # e2e: the chunk's rows from pinned host memory every step (on a copy stream,
    # in growing layer groups), the last layer's slots back to the host
    hk, hv = c["k"].pin_memory(), c["v"].pin_memory()
    hq = c["q"].pin_memory() if args.prep else None
    h_out = torch.empty(T, dtype=torch.int64).pin_memory()
    ek, ev_ = torch.empty_like(dk), torch.empty_like(dv)
    eq = torch.empty_like(dq) if args.prep else None
    s_in = torch.cuda.Stream(device)
    groups, l0, n = [], 0, 1
    while l0 < L:
        groups.append((l0, min(L, l0 + n) - 1))
        l0, n = l0 + n, 3 * n
    ev_in = [torch.cuda.Event() for _ in groups]

    def e2e_step():
        main = torch.cuda.current_stream(device)
        s_in.wait_stream(main)
        with torch.cuda.stream(s_in):
            for gi, (a, b) in enumerate(groups):
                ek[a:b + 1].copy_(hk[a:b + 1], non_blocking=True)
                ev_[a:b + 1].copy_(hv[a:b + 1], non_blocking=True)
                if args.prep:
                    eq[a:b + 1].copy_(hq[a:b + 1], non_blocking=True)
                ev_in[gi].record(s_in)
        step_inputs(drow)
        for gi, (a, b) in enumerate(groups):
            main.wait_event(ev_in[gi])
            for l in range(a, b + 1):
                layer(l, ek[l], ev_[l], drow, eq[l] if args.prep else None)
        main.wait_stream(s_in)
        res = outs[L - 1] if not args.prep else slots
        h_out.copy_(res, non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    eg = capture(e2e_step)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        eg.replay()
    e1.record()
    torch.cuda.synchronize()
    barrier()
    e_ms = reduce_max(e0.elapsed_time(e1))
    del eg
    pkg.check_device_errors(device)
    h2d = (hk.numel() + hv.numel() + (hq.numel() if args.prep else 0)) * 2
    peak, kind = peaks()
    per_layer_us = ms / args.steps / L * 1e3
    line = {"metric": PREFILL_METRIC, "value": round(world * step_b * args.steps / (ms / 1e3) / 1e9, 2),
            "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": config,
            "tokens_per_s": round(world * T * args.steps / (ms / 1e3), 1),
            "gpu_launches": args.steps * (L + 1 if args.prep else L),
            "e2e": {"value": round(world * step_b * args.steps / (e_ms / 1e3) / 1e9, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": int(world * h2d), "d2h_bytes_per_step": int(world * T * 8),
                    "ms_per_step": round(e_ms / args.steps, 4)},
            "clocks": clocks.summary(),
            "roofline": {"bound": "hbm", "achieved": round(lay_b / (per_layer_us / 1e6) / 1e9, 1), "peak": peak,
                         "unit": "GB/s", "frac": round(lay_b / (per_layer_us / 1e6) / 1e9 / peak, 4),
                         "traffic": None, "peak_source": f"{kind} (MEASURED_PEAKS.json hbm_gbs)",
                         "kernel": ("qk_norm_rope_vec_kernel (append fused; slots once per step)" if args.prep
                                    else "prefill_append_kernel (slots computed in the kernel)"),
                         "algorithmic_bytes_per_launch": int(lay_b), "avg_launch_us": round(per_layer_us, 2),
                         "timing": "graph replay / layers (the layer's launches together)"}}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import oracle
        oracle.build()
        cores = oracle.use_all_cores()
        kc = kcs[0].cpu()
        vc = vcs[0].cpu()
        hs = slots.cpu()
        hrope = rope.cpu() if args.prep else None
        t0, calls = time.perf_counter(), 0
        while True:
            k, v = c["k"][calls % L], c["v"][calls % L]
            if args.prep:
                _, k_r, _ = oracle.qk_norm_rope(c["q"][calls % L], k, c["q_w"][calls % L], c["k_w"][calls % L],
                                                hrope, torch.arange(T).numpy(), 1e-6)
                k = torch.from_numpy(k_r).to(torch.bfloat16)
            oracle.kv_append(k, v, kc, vc, hs)
            calls += 1
            el = time.perf_counter() - t0
            if el >= min(args.cpu_seconds, 5.0) or calls >= 100000:
                break
        line["cpu_baseline"] = {"value": round(lay_b * calls / el / 1e9, 4), "unit": "GB/s", "cores": cores,
                                "kind": "port", **host_info(), "sample": f"{calls} layer write(s) of the 2048-token chunk, {el:.1f} s"}
    if rank == 0:
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def box_scale_record(args, pkg, rank: int, world: int, device, reduce_max, barrier):
    """Strong-scaling sub-record carried by every default line: the box-scale
    batch (1024 requests, contexts log-normal with median 1024, clipped to
    [128, 4096]) split over the N GPUs of this run by ``plan_shards`` (LPT
    placement, KV-head split of contexts over 2048 tokens; no collective on the
    data path), each layer-call its KV append + attention launch(es), timed like
    the main step (CUDA-graph replay, device events, max over ranks). Rank 0
    then runs the whole batch alone (the one-GPU plan) in the same process, the
    baseline of the efficiency value_N / (N * value_1). ``--box-scale-layers``
    per-layer caches rotate (4.5 GB each on one GPU: every layer-call streams
    from HBM)."""
    import torch
    wl = pkg.workloads
    spec = wl.NAMED["box_scale"]
    L = args.box_scale_layers

    def timed(parts, seed0):
        devs = [wl.materialize_device(lay, seed0 + i, spec["dtype"], spec["scale_values"], L)
                for i, (_, lay) in enumerate(parts)]
        outs = [[torch.empty_like(d["q"][l]) for l in range(L)] for d in devs]

        def step():
            for l in range(L):
                for i, d in enumerate(devs):
                    pkg.paged_attention(d["q"][l], d["k_caches"][l], d["v_caches"][l], d["block_table"],
                                        d["context_lens"], out=outs[i][l], k_new=d["k_new"][l], v_new=d["v_new"][l],
                                        overlap_previous=True)

        for _ in range(max(3, args.warmup)):
            step()
        torch.cuda.synchronize()
        pkg.check_device_errors(device)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            step()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            step()
        for _ in range(max(3, args.warmup)):
            g.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        with ClockSampler(device.index) as clocks:
            e0.record()
            for _ in range(args.steps):
                g.replay()
            e1.record()
            torch.cuda.synchronize()
        del g
        pkg.check_device_errors(device)
        step_bytes = L * sum(wl.algorithmic_bytes(lay, 2)["layer_call"] for _, lay in parts)
        launches = L * len(parts)
        del devs, outs
        torch.cuda.empty_cache()
        return e0.elapsed_time(e1), step_bytes, launches, clocks.summary()

    parts, _, glay = build_parts(pkg, "box_scale", rank, world)
    barrier()
    ms, step_bytes, launches, clk = timed(parts, 5000 + 31 * rank)
    barrier()
    ms_max = reduce_max(ms)
    bytes_all = float(step_bytes)
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([bytes_all], device=device, dtype=torch.float64)
        dist.all_reduce(t)
        bytes_all = float(t.item())
    value = bytes_all * args.steps / (ms_max / 1e3) / 1e9
    peak, _ = peaks()
    rec = {"workload": "box_scale", "requests": int(glay.batch), "sigma": 0.6, "layers": L,
           "value": round(value, 2), "unit": "GB/s", "ms_per_step": round(ms_max / args.steps, 4),
           "frac_per_gpu": round(value / world / peak, 4), "gpu_launches_per_rank_step": launches,
           "timing": "graph replay, device events, max over ranks", "clocks": clk,
           "plan": "plan_shards: LPT on KV bytes, KV heads of contexts > 2048 split across GPUs"}
    if world == 1:
        rec.update(value_1gpu=rec["value"], efficiency=1.0)
    else:
        v1 = None
        if rank == 0:
            p1, _, _ = build_parts(pkg, "box_scale", 0, 1)
            ms1, b1, _, _ = timed(p1, 7000)
            v1 = b1 * args.steps / (ms1 / 1e3) / 1e9
        barrier()
        if rank == 0:
            rec.update(value_1gpu=round(v1, 2), efficiency=round(value / (world * v1), 4),
                       value_1gpu_source="the whole batch on rank 0's GPU alone, same process, after the N-GPU run")
    return rec


def reference_cpu_path(workload: str):
    """The reference's own Python path (paged_decode_attention_ref + write_kv)
    timed where the reference is importable, on a subsample extrapolated per
    (sequence, head, position): oracle/reference_cpu_path.json, written by
    oracle/time_reference_cpu.py. None when absent."""
    try:
        with open(os.path.join(ROOT, "oracle", "reference_cpu_path.json")) as f:
            rec = json.load(f)
    except (OSError, ValueError):
        return None
    w = rec.get("workloads", {}).get(workload)
    if w is None:
        return None
    return {"value": w["value"], "unit": w["unit"], "layer_calls_per_s": w["layer_calls_per_s"],
            "cores": w["torch_threads"], "kind": "reference", "extrapolated": True,
            "cpu_model": rec.get("cpu_model"), "cpu_count": rec.get("cpu_count"), "when": rec.get("when"),
            "measured_on": "the build host, where the reference is importable (it does not travel to the GPU host)",
            "sample": (f"reference paged_decode_attention_ref + PagedKVCache.write_kv, unmodified, on sequences "
                       f"{w['sample']['sequences']} (contexts {w['sample']['context_lens']}), all heads, one layer: "
                       f"{w['per_seq_head_pos_us']} us per (sequence, head, position), extrapolated to the whole "
                       f"layer-call ({w['extrapolated_layer_call_s']} s)")}


def main():
    args = parse()
    if args.op == "handoff":
        return bench_handoff(args)
    if args.op == "prefill":
        return bench_prefill(args)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    import torch
    import torch.distributed as dist
    from __graft_entry__ import load_package

    pkg = load_package()
    wl = pkg.workloads
    spec = wl.NAMED[args.workload]
    ebytes = {"float32": 4, "bfloat16": 2, "float16": 2}[spec["dtype"]]
    dtype_tag = {"float32": "f32", "bfloat16": "bf16", "float16": "f16"}[spec["dtype"]]
    parts, scaling, glay = build_parts(pkg, args.workload, rank, world)
    abs_ = [wl.algorithmic_bytes(lay, ebytes) for _, lay in parts]
    config = {"workload": args.workload, "batch": glay.batch if scaling == "strong" else glay.batch * world,
              "batch_per_gpu": sum(l.batch for _, l in parts), "ctx_mean": float(glay.context_lens.mean()),
              "heads": [glay.num_heads, glay.num_kv_heads, glay.head_dim], "page": glay.block_size,
              "layers": args.layers,
              "layer_call": ("q/k RMSNorm + rotary + KV append + attention" if args.prep
                             else "KV append + attention"),
              "kv_bytes_per_layer_per_gpu": int(sum(
                  2 * l.num_blocks * l.block_size * l.num_kv_heads * l.head_dim * ebytes for _, l in parts)),
              "l2": f"inputs > L2: {args.layers} rotating per-layer caches",
              "parallelism": f"{world} GPU(s), requests" + (" and long-context KV heads" if scaling == "strong"
                                                            else "") + " partitioned, no collective"}

    if args.impl == "reference":
        if rank != 0:
            return
        name, lay = parts[0]
        on_gpu = torch.cuda.is_available()
        if on_gpu:
            torch.cuda.set_device(local)
        dev = wl.materialize_device(lay, 7, spec["dtype"], spec["scale_values"], 1,
                                    device="cuda" if on_gpu else "cpu")
        host = host_layer(dev, 0)
        del dev
        from oracle import oracle
        oracle.build()
        oracle.use_all_cores()  # torchrun sets OMP_NUM_THREADS=1 for its ranks
        times = []
        for i in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            cpu_layer_call(oracle, host)
            if i >= args.warmup:
                times.append(time.perf_counter() - t0)
        tot = sum(times)
        gbs = abs_[0]["layer_call"] * len(times) / tot / 1e9
        cores = oracle.num_threads()
        sample = (f"one layer-call (append + attention) of the {lay.batch}-sequence '{name}' part per step, "
                  f"C oracle, OpenMP on {cores} host threads")
        print(json.dumps({
            "metric": METRIC, "value": round(gbs, 4), "unit": "GB/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * tot / len(times),
            "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": dtype_tag,
            "data": "synthetic", "config": config, "layer_calls_per_s": len(times) / tot,
            "cpu_baseline": {"value": round(gbs, 4), "unit": "GB/s", "cores": cores, "kind": "port", **host_info(),
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
    devs = [wl.materialize_device(lay, 7 + 31 * rank + i, spec["dtype"], spec["scale_values"], L)
            for i, (_, lay) in enumerate(parts)]
    outs = [[torch.empty_like(d["q"][l]) for l in range(L)] for d in devs]
    if args.prep and args.separate:
        raise SystemExit("--prep runs the fused launch; it does not combine with --separate")
    if args.cascade and (args.prep or args.separate):
        raise SystemExit("--cascade runs the fused append; it does not combine with --prep or --separate")
    plan_ms = 0.0
    if args.cascade:
        for d, (_, lay) in zip(devs, parts):
            pkg.plan_cascade(lay.block_table, lay.context_lens, lay.num_heads, lay.num_kv_heads, device=device)
            t0 = time.perf_counter()  # timed warm: the host cost of planning one step
            d["plan"] = pkg.plan_cascade(lay.block_table, lay.context_lens, lay.num_heads, lay.num_kv_heads,
                                         device=device)
            plan_ms += (time.perf_counter() - t0) * 1e3
    rope = None
    if args.prep:
        # per-layer q_norm / k_norm weights near 1 and the model's rotary table
        # (max_seq_len * 2 rows, as the model registers it)
        D = glay.head_dim
        g = torch.Generator(device=device)
        g.manual_seed(11 + rank)
        for d in devs:
            td = d["q"][0].dtype
            d["q_w"] = [(1 + 0.1 * torch.randn(D, generator=g, device=device)).to(td) for _ in range(L)]
            d["k_w"] = [(1 + 0.1 * torch.randn(D, generator=g, device=device)).to(td) for _ in range(L)]
        rope = pkg.rope_table(D, 2 * 2048, 500000.0, device=device)
    kw = dict(schedule=args.schedule, split_pages=args.split_pages)
    launches_per_call = (2 if args.separate else 1) + (1 if args.schedule == "split" else 0)
    if args.cascade and any(d["plan"].num_work for d in devs):
        one = pkg.cascade.one_launch_possible(glay.num_kv_heads, glay.head_dim) and args.schedule != "split" and \
            (args.prefix_ctas is None or args.prefix_ctas > 0)
        launches_per_call += 1 if one else 2
    calls_per_step = L * len(parts)

    def layer_call(d, l, q, k_new, v_new, block_table, context_lens, out, slots=None, timer=None):
        """One layer-call: the new token's K/V append, then attention (engine.py:213-224)."""
        if args.separate:
            pkg.kv_append(k_new, v_new, d["k_caches"][l], d["v_caches"][l], slots)
        if timer is not None:
            timer[0].record()
        if args.separate:
            pkg.paged_attention(q, d["k_caches"][l], d["v_caches"][l], block_table, context_lens, out=out, **kw)
        elif args.cascade:
            pkg.paged_attention_cascade(q, d["k_caches"][l], d["v_caches"][l], d["plan"], out=out, k_new=k_new,
                                        v_new=v_new, overlap_previous=args.overlap, schedule=args.schedule,
                                        prefix_ctas=args.prefix_ctas)
        elif args.prep:
            pkg.paged_decode_prep_attention(q, k_new, v_new, d["q_w"][l], d["k_w"][l], rope, d["k_caches"][l],
                                            d["v_caches"][l], block_table, context_lens, 1e-6, out=out,
                                            schedule=args.schedule, overlap_previous=args.overlap)
        else:
            # the previous kernel on the stream is another layer-call's attention (or a
            # copy): it writes neither this pool nor the block table / context lengths
            pkg.paged_attention(q, d["k_caches"][l], d["v_caches"][l], block_table, context_lens, out=out,
                                k_new=k_new, v_new=v_new, overlap_previous=args.overlap, **kw)
        if timer is not None:
            timer[1].record()

    def step(timers=None):
        for l in range(L):
            for i, d in enumerate(devs):
                layer_call(d, l, d["q"][l], d["k_new"][l], d["v_new"][l], d["block_table"], d["context_lens"],
                           outs[i][l], d["slot_mapping"], None if timers is None else timers[l * len(devs) + i])

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def reduce(x: float, op) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=op)
        return float(t.item())

    def capture(fn):
        """CUDA graph of fn (run once on a side stream first, as graph capture needs)."""
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
    timers = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(calls_per_step)] for _ in range(args.steps)]
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
    ms_max = reduce(ms, dist.ReduceOp.MAX)
    pkg.check_device_errors(device)

    # ---- dominant kernel: average launch time on its own stream
    bytes_attn = sum(a["attention"] for a in abs_)
    bytes_call = sum(a["layer_call"] for a in abs_)
    if args.prep:  # + the two norm weights and each sequence's rotary table row
        bytes_call += sum(2 * l.head_dim * ebytes + l.batch * l.head_dim * 4 for _, l in parts)
    if graph is None:
        t_ms = [a.elapsed_time(b) for row in timers for (a, b) in row]
        kernel_avg_ms = sum(t_ms) / len(t_ms)
    elif args.prep or args.cascade or (not args.separate and args.schedule != "split"):
        kernel_avg_ms = ms / (args.steps * calls_per_step)  # the step is exactly these launches
    else:
        def attn_only():
            for l in range(L):
                for i, d in enumerate(devs):
                    pkg.paged_attention(d["q"][l], d["k_caches"][l], d["v_caches"][l], d["block_table"],
                                        d["context_lens"], out=outs[i][l], **kw)
        ga = capture(attn_only)
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a0.record()
        for _ in range(args.steps):
            ga.replay()
        a1.record()
        torch.cuda.synchronize()
        kernel_avg_ms = a0.elapsed_time(a1) / (args.steps * calls_per_step)
        del ga
    kernel_bytes = (bytes_attn if args.separate else bytes_call) / len(parts)

    # ---- end to end through the public API with host buffers
    # One pinned staging buffer per part, mirrored on the device: block table,
    # context lengths, then each layer's q / new K / new V rows, so a group of
    # layers' inputs moves in one copy.
    hosts = []
    for d in devs:
        specs = [("bt", d["block_table"]), ("cl", d["context_lens"])]
        for l in range(L):
            specs += [(f"q{l}", d["q"][l]), (f"k{l}", d["k_new"][l]), (f"v{l}", d["v_new"][l])]
        stg = Staging([(name, t.shape, t.dtype) for name, t in specs], device)
        for name, t in specs:
            stg.view(stg.host, name).copy_(t.cpu())
        h = {name: stg.view(stg.host, name) for name, _ in specs}
        dd = {name: stg.view(stg.dev, name) for name, _ in specs}
        h["out"] = torch.empty((L,) + tuple(d["q"][0].shape), dtype=d["q"][0].dtype).pin_memory()
        dd["out"] = torch.empty_like(h["out"], device=device)
        dd["pos"] = torch.empty_like(dd["cl"])
        dd["slots"] = torch.empty(dd["cl"].shape[0], dtype=torch.int64, device=device)
        if args.cascade:  # the step's prefix plan travels with its block table
            h["plan"] = {f: getattr(d["plan"], f).cpu().pin_memory() for f in PLAN_FIELDS}
        hosts.append((h, dd, stg))

    # Copies run on their own streams so they overlap the attention launches;
    # each output leaves for the host as soon as it is written. The launching
    # stream waits for the inputs in growing groups of layers (1, 3, 9, ...):
    # a wait between two layer-calls also ends their programmatic overlap, and
    # a layer's inputs copy about three or more times faster than its attention
    # runs. The step ends when the last output has arrived (the copy streams
    # join the launching stream).
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    groups, l0, n = [], 0, 1
    while l0 < L:
        groups.append((l0, min(L, l0 + n) - 1))
        l0, n = l0 + n, 3 * n
    ev_in = [torch.cuda.Event() for _ in groups]
    ev_out = [torch.cuda.Event() for _ in range(L)]

    def e2e_step():
        main = torch.cuda.current_stream(device)
        s_in.wait_stream(main)
        s_out.wait_stream(main)
        with torch.cuda.stream(s_in):
            if args.cascade:
                for (h, dd, stg), d in zip(hosts, devs):
                    for f in PLAN_FIELDS:
                        getattr(d["plan"], f).copy_(h["plan"][f], non_blocking=True)
            for gi, (a, b) in enumerate(groups):
                for h, dd, stg in hosts:
                    stg.copy_range("bt" if a == 0 else f"q{a}", f"v{b}")
                ev_in[gi].record(s_in)
        for gi, (a, b) in enumerate(groups):
            main.wait_event(ev_in[gi])
            if a == 0 and args.separate:
                for h, dd, stg in hosts:
                    torch.sub(dd["cl"], 1, out=dd["pos"])
                    pkg.slot_mapping(dd["bt"], dd["pos"], glay.block_size, out=dd["slots"])
            for l in range(a, b + 1):
                for (h, dd, stg), d in zip(hosts, devs):
                    layer_call(d, l, dd[f"q{l}"], dd[f"k{l}"], dd[f"v{l}"], dd["bt"], dd["cl"], dd["out"][l],
                               dd["slots"])
                ev_out[l].record(main)
                s_out.wait_event(ev_out[l])
                with torch.cuda.stream(s_out):
                    for h, dd, stg in hosts:
                        h["out"][l].copy_(dd["out"][l], non_blocking=True)
        main.wait_stream(s_in)
        main.wait_stream(s_out)

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
    e2e_ms = reduce(e0.elapsed_time(e1), dist.ReduceOp.MAX)
    # the same end-to-end step launched from Python every step, as the engine's
    # eager decode loop calls the ops (engine.py:157-234): no CUDA graph and no
    # events between launches
    e2e_eager_ms = None
    if eg is not None:
        for _ in range(3):
            e2e_step()
        barrier()
        e0.record()
        for _ in range(args.steps):
            e2e_step()
        e1.record()
        torch.cuda.synchronize()
        barrier()
        e2e_eager_ms = reduce(e0.elapsed_time(e1), dist.ReduceOp.MAX)
    h2d = sum(stg.nbytes for _, _, stg in hosts)
    if args.cascade:
        h2d += sum(t.numel() * t.element_size() for h, _, _ in hosts for t in h["plan"].values())
    d2h = sum(h["out"].numel() * h["out"].element_size() for h, _, _ in hosts)
    for (h, _, _), o in zip(hosts, outs):
        assert all(torch.equal(h["out"][l].to(device), o[l]) for l in range(L)), \
            "end-to-end output differs from the device-resident step"
    del eg

    step_bytes_all = reduce(float(bytes_call * L), dist.ReduceOp.SUM)
    h2d_all, d2h_all = reduce(float(h2d), dist.ReduceOp.SUM), reduce(float(d2h), dist.ReduceOp.SUM)
    calls_all = reduce(float(calls_per_step), dist.ReduceOp.SUM)
    value = step_bytes_all * args.steps / (ms_max / 1e3) / 1e9
    e2e_val = step_bytes_all * args.steps / (e2e_ms / 1e3) / 1e9
    peak, peak_kind = peaks()

    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4), "higher_is_better": True,
        "scaling": scaling, "vs_baseline": None, "dtype": dtype_tag, "data": "synthetic", "config": config,
        "layer_calls_per_s": round(calls_all * args.steps / (ms_max / 1e3), 1),
        "frac_of_hbm_peak": round(value / world / peak, 4),
        "gpu_launches": args.steps * calls_per_step * launches_per_call,
        "e2e": {"value": round(e2e_val, 2), "unit": "GB/s", "h2d_bytes_per_step": int(h2d_all),
                "d2h_bytes_per_step": int(d2h_all), "ms_per_step": round(e2e_ms / args.steps, 4)},
        "clocks": clocks.summary(),
        "graph": bool(graph is not None), "append": "separate launch" if args.separate else "fused",
        "prep": "q/k RMSNorm + rotary fused" if args.prep else None,
        "cascade": ({"groups": sum(len(d["plan"].groups) for d in devs), "plan_host_ms": round(plan_ms, 3),
                     "shared_tokens": sum(d["plan"].shared_tokens for d in devs)} if args.cascade else None),
        "overlap_previous": bool(args.overlap and not args.separate),
    }
    if e2e_eager_ms is not None:
        line["e2e_eager"] = {"value": round(step_bytes_all * args.steps / (e2e_eager_ms / 1e3) / 1e9, 2),
                             "unit": "GB/s", "ms_per_step": round(e2e_eager_ms / args.steps, 4),
                             "vs_e2e": round(e2e_ms / e2e_eager_ms, 4),
                             "launch": "the e2e step launched from Python every step: no CUDA graph, no events "
                                       "between launches (the engine's eager loop)"}
    achieved = kernel_bytes / (kernel_avg_ms / 1e3) / 1e9
    line["roofline"] = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                        "frac": round(achieved / peak, 4), "traffic": profiled_traffic(f"cascade_{args.workload}" if args.cascade
                                                               else f"paged_decode_{args.workload}"),
                        "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                        else "fallback 6650 GB/s",
                        "kernel": ("cascade layer-call: cascade_fused_kernel (suffix pages, KV append fused, and "
                                   "shared-prefix tiles in one launch) + cascade_merge_kernel" if args.cascade else
                                   "paged_decode_mma_kernel" + ("" if args.separate else
                                                                " (q/k RMSNorm, rotary, KV append fused)" if args.prep
                                                                else " (KV append fused)")),
                        "algorithmic_bytes_per_launch": int(kernel_bytes),
                        "avg_launch_us": round(kernel_avg_ms * 1e3, 2),
                        "timing": "per-launch CUDA events" if graph is None else "graph replay / launches"}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import oracle
        oracle.build()
        oracle.use_all_cores()
        host = host_layer(devs[0], 0)
        if args.prep:
            host["prep"] = {"q_w": devs[0]["q_w"][0].cpu(), "k_w": devs[0]["k_w"][0].cpu(), "rope": rope.cpu()}
        calls, t0 = 0, time.perf_counter()
        while True:
            cpu_layer_call(oracle, host)
            calls += 1
            el = time.perf_counter() - t0
            if el >= args.cpu_seconds or calls >= 1000:
                break
        cpu_gbs = abs_[0]["layer_call"] * calls / el / 1e9
        line["cpu_baseline"] = {"value": round(cpu_gbs, 4), "unit": "GB/s", "cores": oracle.num_threads(),
                                "kind": "port", **host_info(),
                                "sample": f"{calls} layer-call(s) ({'norm + rotary + ' if args.prep else ''}"
                                          f"append + attention) of layer 0 of this "
                                          f"workload, C oracle with OpenMP, {el:.1f} s"}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        ref_cpu = reference_cpu_path(args.workload)
        if ref_cpu is not None:
            line["cpu_baseline_ref"] = ref_cpu
    del graph
    if (args.box_scale and args.workload == "decode_760m" and not (args.cascade or args.prep or args.separate)
            and args.graph):
        line["box_scale"] = box_scale_record(args, pkg, rank, world, device,
                                             lambda x: reduce(x, dist.ReduceOp.MAX), barrier)
    if rank == 0:
        print(json.dumps(line))
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

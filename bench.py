"""Benchmark of the V1 query-side selection path on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload decode|single|sort|gather|pages|build|shared|signed]

Workloads (synthetic, seeded; shapes of the benchmark configurations):
  decode  128 requests per GPU, context ~U[32K, 128K] tokens, 64 index heads,
          FP8 e4m3 keys with per-token scales, fixed page budget take=40,
          window 64, route -> FP8 score -> Top-2048 -> gather of the 576-dim
          bf16 MLA latent (single output: K and V are the same latent).
  single  1024 single-head queries over 64 built pages + 65-token tail
          (2688 candidates), route -> score -> Top-2048 (no gather).
Component workloads (one line each): sort (_sort + group offsets), gather
(_gather_slots), pages (page lifecycle), build (index build of 1024 buckets),
shared (published-end shared-tail preparation of a 4096-row chunk), signed
(the signed-score Scorer.select of a 1024-row prefill chunk).
A step is one pass of the whole selection path over one batch.  Three
independent batches (separate pools, same context lengths) are in flight on three
streams, in turn, so the gather of one batch overlaps the selection of the next
(`--inflight 1` runs one batch at a time).  Requests are independent, so N
GPUs run N shares of the job's requests (weak scaling, no collective on the data
path); `value` is the whole-job queries/s = N*B*K / max-over-ranks device time of
the K timed steps.  Rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import statistics
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

METRIC = "indexed queries/sec (route+FP8 score+Top2048+gather); HBM GB/s as % of peak"

# DRAM traffic of one decode gather launch (128 requests x 2048 slots of 1152 B),
# dram__bytes_read.sum + dram__bytes_write.sum from one ncu capture; not
# measured in the run that prints it (the roofline line says so)
GATHER_DECODE_DRAM_BYTES = 303167744 + 250278400
GATHER_DECODE_DRAM_SOURCE = ("ncu dram__bytes_read.sum + dram__bytes_write.sum of one gather_rows_kernel launch "
                             "of this workload, captured separately")


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def workload_cfg(name):
    if name == "decode":
        return dict(B=128, H=64, P=2048, take=40, window=64, topk=2048, lo=32768, hi=131072, latent=576)
    if name == "single":
        return dict(B=1024, H=1, P=128, take=40, window=64, topk=2048, lo=4097, hi=4097, latent=0)
    raise SystemExit(f"unknown workload {name}")


def make_case(synth, cfg, seed, device, rows=None, lens=None):
    B = cfg["B"] if rows is None else rows
    if lens is not None:
        lens = list(lens)[:B]
    elif cfg["lo"] == cfg["hi"]:
        lens = [cfg["lo"]] * B
    else:
        lens = synth.decode_lens(cfg["B"], cfg["lo"], cfg["hi"], seed)[:B]
    return synth.make_query_case(B, cfg["H"], lens, P=cfg["P"], take=cfg["take"], window=cfg["window"],
                                 topk=cfg["topk"], seed=seed, device=device, latent_dim=cfg["latent"])


class Clocks:
    """Sample SM clocks and clock-event (throttle) reasons through NVML in a
    background thread every ~2 ms while the timed region runs."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown"}

    def __init__(self, device: torch.device):
        self.device = device
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = None

    def _handle(self, nv):
        try:
            p = torch.cuda.get_device_properties(self.device)
            bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
            return nv.nvmlDeviceGetHandleByPciBusId_v2(bus)
        except Exception:
            return nv.nvmlDeviceGetHandleByIndex(self.device.index or 0)

    def __enter__(self):
        import threading
        try:
            import pynvml as nv
            nv.nvmlInit()
            h = self._handle(nv)
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
        except Exception:
            return self
        self._stop = threading.Event()

        def loop():
            while True:
                try:
                    self.samples.append(float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)))
                    r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                    for bit, name in self.REASONS.items():
                        if r & bit:
                            self.reasons.add(name)
                except Exception:
                    pass
                if self._stop.wait(0.002):
                    break

        self._thr = threading.Thread(target=loop, daemon=True)
        self._thr.start()
        return self

    def __exit__(self, *exc):
        if self._stop is not None:
            self._stop.set()
            self._thr.join(timeout=2)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def _port_sample(cfg, lens_all, count):
    """`count` request indices spread over the job's batch (a fixed stride), so
    the sample's lengths follow the batch's."""
    n = len(lens_all)
    stride = 37 if n % 37 else 1
    return [(k * stride) % n for k in range(count)]


def _port_case(cfg, n, seed):
    """One request of context n as a numpy case for the oracle port (the latent
    pool is a lazily zeroed array: the gather only copies bytes)."""
    import numpy as np
    import oracle.port as port

    synth = importlib.import_module("10_20_b200.synth")
    case = synth.make_query_case(1, cfg["H"], [n], P=cfg["P"], take=cfg["take"], window=cfg["window"],
                                 topk=cfg["topk"], seed=seed, device="cpu", latent_dim=0)
    c = port.to_numpy_case(case)
    if cfg["latent"]:
        c["latent"] = np.zeros((case.native.shape[0] * 64, 1, cfg["latent"]), np.int16)
    return c


def cpu_port_rate(cfg, lens_all, budget_s=20.0):
    """Queries/s of the oracle port on a bounded CPU sample: one query at a time,
    each request of the sample built with its own pools (untimed), its step
    timed; the sample's requests are spread over the GPU batch's lengths."""
    import oracle.port as port

    torch.set_num_threads(os.cpu_count() or 1)
    port.run_rows(_port_case(cfg, lens_all[0], 999), rows=[0])      # warm-up (page-in, BLAS init)
    timed = 0.0
    done = 0
    sample = []
    for i in _port_sample(cfg, lens_all, len(lens_all)):
        c = _port_case(cfg, lens_all[i], 1000 + i)
        t0 = time.perf_counter()
        port.run_rows(c, rows=[0])
        timed += time.perf_counter() - t0
        done += 1
        sample.append(lens_all[i])
        if timed >= budget_s:
            break
    mean_batch = sum(lens_all) / len(lens_all)
    mean_sample = sum(sample) / len(sample)
    return done / timed, (f"{done} requests of the GPU batch's {len(lens_all)} (mean context {mean_sample:.0f} "
                          f"tokens vs the batch's {mean_batch:.0f}), one query each, oracle port (numpy + BLAS, "
                          f"{torch.get_num_threads()} threads), {timed:.2f} s timed")


def run_reference(args, cfg):
    """The reference arm: the CPU port of the path on the host cores (the
    reference's own route/top-k are CUDA for sm_90 with unvendored headers, and
    its scorer is the external DeepGEMM, so the restatement stands in for it).
    One step = one query of one request of the GPU batch -- the same context
    lengths, taken at a fixed stride -- built with its own pools (untimed);
    the arm reports the rate over the steps it timed."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import oracle.port as port

    torch.set_num_threads(os.cpu_count() or 1)
    lens_all = _request_lens(cfg, 1)
    order = _port_sample(cfg, lens_all, max(args.warmup, 1) + args.steps)
    for k in range(max(args.warmup, 1)):
        port.run_rows(_port_case(cfg, lens_all[order[k]], 1000 + order[k]), rows=[0])
    timed, done, t_start = 0.0, 0, time.perf_counter()
    sample = []
    for k in order[max(args.warmup, 1):]:
        c = _port_case(cfg, lens_all[k], 1000 + k)
        t0 = time.perf_counter()
        port.run_rows(c, rows=[0])
        timed += time.perf_counter() - t0
        done += 1
        sample.append(lens_all[k])
        if time.perf_counter() - t_start > 120.0:
            break
    value = done / timed
    cores = os.cpu_count()
    mean_batch = sum(lens_all) / len(lens_all)
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "queries/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": timed / max(done, 1) * 1e3,
            "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp8-e4m3 keys, f32 scores, bf16 latent", "data": "synthetic",
            "config": {"workload": args.workload, **{k: v for k, v in cfg.items()}},
            "cpu_baseline": {"value": value, "unit": "queries/s", "cores": cores, "kind": "port",
                             "sample": f"{done} of {args.steps} steps timed ({timed:.1f} s): one query of one "
                                       f"request of the GPU batch per step (mean context "
                                       f"{sum(sample) / max(len(sample), 1):.0f} vs the batch's {mean_batch:.0f}), "
                                       f"oracle port (numpy + BLAS, {torch.get_num_threads()} threads)"},
            "e2e": {"value": value, "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# Component workloads (the other rows of the path, each on its own config):
# one JSON line each with the kernel roofline and the oracle timed on the host.
# ---------------------------------------------------------------------------

def _dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
    return world, rank, device, dist


def _timed_replays(graph, steps, warmup, dist, device):
    """Back-to-back replays (every component workload moves far more than L2
    per step); device time of the K timed replays, max over ranks."""
    for _ in range(max(warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(device) as clk:
        a.record()
        for _ in range(steps):
            graph.replay()
        b.record()
        torch.cuda.synchronize()
    ms = a.elapsed_time(b)
    tt = torch.tensor([ms], dtype=torch.float64, device=device)
    if dist:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    return float(tt.item()), clk.summary()


def _capture(fn, device):
    s = torch.cuda.Stream(device=device)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
        fn()
    s.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        fn()
    s.synchronize()
    return g


def _cpu_rate(fn, units_per_call, budget_s=10.0):
    fn()
    done, t0 = 0, time.perf_counter()
    while True:
        fn()
        done += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    return units_per_call * done / el, done, el


def _component_line(args, world, metric, unit, value, steps, ms, clocks, cfg, bytes_per_step, kernel,
                    launches, cpu, parity):
    hbm, kind = peaks()
    achieved = bytes_per_step / (ms / steps / 1e3) / 1e9
    line = {"metric": metric, "value": value, "unit": unit, "n_gpus": world, "steps": steps,
            "warmup": args.warmup, "ms_per_step": ms / steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "data": "synthetic", "config": cfg,
            "roofline": {"bound": "hbm", "kernel": kernel, "achieved": achieved, "peak": hbm, "unit": "GB/s",
                         "frac": achieved / hbm, "peak_kind": kind, "traffic": None},
            "gpu_launches": launches * steps, "clocks": clocks, "parity_spot_check": parity}
    if cpu is not None:
        line["cpu_baseline"] = cpu
    return line


def run_sort_workload(args, world, rank, device, dist):
    """d2: _sort over 256 instances of 16 x 4096 records keyed by group ids with
    ~30% duplicate runs, plus the per-segment group offsets (extension)."""
    import numpy as np
    fg = importlib.import_module("10_20_b200.fused_grouping")
    lib = importlib.import_module("10_20_b200._lib")
    inst = 256
    heads = 16 * inst
    rng = np.random.default_rng(11 + rank)
    keys = rng.integers(0, 4096, size=(heads, 4096))
    run = rng.random((heads, 4096)) < 0.3
    run[:, 0] = False
    idx = np.where(run, 0, np.arange(4096)[None, :])
    idx = np.maximum.accumulate(idx, axis=1)           # forward-fill the runs
    keys = np.take_along_axis(keys, idx, axis=1)
    S = torch.as_tensor(keys.astype(np.float32), device=device)
    P = torch.arange(heads * 4096, dtype=torch.int32, device=device).reshape(heads, 4096)
    out = torch.empty_like(P)
    flag = torch.tensor(-1, dtype=torch.int32, device=device)
    offs = torch.empty((heads, 4097), dtype=torch.int32, device=device)
    stream = lambda: torch.cuda.current_stream(device).cuda_stream

    def step():   # the stable permutation and the group offsets, one launch
        fg.sort_grouped(P, out, S, flag, 4096, heads, 4096, offsets=offs)

    g = _capture(step, device)
    ms, clk = _timed_replays(g, args.steps, args.warmup, dist, device)
    # the reference's published configuration: one grouping level of one head
    # (4096 records in segments of N), one _sort launch, timed in a graph of 20
    one_level = {}
    out1 = torch.empty_like(P[0])                 # its own output: out feeds the parity check
    for n in (1024, 512, 256, 128, 64, 32, 16):
        def level(n=n):
            for _ in range(20):
                fg._sort[(4096 // n, 1)](P[0], out1, S[0], flag, n)
        gl = _capture(level, device)
        ml, _ = _timed_replays(gl, 50, 3, None, device)
        one_level[f"N={n}"] = ml / (50 * 20) * 1e3
    records = heads * 4096
    value = records * args.steps * world / (ms / 1e3)
    bytes_per_step = records * 12 + heads * 4097 * 4
    oracle = importlib.import_module("oracle.v1x_oracle")
    torch.cuda.synchronize()
    k16 = keys[:16].astype(np.float32)
    exp = oracle.sort_segments(np.arange(16 * 4096, dtype=np.int32), k16, -1, 4096, 1, 16).reshape(16, 4096)
    parity = bool(np.array_equal(out[:16].cpu().numpy(), exp))
    eo = [oracle.group_offsets(keys[h][exp[h] - h * 4096], 4096) for h in range(16)]
    parity = parity and bool(np.array_equal(offs[:16].cpu().numpy(), np.stack(eo)))
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        Pn = np.arange(16 * 4096, dtype=np.int32)
        rate, n, el = _cpu_rate(lambda: oracle.sort_segments(Pn, k16, -1, 4096, 1, 16), 16 * 4096)
        cpu = {"value": rate, "unit": "records/s", "cores": 1, "kind": "port",
               "sample": f"{n} calls of one 16 x 4096 instance, oracle sort_segments (numpy lexsort), {el:.1f} s"}
    line = _component_line(args, world, "stable-grouped records/s (_sort + group offsets)", "records/s", value,
                           args.steps, ms, clk,
                           {"workload": "sort", "instances_per_gpu": inst, "records_per_instance": 65536,
                            "segments": "16 x 4096 per instance", "keys": "group ids U[0,4096), ~30% duplicate runs",
                            "bytes_per_step": bytes_per_step}, bytes_per_step, "sort_radix_kernel<512,8,offsets>",
                           1, cpu, parity)
    line["one_level_one_head_us"] = one_level   # _sort[(4096 // N, 1)] on 4096 records, per launch
    return line


def run_gather_workload(args, world, rank, device, dist):
    """d4: _gather_slots of 1024 x 2048 selected slots of the 576-wide bf16 latent
    through GatherWorkspace, K and V from the same latent pool, 2M-token pool under
    a shuffled page table (REQ maps logical -> physical slots)."""
    import numpy as np
    gmod = importlib.import_module("10_20_b200.gather")
    rows, top, D, tokens = 1024, 2048, 576, 1 << 21
    gen = torch.Generator(device=device).manual_seed(21 + rank)
    table = torch.randperm(tokens // 64, generator=gen, device=device).to(torch.int32)
    logical = torch.arange(tokens, device=device, dtype=torch.int32)
    req = (table[logical // 64] * 64 + logical % 64).to(torch.int32)
    ids = torch.randint(0, tokens, (rows, top), generator=gen, device=device, dtype=torch.int32)
    ids[torch.rand((rows, top), generator=gen, device=device) < 0.01] = -1
    lat = torch.randn((tokens, 1, D), generator=gen, device=device, dtype=torch.bfloat16)
    ws = gmod.GatherWorkspace(rows, str(device), torch.bfloat16, dim=D, top=top)
    g_kv = _capture(lambda: ws.gather(lat, lat, req, ids, 0), device)
    ms, clk = _timed_replays(g_kv, args.steps, args.warmup, dist, device)
    g_k = _capture(lambda: ws.gather(lat, None, req, ids, 0), device)
    ms1, _ = _timed_replays(g_k, args.steps, args.warmup, None, device)
    slots = rows * top
    row = D * 2
    bytes_kv = slots * row * 3          # rows read once, K and V written
    bytes_k = slots * row * 2
    value = slots * args.steps * world / (ms / 1e3)
    oracle = importlib.import_module("oracle.v1x_oracle")
    torch.cuda.synchronize()
    # spot check against the oracle on 8 rows: the slots they touch, copied to a
    # compact host pool, with the id -> slot map rewritten to index it
    sample = 8
    ids_s = ids[:sample].cpu().numpy()
    req_n = req.cpu().numpy()
    used = np.unique(ids_s[ids_s >= 0])
    slots_used = req_n[used]
    pool = lat.view(torch.int16).reshape(tokens, D)[torch.as_tensor(slots_used, device=device).long()].cpu().numpy()
    req_small = np.zeros(tokens, np.int32)
    req_small[used] = np.arange(used.size, dtype=np.int32)
    exp_k, exp_v = oracle.gather_slots(pool[:, None, :], pool[:, None, :], req_small, ids_s, sample, top, 0)
    kk = ws.k[:sample].view(torch.int16).reshape(-1, D).cpu().numpy()
    vv = ws.v[:sample].view(torch.int16).reshape(-1, D).cpu().numpy()
    parity = bool(np.array_equal(kk, exp_k) and np.array_equal(vv, exp_v))
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        host_tokens = 1 << 18                            # a 256K-token sample pool on the host
        lat_n = lat.view(torch.int16).reshape(tokens, D)[:host_tokens].cpu().numpy()
        req_h = np.random.default_rng(3).integers(0, host_tokens, size=tokens).astype(np.int32)
        ids_h = np.random.default_rng(4).integers(0, tokens, size=(16, top)).astype(np.int32)
        rate, n, el = _cpu_rate(lambda: (lat_n[req_h[ids_h.reshape(-1)]], lat_n[req_h[ids_h.reshape(-1)]]),
                                16 * top, budget_s=8.0)
        cpu = {"value": rate, "unit": "slots/s", "cores": 1, "kind": "port",
               "sample": f"{n} K+V gathers of 16 x 2048 slots from a 256K-token host pool (numpy indexing), "
                         f"{el:.1f} s"}
    hbm, _ = peaks()
    line = _component_line(args, world, "gathered slots/s (_gather_slots, K+V)", "slots/s", value, args.steps, ms,
                           clk, {"workload": "gather", "rows": rows, "top": top, "dim": D, "dtype": "bf16",
                                 "pool_tokens": tokens, "bytes_per_step_kv": bytes_kv,
                                 "bytes_per_step_k_only": bytes_k}, bytes_kv, "gather_rows_kernel<72,4,true>", 1,
                           cpu, parity)
    line["single_output"] = {"ms_per_step": ms1 / args.steps,
                             "achieved_gbs": bytes_k / (ms1 / args.steps / 1e3) / 1e9,
                             "frac": bytes_k / (ms1 / args.steps / 1e3) / 1e9 / hbm}
    return line


def run_pages_workload(args, world, rank, device, dist):
    """d3: the page lifecycle on a 131,072-page arena: 256 live requests whose
    bucket chains (1-128 buckets, 16-2048 pages) grow by up to 8 buckets per round, half of them
    sharing a prefix of another request's chain, a quarter completing (released)
    after every round; 8 rounds, the first untimed.  Per bucket: fingerprint ->
    match_pages -> allocate -> publish as one captured graph (the reference's
    Build execution)."""
    import numpy as np
    synth = importlib.import_module("10_20_b200.synth")
    lifecycle = importlib.import_module("10_20_b200.lifecycle")
    cap, pages, requests = 131072, 2048, 256
    wl = synth.LifecycleWorkload(requests, 128, 8, 31 + rank, cap // 16, share=0.5, grow=8)
    contents = wl.contents(device)
    # the batched driver reads bucket contents in place from the content pool
    src, bsrc = wl.source(contents), wl.pool_source(contents)

    def run_round(arena, ops, batched):
        """One round of operations; batched: consecutive prepares as one
        prepare_many (v1x_prepare_buckets) and consecutive releases as one
        release_many (v1x_release_many), else per bucket and per lease as the
        reference."""
        prep, rel = [], []
        indexed0 = arena.buckets_indexed

        def flush_prep():
            if prep:
                arena.prepare_many(prep, bsrc)
                prep.clear()

        def flush_rel():
            if rel:
                arena.release_many(rel)
                rel.clear()

        for op in ops:
            if op[0] == "prepare" and batched:
                flush_rel()
                prep.append((op[1], op[2]))
            elif op[0] == "prepare":
                arena.prepare(op[1], op[2], src)
            elif batched:
                flush_prep()
                rel.append(op[1])
            else:
                arena.release(op[1])
        flush_prep()
        flush_rel()
        return arena.buckets_indexed - indexed0


    def timed_rounds(batched):
        arena = lifecycle.PageArena(cap, pages, device, max_requests=requests, graphs=not batched)
        run_round(arena, wl.ops[0], batched)
        arena.check()
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        launches0 = arena.kernel_launches
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        # an NVTX range names the timed launches for profilers (ncu --nvtx-include)
        torch.cuda.nvtx.range_push("lifecycle_batched" if batched else "lifecycle_per_bucket")
        with Clocks(device) as clk:
            t0 = time.perf_counter()
            a.record()
            buckets = sum(run_round(arena, ops, batched) for ops in wl.ops[1:])
            b.record()
            torch.cuda.synchronize()
            wall = time.perf_counter() - t0
        torch.cuda.nvtx.range_pop()
        arena.check()
        ms = a.elapsed_time(b)
        tt = torch.tensor([ms], dtype=torch.float64, device=device)
        if dist:
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        launches = arena.kernel_launches - launches0
        del arena
        return buckets, float(tt.item()), clk, wall, launches

    # the reference-shaped driver first (one captured graph per bucket), as a
    # diagnostic beside the batched driver that gives the line's value
    pb_buckets, pb_ms, _, _, _ = timed_rounds(False)
    buckets, ms, clk, wall, launches = timed_rounds(True)
    assert buckets == pb_buckets
    value = buckets * world / (ms / 1e3)
    # algorithmic bytes per bucket (the O(CAP) hash scan excluded): fingerprint
    # reads 16 pages + members, publish writes them (fresh pages) and moves the
    # bucket's 2 centre pages, release touches 16 refcounts
    per_bucket = 16 * (8448 + 256) + 16 * (8448 + 256 + 16) + 4 * 8448 + 64
    # parity spot check: a small arena through the driver and the CPU port
    port = importlib.import_module("oracle.port")
    small = synth.LifecycleWorkload(12, 6, 3, 5, 4096 // 16, share=0.6, grow=3)
    sc = small.contents(device)
    ca = port.ArenaPort(4096, 128, max_requests=16)
    sg, sb, scpu = small.source(sc), small.pool_source(sc), small.source(tuple(x.cpu().numpy() for x in sc))
    parity = True
    for batched in (False, True):
        ga = lifecycle.PageArena(4096, 128, device, max_requests=16, graphs=True)
        ca = port.ArenaPort(4096, 128, max_requests=16)
        for ops in small.ops:
            prep, rel = [], []
            for op in ops + [("end",)]:
                if op[0] != "prepare" and prep:
                    ga.prepare_many(prep, sb)
                    prep = []
                if op[0] != "release" and rel:
                    ga.release_many(rel)
                    rel = []
                if op[0] == "prepare":
                    ca.prepare(op[1], op[2], scpu)
                    if batched:
                        prep.append((op[1], op[2]))
                    else:
                        ga.prepare(op[1], op[2], sg)
                elif op[0] == "release":
                    ca.release(op[1])
                    if batched:
                        rel.append(op[1])
                    else:
                        ga.release(op[1])
        ga.check()
        parity = parity and all(np.array_equal(getattr(ga, n).cpu().numpy(), getattr(ca, n))
                                for n in ("refs", "free", "tables", "members", "hashes", "fine", "centers"))
        parity = parity and int(ga.free_count.item()) == ca.count
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        # the CPU port on the same 131,072-page arena, first buckets of round 0
        host = tuple(x.cpu().numpy() for x in contents)
        carena = port.ArenaPort(cap, pages, max_requests=requests)
        hsrc = wl.source(host)
        done, t0 = 0, time.perf_counter()
        for op in wl.ops[0]:
            if op[0] != "prepare":
                continue
            before = len(carena.states[op[1]]["leases"]) if op[1] in carena.states else 0
            carena.prepare(op[1], op[2], hsrc)
            done += len(carena.states[op[1]]["leases"]) - before
            if time.perf_counter() - t0 > 10.0:
                break
        el = time.perf_counter() - t0
        cpu = {"value": done / el, "unit": "buckets/s", "cores": 1, "kind": "port",
               "sample": f"{done} buckets of round 0 on the same 131,072-page arena, oracle port (numpy), "
                         f"{el:.1f} s"}
    line = _component_line(args, world, "indexed buckets/s (page lifecycle: fingerprint, match, allocate, "
                           "publish; releases)", "buckets/s", value, 1, ms, clk.summary(),
                           {"workload": "pages", "capacity_pages": cap, "requests": requests,
                            "rounds_timed": len(wl.ops) - 1, "buckets_timed": buckets, "share": 0.5,
                            "bytes_per_bucket": per_bucket,
                            "driver": "prepare_many / release_many: consecutive prepares batched through "
                                      "v1x_prepare_buckets (<= 64 buckets, 5 launches per call, bucket contents read in place "
                                      "from the content pool), consecutive "
                                      "releases through v1x_release_many (1 launch)"},
                           per_bucket * buckets, "confirm_kernel + publish", 5, cpu, parity)
    line["steps"] = len(wl.ops) - 1
    line["ms_per_bucket"] = ms / max(buckets, 1)
    line["stage_tail_shared"] = _stage_tail_shared_diag(device, rank)
    line["per_bucket_driver"] = {"value": pb_buckets * world / (pb_ms / 1e3), "unit": "buckets/s",
                                 "ms_per_bucket": pb_ms / max(pb_buckets, 1),
                                 "how": "PageArena.prepare: one captured graph of the four kernels per bucket "
                                        "(the reference's Build execution)"}
    line["wall_s"] = wall
    line["gpu_launches"] = launches
    return line


def _stage_tail_shared_diag(device, rank):
    """The sink/tail staging of the d3 configuration: 1024 query rows in groups of
    four sharing one request's tail (the owner row stages, the others read its
    copy), as DS/test_page_management_and_tail_small.py:59-88 pairs them, after a
    64K-token history; the reference's launch (grid (B/32, 68), 32 rows per
    program).  Device time per launch from replays of a graph of 20 launches,
    and a bit-exact spot check of a small case against the oracle."""
    import numpy as np
    K = importlib.import_module("10_20_b200.kernels")
    oracle = importlib.import_module("oracle.v1x_oracle")
    B, NP, pool, cap, scratch = 1024, 1026, 32768, 64, 68
    gen = torch.Generator(device=device).manual_seed(61 + rank)
    native = torch.randint(0, 256, (pool, 8448), generator=gen, device=device, dtype=torch.uint8)
    nt = torch.randint(0, pool, (B, NP), generator=gen, device=device, dtype=torch.int32)
    lens = (65536 + torch.arange(B, device=device) % 4).to(torch.int32)
    owners = (torch.arange(B, device=device) // 4 * 4).to(torch.int32)
    fine = torch.zeros((cap + B * scratch, 8448), dtype=torch.uint8, device=device)
    own_each = torch.arange(B, device=device, dtype=torch.int32)   # every row its own tail (no sharing)
    out = {}
    for tag, own, window in (("groups_of_4", owners, 64), ("groups_of_4", owners, 2048),
                             ("every_row_owns", own_each, 2048)):
        def launch(own=own, window=window):
            K.stage_tail_shared[((B + 31) // 32, scratch)](native, native.view(torch.float32), nt, lens, fine,
                                                          fine.view(torch.float32), own, cap, NP, scratch, 64,
                                                          window, ROWS=B, GROUP=32)

        def launch_n():
            for _ in range(20):
                launch()
        g = _capture(launch_n, device)
        ms, _ = _timed_replays(g, 50, 3, None, device)
        us = ms / (50 * 20) * 1e3
        count = 64 + min(window, 65536 - 64)                 # staged tokens per owner (sink + window)
        moved = int((own == torch.arange(B, device=device)).sum()) * -(-count // 64) * 8448 * 2
        out[f"{tag}_window_{window}"] = {"us_per_launch": us, "bytes_moved": moved,
                                         "gb_per_s": moved / (us * 1e-6) / 1e9}
    # spot check: 8 rows (two groups of four) of a small pool against the oracle
    b, np_, pl = 8, 20, 64
    nat_s = torch.randint(0, 256, (pl, 8448), generator=gen, device=device, dtype=torch.uint8)
    nt_s = torch.randint(0, pl, (b, np_), generator=gen, device=device, dtype=torch.int32)
    lens_s = torch.tensor([1100, 1101, 1102, 1103, 1230, 1231, 1232, 1233], dtype=torch.int32, device=device)
    own_s = torch.tensor([0, 0, 0, 0, 4, 4, 4, 4], dtype=torch.int32, device=device)
    fine_s = torch.full((4 + b * scratch, 8448), 7, dtype=torch.uint8, device=device)
    K.stage_tail_shared[((b + 31) // 32, scratch)](nat_s, nat_s.view(torch.float32), nt_s, lens_s, fine_s,
                                                  fine_s.view(torch.float32), own_s, 4, np_, scratch, 64, 64,
                                                  ROWS=b, GROUP=32)
    exp = oracle.stage_tail_shared(nat_s.cpu().numpy(), nt_s.cpu().numpy(), lens_s.cpu().numpy(),
                                   np.full((4 + b * scratch, 8448), 7, np.uint8), own_s.cpu().numpy(), 4, np_,
                                   scratch, 64, 64, b, 32, (b + 31) // 32, scratch)
    out["parity_spot_check"] = bool(np.array_equal(fine_s.cpu().numpy(), exp))
    out["config"] = ("1024 rows after a 64K-token history (+0..3 tokens), sink 64; owners stage sink + tail "
                     "pages (read + write counted); grid (32, 68), 32 rows per program")
    return out


def run_build_workload(args, world, rank, device, dist):
    """Index build (Build.compute's initialize / grouping / assemble): 1024
    buckets per step (16 native pages each, a 138 MB native pool read once per
    step) built in one launch, one 8-CTA cluster per bucket; also the latency of
    a single bucket (the reference's unit of work)."""
    import numpy as np
    ib = importlib.import_module("10_20_b200.index_build")
    oracle = importlib.import_module("oracle.v1x_oracle")
    nb = args.requests or 1024    # buckets per step (--requests: smaller cases for profiling)
    gen = torch.Generator().manual_seed(41 + rank)
    pages = nb * 16
    k = torch.randn((pages, 64, 128), generator=gen).to(torch.float8_e4m3fn)
    host = torch.zeros((pages, 8448), dtype=torch.uint8)
    host[:, :8192] = k.view(torch.uint8).reshape(pages, 8192)
    host.view(torch.float32)[:, 2048:] = torch.rand((pages, 64), generator=gen) + 0.25
    native = host.to(device)
    source = torch.randperm(pages, generator=gen).to(torch.int32).reshape(nb, 16).to(device)
    starts = (torch.arange(nb, dtype=torch.int32) * 1024).to(device)
    builder = ib.BucketBuilder(device, nb)
    g = _capture(lambda: builder.build(native, source, starts), device)
    ms, clk = _timed_replays(g, args.steps, args.warmup, dist, device)
    value = nb * args.steps * world / (ms / 1e3)
    # one bucket at a time (latency), back to back
    one = ib.BucketBuilder(device, 1)
    g1 = _capture(lambda: one.build(native, source[:1], starts[:1]), device)
    ms1, _ = _timed_replays(g1, 200, 5, None, device)
    per_bucket = 16 * 8448 + 16 * 8448 + 2 * 8448 + 1024 * 4 + 1024 * 4
    # parity spot check: four buckets against the oracle
    tmp, centers, mapping, perm = (x.cpu().numpy() for x in builder.build(native, source, starts))
    src_np, pool = source.cpu().numpy(), host.numpy()
    parity = True
    for b in sorted({0, 1, nb // 2, nb - 1}):
        unit, _ = oracle.build_initialize(pool, src_np[b])
        e_perm = oracle.group_bucket(unit)
        e_tmp, e_centers, e_map = oracle.build_assemble(pool, src_np[b], b * 1024, e_perm)
        parity = parity and all(np.array_equal(x, y) for x, y in
                                ((perm[b], e_perm), (tmp[b], e_tmp), (centers[b], e_centers), (mapping[b], e_map)))
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        rate, n, el = _cpu_rate(lambda: oracle.build_bucket(pool, src_np[0], 0), 1)
        cpu = {"value": rate, "unit": "buckets/s", "cores": 1, "kind": "port",
               "sample": f"{n} calls of one bucket, oracle build_bucket (numpy), {el:.1f} s"}
    line = _component_line(args, world, "index-built buckets/s (initialize + 7 grouping levels + assemble)",
                           "buckets/s", value, args.steps, ms, clk,
                           {"workload": "build", "buckets_per_step": nb, "native_pages": pages,
                            "bytes_per_bucket": per_bucket,
                            "l2": f"the {pages * 8448 / 1e6:.0f} MB native pool is read once per step"},
                           per_bucket * nb, "build_bucket_kernel", 1, cpu, parity)
    line["ms_per_bucket_single"] = ms1 / 200
    line["workspace_bytes_per_bucket"] = int(builder.work.numel() // nb)
    return line


def run_shared_workload(args, world, rank, device, dist):
    """Published-end shared-tail preparation (experiments/tail_union_lab_20261021,
    fine_pool_shared_20261021) at the reference's configuration: a 4096-row chunk
    of one request after 65,536 tokens, sink 64, window 2048, published end
    65,536, 40 selected pages per row.  One step = stage_union + tables (the
    reference's `prepare`), captured as a graph; diagnostics: stage_union alone
    for 1024 and 4096 rows, and normalize over the chunk's fine scores."""
    import numpy as np
    ST = importlib.import_module("10_20_b200.shared_tail")
    oracle = importlib.import_module("oracle.v1x_oracle")
    history, rows, sink, window, take = 65536, (args.requests or 4096), 64, 2048, 40
    gen = torch.Generator().manual_seed(51 + rank)
    npg = -(-(history + rows) // 64) + 2
    k = torch.randn((npg, 64, 128), generator=gen).to(torch.float8_e4m3fn)
    host = torch.zeros((npg, 8448), dtype=torch.uint8)
    host[:, :8192] = k.view(torch.uint8).reshape(npg, 8192)
    host.view(torch.float32)[:, 2048:] = torch.rand((npg, 64), generator=gen) + 0.05
    src = host.to(device)
    nt = torch.randperm(npg, generator=gen).to(torch.int32).to(device)
    lens = torch.arange(history + 1, history + rows + 1, dtype=torch.int32, device=device)
    end = torch.tensor([history], dtype=torch.int32, device=device)
    cap = 64
    union_cap = 1 + -(-(history + rows) // 64) - (history - window) // 64 + 2
    fine = torch.zeros((cap + union_cap, 8448), dtype=torch.uint8, device=device)
    meta = torch.zeros((rows, 3), dtype=torch.int32, device=device)
    desc = torch.zeros(4, dtype=torch.int32, device=device)
    c_max = oracle.shared_bounds(history + rows, history, sink, window)[2]
    width = -(-(take * 64 + c_max + 128) // 256) * 256
    fp = width // 64
    takes = torch.full((rows,), take, dtype=torch.int32, device=device)
    selected = ((torch.arange(take, device=device)[None, :] + torch.arange(rows, device=device)[:, None]) % cap).int()
    ft = torch.zeros((rows, fp), dtype=torch.int32, device=device)
    dg = torch.zeros(rows, dtype=torch.int32, device=device)
    cl = torch.zeros(rows, dtype=torch.int32, device=device)
    stage = ST.PreparedStage(src, nt, lens, end, fine[cap:], meta, desc, sink, window)

    def prepare():
        stage()
        ST.tables[(rows,)](lens, end, takes, selected, desc, ft, dg, cl, cap, take, 0, fp, sink, window, fp, True)

    # 20 prepares per captured graph (as the reference's do_bench_cudagraph
    # measures), so a replay's launch cost is spread over them
    per_graph = 20

    def prepare_n():
        for _ in range(per_graph):
            prepare()

    g = _capture(prepare_n, device)
    ms, clk = _timed_replays(g, args.steps, args.warmup, dist, device)
    ms /= per_graph
    value = rows * args.steps * world / (ms / 1e3)
    desc_h = desc.cpu().numpy()
    union_pages = int(desc_h[3])
    bytes_per_step = union_pages * 8448 * 2 + rows * (3 + fp + 2) * 4 + rows * take * 4 + rows * 4
    # diagnostics: the union staging alone (1024 and the full chunk) and normalize
    diag = {}
    for r_sub in sorted({1024, rows}):
        sub = ST.PreparedStage(src, nt, lens[:r_sub], end, fine[cap:], meta[:r_sub], desc, sink, window)

        def sub_n(sub=sub):
            for _ in range(per_graph):
                sub()

        gs = _capture(sub_n, device)
        ms_s, _ = _timed_replays(gs, 50, 5, None, device)
        diag[f"stage_union_us_rows_{r_sub}"] = ms_s / (50 * per_graph) * 1e3
    members = torch.randint(0, history, (cap, 64), generator=gen, dtype=torch.int32).to(device)
    raw = torch.randn((rows, width), generator=gen).to(device)
    norm = torch.empty_like(raw)
    gn = _capture(lambda: ST.normalize[(rows, width // 256)](raw, lens, end, takes, selected, members, norm, take,
                                                             width, width, sink, window, 256, True), device)
    ms_n, _ = _timed_replays(gn, 50, 3, None, device)
    diag["normalize_us"] = ms_n / 50 * 1e3
    # parity spot check: the union, bounds and tables against the oracle
    prepare()
    torch.cuda.synchronize()
    e_dst, e_meta, e_desc = oracle.stage_union(host.numpy(), nt.cpu().numpy(), lens.cpu().numpy(), history,
                                               union_cap, sink, window)
    e_ft, e_dg, e_cl = oracle.shared_tables(lens.cpu().numpy(), history, takes.cpu().numpy(),
                                            selected.cpu().numpy(), e_desc, cap, take, 0, fp, sink, window, True)
    tot = int(e_desc[3])
    parity = bool(np.array_equal(fine[cap:cap + tot].cpu().numpy(), e_dst[:tot])
                  and np.array_equal(meta.cpu().numpy(), e_meta) and np.array_equal(desc_h, e_desc)
                  and np.array_equal(ft.cpu().numpy(), e_ft) and np.array_equal(dg.cpu().numpy(), e_dg)
                  and np.array_equal(cl.cpu().numpy(), e_cl))
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        hn, ntn, ln = host.numpy(), nt.cpu().numpy(), lens.cpu().numpy()
        tk, sl = takes.cpu().numpy(), selected.cpu().numpy()

        def cpu_prepare():
            _, _, dd = oracle.stage_union(hn, ntn, ln, history, union_cap, sink, window)
            oracle.shared_tables(ln, history, tk, sl, dd, cap, take, 0, fp, sink, window, True)

        rate, n, el = _cpu_rate(cpu_prepare, rows)
        cpu = {"value": rate, "unit": "rows/s", "cores": 1, "kind": "port",
               "sample": f"{n} calls of the whole {rows}-row prepare, oracle (numpy), {el:.1f} s"}
    line = _component_line(args, world, "shared-tail prepared rows/s (stage_union + tables)", "rows/s", value,
                           args.steps, ms, clk,
                           {"workload": "shared", "history": history, "rows": rows, "sink": sink, "window": window,
                            "indexed_end": history, "take": take, "union_pages": union_pages, "width": width,
                            "bytes_per_step": bytes_per_step,
                            "l2": "small working set (union 0.8 MB): replays run from L2; latency-bound"},
                           bytes_per_step, "stage_union_kernel + shared_tables_kernel", 2, cpu, parity)
    line["us_per_step"] = ms / args.steps * 1e3
    line["prepares_per_graph"] = per_graph
    line["gpu_launches"] = 2 * per_graph * args.steps
    line["diagnostics"] = diag
    return line


def run_signed_workload(args, world, rank, device, dist):
    """The signed-score path (NA/scoring.py:60-99): one Scorer.select in v1 mode
    over one KV head for a 1024-row prefill chunk after 122,880 tokens of
    history indexed in 4096-token buckets (1,856 built pages, fraction 0.5 ->
    928 routed pages, 49 fixed pages of sink + window + chunk; 62,528 fine
    candidates per row), four query heads padded to 32.  One step = pack_q,
    the signed centre logits, the route, the signed fine logits, mask_scores
    and the mapped Top-2048, captured as a graph.  Bytes per step are the
    designed traffic of that composition (the reference's): both pools once,
    the centre and fine logit matrices written and read once, q in, ids out."""
    import math
    import numpy as np
    NS = importlib.import_module("10_20_b200.native_scoring")
    oracle = importlib.import_module("oracle.v1x_oracle")
    rows = args.requests or 1024
    prefix, sink, window, bucket = 122880, 64, 2048, 4096
    pages = (prefix - sink - window) // bucket * 64
    fixed_n = math.ceil((sink + window + rows) / 64)
    fp = pages + fixed_n
    C = pages * 8
    cp = (C + 63) // 64
    gen = torch.Generator().manual_seed(61 + rank)

    def pool(n):
        k = torch.randn((n, 64, 128), generator=gen).to(torch.float8_e4m3fn)
        buf = torch.zeros((n, 8448), dtype=torch.uint8)
        buf[:, :8192] = k.view(torch.uint8).reshape(n, 8192)
        buf.view(torch.float32)[:, 2048:] = torch.rand((n, 64), generator=gen) * 0.5 + 0.05
        return buf.reshape(n, 64, 1, 132)

    class State:
        pass

    st = State()
    st.pages = pages
    centers_h, fine_h = pool(cp), pool(fp)
    st.centers, st.fine = centers_h[None].to(device), fine_h[None].to(device)
    valid_h = torch.rand((1, C), generator=gen) > 0.02
    st.valid = valid_h.to(device)
    # middle pages hold history tokens [sink, prefix - window) in a shuffled order
    # (buckets are reordered by grouping); fixed pages: sink, window, the chunk
    mid = torch.randperm(prefix - window - sink, generator=gen)[:pages * 64].int() + sink
    tail = torch.cat((torch.arange(sink), torch.arange(prefix - window, prefix + rows))).int()
    tail = torch.cat((tail, torch.full((fixed_n * 64 - tail.numel(),), -1, dtype=torch.int32)))
    mapping_h = torch.cat((mid, tail))[None].contiguous()
    st.mapping = mapping_h.to(device)
    fixed = torch.arange(pages, fp, dtype=torch.int32, device=device)

    class Cfg:
        mode, share_active_pages, fraction = "v1", False, 0.5

        def budget(self, n):
            return min(n, math.ceil(n * self.fraction))

    scorer = NS.Scorer(Cfg(), device)
    q = torch.randn((rows, 4, 128), generator=gen).to(torch.bfloat16).to(device)
    take = Cfg().budget(pages)
    W = (take + fixed_n) * 64
    out = {}

    def step():
        out["ids"] = scorer.select(q, st, 0, prefix, 0, 0, fixed, 0.0883883)

    g = _capture(step, device)
    ms, clk = _timed_replays(g, args.steps, args.warmup, dist, device)
    value = rows * args.steps * world / (ms / 1e3)
    bytes_per_step = (cp + fp) * 8448 + rows * (C * 4 * 2 + W * 4 * 2 + 4 * 128 * 2 + 2048 * 4)
    # stage split of one select (eager, events between the operators)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(8)]
    ct = torch.arange(cp, device=device, dtype=torch.int32)
    table = torch.empty((rows, take + fixed_n), device=device, dtype=torch.int32)
    table[:, take:] = fixed[None]
    positions = torch.arange(prefix, prefix + rows, device=device, dtype=torch.int32)
    used = torch.cat((torch.arange(min(2048, fp), device=device, dtype=torch.int32), fixed))
    split = {}
    for rep in range(4):
        ev[0].record()
        qp = scorer._pack(q, 0.0883883)
        ev[1].record()
        coarse = scorer._logits(qp, st.centers[0], ct, C, key_valid=st.valid[0, :C])
        ev[2].record()
        NS.extension(64, 4).route(coarse, table, pages, take)
        ev[3].record()
        sc = scorer._logits(qp, st.fine[0], used, used.numel() * 64, table, mask=(st.mapping[0], positions))
        ev[4].record()
        NS.mapped_top2048(sc, table, st.mapping[0])
        ev[5].record()
        torch.cuda.synchronize()
        if rep:
            for i, name in enumerate(("pack_q", "centre_logits", "route", "fine_logits", "mapped_top2048")):
                split.setdefault(name, []).append(ev[i].elapsed_time(ev[i + 1]) * 1e3)
    split = {k: statistics.median(v) for k, v in split.items()}
    # the dsa mode (flat keys, causal windows) over the same history and rows
    st.flat_k = torch.randn((1, prefix, 128), generator=gen).to(torch.float8_e4m3fn).to(device)
    st.flat_scale = (torch.rand((1, prefix), generator=gen) * 0.5 + 0.05).to(device)
    dsa = NS.Scorer(type("DsaCfg", (Cfg,), {"mode": "dsa"})(), device)
    gd = _capture(lambda: out.__setitem__("dsa", dsa.select(q, st, 0, prefix - rows, 0, prefix, fixed, 0.0883883)),
                  device)
    ms_d, _ = _timed_replays(gd, 10, 3, None, device)
    split["dsa_select"] = ms_d / 10 * 1e3
    del gd, st.flat_k, st.flat_scale
    # the grouped scorer's MMAs: every key of the used pages against 32 rows x 4 heads per group
    fine_flop = 2.0 * (-(-rows // 32)) * used.numel() * 64 * 128 * 128
    split["fine_logits_mma_tflops"] = fine_flop / (split["fine_logits"] * 1e-6) / 1e12
    del coarse, sc
    # parity spot check: two rows through the fixed-order scorer against the oracle's composition
    parity = None
    if not args.no_parity:
        scorer.impl = "simt"
        got = scorer.select(q[:2], st, 0, prefix, 0, 0, fixed, 0.0883883).cpu().numpy()
        scorer.impl = "auto"
        q8o, wo = oracle.pack_q(q[:2].float().cpu().numpy(), 32, np.float32(0.0883883 / 4))
        co = oracle.score_paged(q8o, wo, centers_h.numpy(), np.arange(cp)[None].repeat(2, 0), [C] * 2, C,
                                relu=False)
        co[:, ~valid_h[0].numpy()] = -np.inf
        sel, _ = oracle.page_route(co, pages, take)
        tb = np.concatenate([sel, np.arange(pages, fp)[None].repeat(2, 0)], 1).astype(np.int32)
        fo = oracle.score_paged(q8o, wo, fine_h.numpy(), tb, [W] * 2, W, relu=False)
        fo = oracle.mask_scores(fo, tb, mapping_h[0].numpy().reshape(-1, 64), np.arange(prefix, prefix + 2))
        want, _ = oracle.topk_transform(fo, [W] * 2, tb, 64, 2048, original_ids=mapping_h[0].numpy())
        parity = {"rows": 2, "scorer": "simt (fixed order)", "bit_exact": bool(np.array_equal(got, want)),
                  "ids_differing": int((got != want).sum())}
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        q8o, wo = oracle.pack_q(q[:1].float().cpu().numpy(), 32, np.float32(0.0883883 / 4))
        ch, fh, mh = centers_h.numpy(), fine_h.numpy(), mapping_h[0].numpy()

        def cpu_row():
            co = oracle.score_paged(q8o, wo, ch, np.arange(cp)[None], [C], C, relu=False, exact=False)
            co[:, ~valid_h[0].numpy()] = -np.inf
            sel, _ = oracle.page_route(co, pages, take)
            tb = np.concatenate([sel, np.arange(pages, fp)[None]], 1).astype(np.int32)
            fo = oracle.score_paged(q8o, wo, fh, tb, [W], W, relu=False, exact=False)
            fo = oracle.mask_scores(fo, tb, mh.reshape(-1, 64), [prefix])
            oracle.topk_transform(fo, [W], tb, 64, 2048, original_ids=mh)

        rate, n, el = _cpu_rate(cpu_row, 1)
        cpu = {"value": rate, "unit": "rows/s", "cores": torch.get_num_threads(), "kind": "port",
               "sample": f"{n} single-row selects of this workload, oracle (numpy, BLAS logits), {el:.1f} s"}
    line = _component_line(args, world, "signed-score selected rows/s (Scorer.select, v1 mode)", "rows/s", value,
                           args.steps, ms, clk,
                           {"workload": "signed", "rows": rows, "prefix": prefix, "built_pages": pages,
                            "take": take, "fixed_pages": fixed_n, "fine_candidates": W, "q_heads": 4,
                            "scorer": "grouped tensor cores: 32 rows x 4 heads per MMA operand",
                            "bytes_per_step": bytes_per_step,
                            "l2": "the logit matrices (61 + 256 MB) exceed L2 every step"},
                           bytes_per_step, "score_tc_kernel (fine logits)", 6, cpu, parity)
    line["us_per_step"] = ms / args.steps * 1e3
    line["stage_us"] = split
    return line


def run_component(args):
    world, rank, device, dist = _dist_setup()
    importlib.import_module("10_20_b200").load()
    if args.workload == "sort":
        line = run_sort_workload(args, world, rank, device, dist)
    elif args.workload == "gather":
        line = run_gather_workload(args, world, rank, device, dist)
    elif args.workload == "build":
        line = run_build_workload(args, world, rank, device, dist)
    elif args.workload == "shared":
        line = run_shared_workload(args, world, rank, device, dist)
    elif args.workload == "signed":
        line = run_signed_workload(args, world, rank, device, dist)
    else:
        line = run_pages_workload(args, world, rank, device, dist)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()
    return 0


def _request_lens(cfg, world):
    """The job's context lengths: world * B requests from the benchmark seed."""
    synth = importlib.import_module("10_20_b200.synth")
    if cfg["lo"] == cfg["hi"]:
        return [cfg["lo"]] * (world * cfg["B"])
    return synth.decode_lens(world * cfg["B"], cfg["lo"], cfg["hi"], 1000)


def _shard(cfg, lens_all, world, rank, per_rank):
    """This rank's share of the job's requests (longest first by bytes)."""
    if world == 1:
        return list(lens_all)
    sharding = importlib.import_module("10_20_b200.sharding")
    row = cfg["latent"] * 2
    costs = [sharding.row_bytes(n, cfg["H"], cfg["take"], cfg["window"], cfg["topk"], row)["total"]
             for n in lens_all]
    return [lens_all[i] for i in sharding.shard_requests(costs, world, per_rank=per_rank)[rank]]


class Batches:
    """`inflight` independent batches of the same request lengths (each its own
    seeded pools, tables and queries), each step captured as one CUDA graph on
    its own stream; steps alternate over the batches, so the gather of one
    overlaps the selection of the next and consecutive steps touch disjoint
    data.  Events on the caller's stream bracket a run."""

    def __init__(self, cfg, lens, seed, inflight, device, score_ctas=0):
        synth = importlib.import_module("10_20_b200.synth")
        pipeline = importlib.import_module("10_20_b200.pipeline")
        self.device = device
        self.sets = []
        for i in range(inflight):
            case = make_case(synth, dict(cfg, B=len(lens)), seed + 7919 * i, device, lens=lens)
            step = pipeline.SelectionStep(case, gather=cfg["latent"] > 0, score_ctas=score_ctas)
            st = torch.cuda.Stream(device=device)
            st.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(st):
                for _ in range(2):
                    step.run()
            st.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=st):
                step.run()
            st.synchronize()
            self.sets.append(dict(case=case, step=step, stream=st, graph=g))
        for st in self.sets:   # pinned host copies of the step's inputs and output
            c = st["case"]
            st["pin"] = [(c.q8.view(torch.uint8), c.q8.view(torch.uint8).cpu().pin_memory()),
                         (c.w, c.w.cpu().pin_memory()), (c.lens, c.lens.cpu().pin_memory()),
                         (c.native_table, c.native_table.cpu().pin_memory())]
            st["out_host"] = torch.empty(st["step"].physical.shape, dtype=torch.int32).pin_memory()
        self.h2d = sum(h.numel() * h.element_size() for _, h in self.sets[0]["pin"])
        self.d2h = self.sets[0]["out_host"].numel() * 4

    def run(self, n, e2e=False):
        main = torch.cuda.current_stream(self.device)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(main)
        for st in self.sets:
            st["stream"].wait_stream(main)
        for k in range(n):
            st = self.sets[k % len(self.sets)]
            with torch.cuda.stream(st["stream"]):
                if e2e:     # host -> device inputs of this step, from pinned memory
                    for dst, hst in st["pin"]:
                        dst.copy_(hst, non_blocking=True)
                st["graph"].replay()
                if e2e:     # device -> host: the step's physical slot ids
                    st["out_host"].copy_(st["step"].physical, non_blocking=True)
        for st in self.sets:
            main.wait_stream(st["stream"])
        b.record(main)
        return a, b

    def release(self):
        for st in self.sets:
            st.pop("graph", None)


def _timed(fn, dist, device, clocks=False):
    """Barrier, then time fn() (which returns an event pair); max over ranks."""
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clk = Clocks(device) if clocks else None
    if clk:
        clk.__enter__()
    t0 = time.perf_counter()
    a, b = fn()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    if clk:
        clk.__exit__()
    ms = a.elapsed_time(b)
    t = torch.tensor([ms], dtype=torch.float64, device=device)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item()), wall, (clk.summary() if clk else None)


def _stage_split(step, reps=5):
    """Per-stage device time (us) of one batch run eagerly with events between
    its launches, after a 256 MB L2-evicting read; mean over reps."""
    flush = torch.ones(256 << 20, dtype=torch.uint8, device=step.case.lens.device)
    acc = {}
    for _ in range(reps):
        flush.sum()
        marks = []
        step.run(marks=marks)
        torch.cuda.synchronize()
        for (_, a), (name, b) in zip(marks, marks[1:]):
            acc[name] = acc.get(name, 0.0) + a.elapsed_time(b) * 1e3 / reps
    return {k: round(v, 2) for k, v in acc.items()}


def _indexer_e2e(cases, cfg, steps, warmup, device, dist):
    """End to end through the reference-facing API: per step, pinned host ->
    device copies of q, weights, native page tables and lengths, then
    Indexer.query (runtime.py:828-907; the fixed page budget installed as the
    reference's benchmark does, qwen_gqa_probe_backend.py:48) and
    GatherWorkspace.gather of the returned slots (NA/kernels.py:102-111), and a
    device -> host copy of the slot ids.  One Indexer per independent batch
    (its own native cache and arena), each on its own stream; steps alternate
    over them as the headline's batches in flight do, so one batch's copies and
    gather overlap another's selection.  Returns (ms for `steps` steps, h2d
    bytes, d2h bytes)."""
    pkg = "10_20_b200"
    Config = importlib.import_module(pkg + ".config").Config
    Indexer = importlib.import_module(pkg + ".indexer").Indexer
    K = importlib.import_module(pkg + ".kernels")
    gmod = importlib.import_module(pkg + ".gather")
    c0 = cases[0]
    B = c0.B
    qb = tuple(sorted({1, 4, 16, 64, B}))
    conf = Config(max_context=c0.P * 64, heads=c0.H, max_requests=B, topk=c0.topk,
                  page_fraction=c0.take / c0.topk, window=c0.window, q_buckets=qb, budget_bytes=1 << 40)
    saved = K.query_metadata
    K.query_metadata = K.BudgetMetadata(torch.tensor([c0.take], dtype=torch.int32, device=device))
    def packed(case):
        """The step's inputs packed in one pinned host buffer (one host -> device
        copy per step) and typed views of its device twin: q, weights, native
        tables, lengths at 256-byte aligned offsets."""
        parts = [case.q8.view(torch.uint8), case.w, case.native_table, case.lens]
        offs, total = [], 0
        for t in parts:
            offs.append(total)
            total += (t.numel() * t.element_size() + 255) // 256 * 256
        host = torch.empty(total, dtype=torch.uint8).pin_memory()
        dev = torch.empty(total, dtype=torch.uint8, device=device)
        views = []
        for t, o in zip(parts, offs):
            n = t.numel() * t.element_size()
            host[o:o + n].copy_(t.contiguous().view(torch.uint8).reshape(-1).cpu())
            views.append(dev[o:o + n].view(t.dtype).view(t.shape))
        views[0] = views[0].view(torch.float8_e4m3fn)
        return host, dev, views, sum(t.numel() * t.element_size() for t in parts)

    sets = []
    try:
        for case in cases:
            host, dev, views, nbytes = packed(case)
            st = {"case": case, "ix": Indexer(case.native, conf), "lens": case.lens.cpu().tolist(),
                  "stream": torch.cuda.Stream(device=device), "host": host, "dev": dev, "views": views,
                  "h2d": nbytes, "out_host": torch.empty((B, case.topk), dtype=torch.int32).pin_memory(),
                  "ws": gmod.GatherWorkspace(B, device, case.latent.dtype, dim=case.latent.shape[-1],
                                             top=case.topk)}
            sets.append(st)
        owners = list(range(B))

        def one(k):
            st = sets[k % len(sets)]
            with torch.cuda.stream(st["stream"]):
                st["dev"].copy_(st["host"], non_blocking=True)
                q, w, nt, ln = st["views"]
                ids = st["ix"].query(q, w, nt, ln, owners, st["lens"])
                st["ws"].gather(st["case"].latent, None, None, ids, 0)
                st["out_host"].copy_(ids, non_blocking=True)

        for k in range(len(sets)):  # builds every request's index (prepare), captures the query graphs
            one(k)
        torch.cuda.synchronize()
        for k in range(max(warmup, 3) * len(sets)):
            one(k)

        issue = []

        def run():
            main = torch.cuda.current_stream(device)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(main)
            for st in sets:
                st["stream"].wait_stream(main)
            t0 = time.perf_counter()
            for k in range(steps):
                one(k)
            issue.append(time.perf_counter() - t0)
            for st in sets:
                main.wait_stream(st["stream"])
            b.record(main)
            return a, b
        ms, _, _ = _timed(run, dist, device)
        return ms, sets[0]["h2d"], sets[0]["out_host"].numel() * 4, issue[0] / steps * 1e6
    finally:
        for st in sets:
            st["ix"].close()
        K.query_metadata = saved


def run_decode(args, cfg):
    world, rank, device, dist = _dist_setup()
    importlib.import_module("10_20_b200").load()
    B = cfg["B"]
    inflight = max(1, args.inflight)
    lens_all = _request_lens(cfg, world)
    lens = _shard(cfg, lens_all, world, rank, B)
    # with batches in flight the centre scorer takes one CTA per SM (it leaves
    # room for the other batches' kernels); one batch alone keeps two per SM
    n_sms = torch.cuda.get_device_properties(device).multi_processor_count
    score_ctas = args.score_ctas if args.score_ctas >= 0 else (n_sms if inflight > 1 else 0)
    bat = Batches(cfg, lens, 1000 + rank, inflight, device, score_ctas=score_ctas)
    case, step = bat.sets[0]["case"], bat.sets[0]["step"]
    acct = step.algorithmic_bytes()
    gather_on = step.gather

    # ---- the headline: K steps, three batches in flight ----------------------------
    for _ in range(max(args.warmup, 3)):
        bat.run(inflight)
    # an NVTX range names the timed launches for profilers (ncu --nvtx-include)
    torch.cuda.nvtx.range_push("decode_steps")
    total_ms, wall, clocks = _timed(lambda: bat.run(args.steps), dist, device, clocks=True)
    torch.cuda.nvtx.range_pop()
    queries = B * args.steps * world
    value = queries / (total_ms / 1e3)

    # ---- diagnostics of one batch ---------------------------------------------------
    s = bat.sets[0]["stream"]

    def capture(fn):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            fn()
        s.synchronize()
        return g

    # one batch alone: the default grid (two CTAs per SM)
    step.score_ctas = 0
    one_graph = capture(step.run)
    step.gather = False
    sel_graph = capture(step.run)
    step.gather = gather_on
    gat_graph = None
    if gather_on:
        gmod = importlib.import_module("10_20_b200.gather")
        lat = case.latent
        gat_graph = capture(lambda: gmod._gather_impl((1,), lat, None, None, step.physical, step.kv, None, B,
                                                      case.topk, 0, *lat.stride(), 0, 0, 0,
                                                      step.physical.stride(0)))
    flush = torch.ones(256 << 20, dtype=torch.uint8, device=device)

    def timed_each(graph, n, flush_first=True):
        evs = []
        for _ in range(n):
            if flush_first:
                flush.sum()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            graph.replay()
            b.record()
            evs.append((a, b))
        torch.cuda.synchronize()
        return [a.elapsed_time(b) for a, b in evs]

    diag_steps = min(args.steps, 20)
    one_ms = timed_each(one_graph, diag_steps)
    sel_ms = timed_each(sel_graph, diag_steps)
    # the gather kernel alone, replayed back to back: its 604 MB per launch is far
    # larger than L2, and its own write-backs stay in the timing
    gather_ms = timed_each(gat_graph, diag_steps + 1, flush_first=False)[1:] if gat_graph is not None else [0.0]
    split = _stage_split(step)

    # ---- end to end -----------------------------------------------------------------
    bat.run(2 * inflight, e2e=True)
    e2e_ms, _, _ = _timed(lambda: bat.run(args.steps, e2e=True), dist, device)
    e2e_graph_value = queries / (e2e_ms / 1e3)
    api = None
    if gather_on and args.workload == "decode":
        api_steps = min(args.steps, 200)
        api_ms, api_h2d, api_d2h, host_us = _indexer_e2e([st["case"] for st in bat.sets], cfg, api_steps,
                                                           args.warmup, device, dist)
        api = {"value": B * api_steps * world / (api_ms / 1e3), "unit": "queries/s", "h2d_bytes_per_step": api_h2d,
               "d2h_bytes_per_step": api_d2h, "steps": api_steps, "ms_per_step": api_ms / api_steps,
               "host_us_per_step": host_us}

    # ---- strong scaling: ONE job of B requests split across the ranks ---------------
    strong = None
    if world > 1 and B % world == 0:
        bs = B // world
        # the N = 1 batch's requests (the benchmark's 128), split by bytes
        lens_s = _shard(cfg, _request_lens(cfg, 1), world, rank, bs)
        strong = {"job_requests": B, "requests_per_gpu": bs, "unit": "queries/s"}
        # the headline's depth of batches in flight, then a depth that keeps as
        # many rows in flight per GPU as one GPU holds with the whole job
        n_sm = torch.cuda.get_device_properties(device).multi_processor_count
        for depth in (inflight, min(inflight * world, 24)):
            # the deep pipeline's centre scorer takes about its batch's share of
            # the SMs (many small batches on separate streams): grid capped at
            # 2 * SMs / depth, at least 16 CTAs
            ctas = 0 if depth == inflight else max(16, 2 * n_sm // depth)
            sb = Batches(dict(cfg, B=bs), lens_s, 2000 + rank, depth, device, score_ctas=ctas)
            for _ in range(max(args.warmup, 3)):
                sb.run(depth)
            sms, _, _ = _timed(lambda: sb.run(args.steps), dist, device)
            entry = {"batches_in_flight": depth, "value": B * args.steps / (sms / 1e3),
                     "ms_per_step": sms / args.steps, "score_ctas": ctas or None}
            if depth == inflight:
                strong.update(entry)
                split = strong["single_batch_stage_us"] = _stage_split(sb.sets[0]["step"])
            else:
                strong["rows_in_flight_as_one_gpu"] = entry
            sb.release()
            del sb
            torch.cuda.empty_cache()
        strong["limiter"] = (
            f"the row latency of select_fused (one CTA per row, {split.get('select', 0):.0f} us for a batch of "
            f"{bs} rows, as for 128): with {inflight} batches in flight only {bs * inflight} rows are selected "
            f"at once on 148 SMs, so the step is latency-bound; a deeper pipeline restores the rows in flight "
            f"(its centre scorer's grid capped to the batch's share of the SMs)")

    # ---- parity spot check (rank 0): sampled rows of batch 0 against the oracle -----
    parity = None
    if rank == 0 and not args.no_parity:
        SC = importlib.import_module("oracle.selection_check")
        bat.sets[0]["graph"].replay()
        torch.cuda.synchronize()
        ln = case.lens.cpu().numpy()
        order = ln.argsort(kind="stable")
        rows = sorted({int(order[0]), int(order[-1]), int(order[len(order) // 2]), 1 % B})
        t0 = time.perf_counter()
        parity = SC.check_rows(step, case, rows)
        parity["seconds"] = round(time.perf_counter() - t0, 1)

    if rank == 0:
        hbm, kind = peaks()
        if gather_on:
            dom_bytes, dom_ms, dom = acct["gather"], statistics.mean(gather_ms), "gather_rows_kernel"
        else:
            dom_bytes, dom_ms, dom = acct["total"], statistics.mean(sel_ms), "selection graph"
        achieved = dom_bytes / (dom_ms / 1e3) / 1e9
        traffic = traffic_src = None
        if gather_on and args.workload == "decode" and B == 128:
            # DRAM bytes of one decode gather launch (128 requests x 2048 slots of 1152 B)
            traffic = GATHER_DECODE_DRAM_BYTES
            traffic_src = GATHER_DECODE_DRAM_SOURCE
        one_batch = statistics.mean(one_ms)
        line = {
            "metric": METRIC, "value": value, "unit": "queries/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp8-e4m3 keys, f32 scores, bf16 latent",
            "data": "synthetic",
            "config": {"workload": args.workload, "requests_per_gpu": B, "heads": case.H,
                       "page_budget": case.take, "topk": case.topk, "window": case.window,
                       "context": [cfg["lo"], cfg["hi"]], "latent_dim": cfg["latent"],
                       "parallelism": f"requests sharded by bytes (longest first), {world} ranks x "
                                      f"{B} requests, no data-path collective",
                       "batches_in_flight": inflight,
                       "centre_scorer_ctas": score_ctas or "two per SM (one batch alone: always)",
                       "l2": "inputs larger than L2: consecutive steps alternate between independent batches "
                             "(separate pools, ~12 GB each); single-batch diagnostics after a 256 MB read",
                       "algorithmic_bytes_per_step": acct["total"]},
            "step_hbm_gbs": acct["total"] / (total_ms / args.steps / 1e3) / 1e9,
            "step_frac_of_peak": acct["total"] / (total_ms / args.steps / 1e3) / 1e9 / hbm,
            "single_batch": {"ms": one_batch, "hbm_gbs": acct["total"] / (one_batch / 1e3) / 1e9,
                             "frac_of_peak": acct["total"] / (one_batch / 1e3) / 1e9 / hbm},
            "roofline": {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": hbm, "unit": "GB/s",
                         "frac": achieved / hbm, "peak_kind": kind, "traffic": traffic,
                         "traffic_source": traffic_src},
            "stage_ms": {"step": total_ms / args.steps, "single_batch_latency": one_batch,
                         "selection_alone": statistics.mean(sel_ms), "gather_alone": statistics.mean(gather_ms)},
            "stage_us_one_batch": split,
            "e2e": api if api is not None else
                   {"value": e2e_graph_value, "unit": "queries/s", "h2d_bytes_per_step": bat.h2d,
                    "d2h_bytes_per_step": bat.d2h},
            "e2e_step_graphs": {"value": e2e_graph_value, "unit": "queries/s", "h2d_bytes_per_step": bat.h2d,
                                "d2h_bytes_per_step": bat.d2h,
                                "how": "SelectionStep graph replays, batches in flight, pinned copies per step"},
            "gpu_launches": step.launches() * args.steps,
            "clocks": clocks,
            "wall_s": wall,
        }
        if api is not None:
            line["e2e"]["how"] = (f"Indexer.query + GatherWorkspace.gather per step, {inflight} batches in flight "
                                  "(one Indexer and stream each): one pinned H2D copy of the packed q, weights, "
                                  "native tables and lengths; D2H of the slot ids; host_us_per_step = the host's "
                                  "issue time per step")
        if strong is not None:
            line["strong_scaling"] = strong
        if parity is not None:
            line["parity"] = parity
        if world == 1 and not args.no_cpu_baseline:
            v, meta = cpu_port_rate(cfg, lens_all, budget_s=15.0)
            line["cpu_baseline"] = {"value": v, "unit": "queries/s", "cores": os.cpu_count(), "kind": "port",
                                    "sample": meta}
        print(json.dumps(line), flush=True)
    if dist:
        bat.release()
        del sel_graph, gat_graph
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000,
                    help="timed steps (the default times ~0.3 s, enough for the NVML clock samples)")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--requests", type=int, default=0,
                    help="override the per-GPU batch (small cases for profiling; not a bench config)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="decode",
                    choices=["decode", "single", "sort", "gather", "pages", "build", "shared", "signed"],
                    help="decode (the headline), single (1024 single-head queries), sort (_sort, 256 x 65,536 "
                         "records), gather (_gather_slots, 1024 x 2048 slots of 576 bf16), pages (page "
                         "lifecycle), build (index build, 1024 buckets per step), shared (published-end "
                         "shared-tail preparation, 4096-row chunk), signed (the signed-score Scorer.select of "
                         "a 1024-row chunk)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true", help="skip the oracle spot check of sampled rows")
    ap.add_argument("--inflight", type=int, default=3,
                    help="independent batches in flight (the gather of one overlaps the selection of the next)")
    ap.add_argument("--score-ctas", type=int, default=-1,
                    help="cap of the centre scorer's persistent grid with batches in flight (0: two CTAs per SM; "
                         "-1: one CTA per SM when more than one batch is in flight, else 0)")
    args = ap.parse_args()
    if args.workload in ("sort", "gather", "pages", "build", "shared", "signed"):
        if args.impl == "reference":
            if int(os.environ.get("RANK", "0")) == 0:
                print(json.dumps({"impl": "reference", "workload": args.workload,
                                  "unavailable": "the reference arm times the decode and single workloads; each "
                                                 "component line carries its CPU port timing in cpu_baseline"}),
                      flush=True)
            return 0
        return run_component(args)
    cfg = workload_cfg(args.workload)
    if args.requests:
        cfg["B"] = args.requests
    if args.impl == "reference":
        return run_reference(args, cfg)
    return run_decode(args, cfg)


if __name__ == "__main__":
    sys.exit(main())

"""Benchmark of the V1 query-side selection path on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload decode|single]

Workloads (synthetic, seeded; shapes of the benchmark configurations):
  decode  128 requests per GPU, context ~U[32K, 128K] tokens, 64 index heads,
          FP8 e4m3 keys with per-token scales, fixed page budget take=40,
          window 64, route -> FP8 score -> Top-2048 -> gather of the 576-dim
          bf16 MLA latent (single output: K and V are the same latent).
  single  1024 single-head queries over 64 built pages + 65-token tail
          (2688 candidates), route -> score -> Top-2048 (no gather).
A step is one pass of the whole selection path over one batch.  Requests are
independent, so N GPUs run N independent batches (weak scaling, no collective
on the data path); `value` is the whole-job queries/s = N*B*K / max-over-ranks
device time.  Rank 0 prints one JSON line.
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


def cpu_port_rate(cfg, seed, rows, budget_s=20.0):
    """Queries/s of the oracle port on a bounded CPU sample (all host cores for BLAS)."""
    import oracle.port as port

    synth = importlib.import_module("10_20_b200.synth")
    torch.set_num_threads(os.cpu_count() or 1)
    case = make_case(synth, cfg, seed, "cpu", rows=rows)
    c = port.to_numpy_case(case)
    port.run_rows(c, rows=[0])            # warm-up (page-in, BLAS init)
    done, t0 = 0, time.perf_counter()
    while True:
        port.run_rows(c, rows=[done % rows])
        done += 1
        el = time.perf_counter() - t0
        if el >= budget_s or done >= 64 * rows:
            break
    return done / el, dict(rows=done, seconds=round(el, 3), sample_requests=rows,
                           lens=[int(x) for x in c["lens"]])


def run_reference(args, cfg):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    rows = 4 if args.workload == "decode" else 32
    vals = []
    for _ in range(args.warmup):
        cpu_port_rate(cfg, 1000, rows, budget_s=2.0)
    meta = None
    for _ in range(args.steps):
        v, meta = cpu_port_rate(cfg, 1000, rows, budget_s=max(5.0, 60.0 / max(args.steps, 1)))
        vals.append(v)
    value = statistics.median(vals)
    cores = os.cpu_count()
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "queries/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp8-e4m3 keys, f32 scores, bf16 latent", "data": "synthetic",
            "config": {"workload": args.workload, **{k: v for k, v in cfg.items()}},
            "cpu_baseline": {"value": value, "unit": "queries/s", "cores": cores, "kind": "port",
                             "sample": f"{meta['rows']} queries of a {rows}-request sample "
                                       f"(oracle port, numpy/BLAS), per step"},
            "e2e": {"value": value, "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--requests", type=int, default=0,
                    help="override the per-GPU batch (small cases for profiling; not a bench config)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="decode", choices=["decode", "single"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    cfg = workload_cfg(args.workload)
    if args.requests:
        cfg["B"] = args.requests
    if args.impl == "reference":
        return run_reference(args, cfg)

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

    pkg = importlib.import_module("10_20_b200")
    pkg.load()
    synth = importlib.import_module("10_20_b200.synth")
    pipeline = importlib.import_module("10_20_b200.pipeline")

    # the job's requests: world * B context lengths from one seed, split across the
    # ranks by bytes (longest first, B requests per rank); each rank builds its own
    # pools and tables for its share
    sharding = importlib.import_module("10_20_b200.sharding")
    lens = None
    if cfg["lo"] != cfg["hi"]:
        lens_all = synth.decode_lens(world * cfg["B"], cfg["lo"], cfg["hi"], 1000)
        if world > 1:
            row = cfg["latent"] * 2
            costs = [sharding.row_bytes(n, cfg["H"], cfg["take"], cfg["window"], cfg["topk"], row)["total"]
                     for n in lens_all]
            lens = [lens_all[i] for i in sharding.shard_requests(costs, world, per_rank=cfg["B"])[rank]]
        else:
            lens = lens_all
    seed = 1000 + rank
    case = make_case(synth, cfg, seed, device, lens=lens)
    step = pipeline.SelectionStep(case, gather=cfg["latent"] > 0)
    acct = step.algorithmic_bytes()
    gather_on = step.gather
    s = torch.cuda.Stream(device=device)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            step.run()
    s.synchronize()

    def capture(fn):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            fn()
        s.synchronize()
        return g

    # the timed step: one graph holding the whole pipelined step (selection of
    # every chunk and the gathers)
    step_graph = capture(step.run)
    # diagnostics, timed separately: selection alone and the gather kernel alone
    # (the roofline's dominant kernel)
    step.gather = False
    sel_graph = capture(step.run)
    step.gather = gather_on
    gat_graph = None
    if gather_on:
        from importlib import import_module
        gmod = import_module("10_20_b200.gather")
        lat = case.latent
        gat_graph = capture(lambda: gmod._gather_impl((1,), lat, None, None, step.physical, step.kv, None, case.B,
                                                      case.topk, 0, *lat.stride(), 0, 0, 0,
                                                      step.physical.stride(0)))
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    launches_per_step = 6 + (1 if gather_on else 0)

    def timed(graph, n):
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
        for a, b in evs:
            flush.fill_(1)                      # evict L2 between timed iterations
            a.record()
            graph.replay()
            b.record()
        return evs

    for _ in range(max(args.warmup, 3)):
        timed(step_graph, 1)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with Clocks(device) as clk:
        t0 = time.perf_counter()
        events = timed(step_graph, args.steps)
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
    if dist:
        dist.barrier()
    step_ms = [a.elapsed_time(b) for a, b in events]
    total_ms = sum(step_ms)
    t = torch.tensor([total_ms], dtype=torch.float64, device=device)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = float(t.item())
    queries = case.B * args.steps * world
    value = queries / (total_ms / 1e3)
    diag_steps = min(args.steps, 20)
    sel_ev = timed(sel_graph, diag_steps)
    gat_ev = timed(gat_graph, diag_steps) if gat_graph is not None else []
    torch.cuda.synchronize()
    sel_ms = [a.elapsed_time(b) for a, b in sel_ev]
    gather_ms = [a.elapsed_time(b) for a, b in gat_ev] or [0.0]

    # end-to-end through the public step: pinned H2D of the step's inputs,
    # the step, D2H of the selected slot ids.  No L2 flush inside this loop: the
    # step's working set (~0.86 GB) is far larger than L2.
    pin_q = case.q8.view(torch.uint8).cpu().pin_memory()
    pin_w = case.w.cpu().pin_memory()
    pin_l = case.lens.cpu().pin_memory()
    pin_nt = case.native_table.cpu().pin_memory()
    out_host = torch.empty(step.physical.shape, dtype=torch.int32).pin_memory()
    h2d = pin_q.numel() + pin_w.numel() * 4 + pin_l.numel() * 4 + pin_nt.numel() * 4
    d2h = out_host.numel() * 4

    def e2e_step():
        case.q8.view(torch.uint8).copy_(pin_q, non_blocking=True)
        case.w.copy_(pin_w, non_blocking=True)
        case.lens.copy_(pin_l, non_blocking=True)
        case.native_table.copy_(pin_nt, non_blocking=True)
        step_graph.replay()
        out_host.copy_(step.physical, non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    ea, eb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ea.record()
    for _ in range(args.steps):
        e2e_step()
    eb.record()
    torch.cuda.synchronize()
    e2e_ms = ea.elapsed_time(eb)
    te = torch.tensor([e2e_ms], dtype=torch.float64, device=device)
    if dist:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = queries / (float(te.item()) / 1e3)

    if rank == 0:
        hbm, kind = peaks()
        if gather_on:
            dom_bytes, dom_ms, dom = acct["gather"], statistics.mean(gather_ms), "gather_vec_kernel"
        else:
            dom_bytes, dom_ms, dom = acct["total"], statistics.mean(sel_ms), "selection graph"
        achieved = dom_bytes / (dom_ms / 1e3) / 1e9
        line = {
            "metric": METRIC, "value": value, "unit": "queries/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp8-e4m3 keys, f32 scores, bf16 latent",
            "data": "synthetic",
            "config": {"workload": args.workload, "requests_per_gpu": case.B, "heads": case.H,
                       "page_budget": case.take, "topk": case.topk, "window": case.window,
                       "context": [cfg["lo"], cfg["hi"]], "latent_dim": cfg["latent"],
                       "parallelism": f"requests sharded by bytes (longest first), {world} ranks x "
                                      f"{case.B} requests, no data-path collective",
                       "l2": "flushed (256 MB write) between timed steps; e2e: working set 0.86 GB > L2",
                       "algorithmic_bytes_per_step": acct["total"]},
            "step_hbm_gbs": acct["total"] / (total_ms / args.steps / 1e3) / 1e9,
            "step_frac_of_peak": acct["total"] / (total_ms / args.steps / 1e3) / 1e9 / hbm,
            "roofline": {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": hbm, "unit": "GB/s",
                         "frac": achieved / hbm, "peak_kind": kind, "traffic": None},
            "stage_ms": {"step": total_ms / args.steps, "selection_alone": statistics.mean(sel_ms),
                         "gather_alone": statistics.mean(gather_ms)},
            "e2e": {"value": e2e_value, "unit": "queries/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk.summary(),
            "wall_s": wall,
        }
        if world == 1 and not args.no_cpu_baseline:
            rows = 4 if args.workload == "decode" else 32
            v, meta = cpu_port_rate(cfg, 1000, rows, budget_s=15.0)
            line["cpu_baseline"] = {"value": v, "unit": "queries/s", "cores": os.cpu_count(), "kind": "port",
                                    "sample": f"{meta['rows']} queries from a {rows}-request sample of the "
                                              f"same workload, oracle port (numpy + BLAS), "
                                              f"{meta['seconds']} s"}
        print(json.dumps(line), flush=True)
    if dist:
        del step_graph, sel_graph, gat_graph
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())

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
    ap.add_argument("--inflight", type=int, default=3,
                    help="independent batches in flight (the gather of one overlaps the selection of the next)")
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
    # `inflight` independent batches (each its own seeded pools, tables and
    # queries; the same context lengths, so every step moves the same bytes) are
    # processed alternately on their own streams: the gather of one batch runs
    # while the next batch is selected.  Consecutive steps touch disjoint data.
    inflight = max(1, args.inflight)
    sets = []
    for i in range(inflight):
        case_i = make_case(synth, cfg, 1000 + rank + 7919 * i, device, lens=lens)
        step_i = pipeline.SelectionStep(case_i, gather=cfg["latent"] > 0)
        st = torch.cuda.Stream(device=device)
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):
            for _ in range(2):
                step_i.run()
        st.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            step_i.run()
        st.synchronize()
        sets.append(dict(case=case_i, step=step_i, stream=st, graph=g))
    case, step = sets[0]["case"], sets[0]["step"]
    acct = step.algorithmic_bytes()
    gather_on = step.gather
    s = sets[0]["stream"]

    def capture(fn):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            fn()
        s.synchronize()
        return g

    # diagnostics of one batch: selection alone and the gather kernel alone (the
    # roofline's dominant kernel)
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
    # L2 eviction before each diagnostic timing: a read of 256 MB that nothing
    # writes, so no dirty lines are left to be written back inside the timing
    flush = torch.ones(256 << 20, dtype=torch.uint8, device=device)
    launches_per_step = 6 + (1 if gather_on else 0)
    main_stream = torch.cuda.current_stream(device)

    def timed(graph, n):
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
        for a, b in evs:
            flush.sum()
            a.record()
            graph.replay()
            b.record()
        return evs

    # end-to-end pieces: pinned inputs of every batch and a pinned output
    for st in sets:
        c = st["case"]
        st["pin"] = [(c.q8.view(torch.uint8), c.q8.view(torch.uint8).cpu().pin_memory()),
                     (c.w, c.w.cpu().pin_memory()), (c.lens, c.lens.cpu().pin_memory()),
                     (c.native_table, c.native_table.cpu().pin_memory())]
        st["out_host"] = torch.empty(st["step"].physical.shape, dtype=torch.int32).pin_memory()
    h2d = sum(hst.numel() * hst.element_size() for _, hst in sets[0]["pin"])
    d2h = sets[0]["out_host"].numel() * 4

    def run_steps(n, e2e=False):
        """Launch n steps alternating over the batches; events on the main stream."""
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(main_stream)
        for st in sets:
            st["stream"].wait_stream(main_stream)
        for k in range(n):
            st = sets[k % inflight]
            with torch.cuda.stream(st["stream"]):
                if e2e:     # host -> device inputs of this step, from pinned memory
                    for dst, hst in st["pin"]:
                        dst.copy_(hst, non_blocking=True)
                st["graph"].replay()
                if e2e:     # device -> host: the step's physical slot ids
                    st["out_host"].copy_(st["step"].physical, non_blocking=True)
        for st in sets:
            main_stream.wait_stream(st["stream"])
        b.record(main_stream)
        return a, b

    for _ in range(max(args.warmup, 3)):
        run_steps(inflight)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with Clocks(device) as clk:
        t0 = time.perf_counter()
        ev = run_steps(args.steps)
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
    if dist:
        dist.barrier()
    total_ms = ev[0].elapsed_time(ev[1])
    t = torch.tensor([total_ms], dtype=torch.float64, device=device)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = float(t.item())
    queries = case.B * args.steps * world
    value = queries / (total_ms / 1e3)

    diag_steps = min(args.steps, 20)
    one_ev = timed(sets[0]["graph"], diag_steps)
    sel_ev = timed(sel_graph, diag_steps)
    # the gather kernel alone, replayed back to back: its 604 MB of traffic per
    # launch is far larger than L2, and its own write-backs stay in the timing
    gat_ev = []
    if gat_graph is not None:
        for _ in range(diag_steps + 1):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            gat_graph.replay()
            b.record()
            gat_ev.append((a, b))
        gat_ev = gat_ev[1:]
    torch.cuda.synchronize()
    one_ms = [a.elapsed_time(b) for a, b in one_ev]
    sel_ms = [a.elapsed_time(b) for a, b in sel_ev]
    gather_ms = [a.elapsed_time(b) for a, b in gat_ev] or [0.0]

    # end to end through the public step: pinned host -> device copies of q, w,
    # lengths and native tables, the step, device -> host copy of the slot ids
    run_steps(2 * inflight, e2e=True)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ee = run_steps(args.steps, e2e=True)
    torch.cuda.synchronize()
    e2e_ms = ee[0].elapsed_time(ee[1])
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
                       "batches_in_flight": inflight,
                       "l2": "inputs larger than L2: consecutive steps alternate between independent batches "
                             "(separate pools, ~12 GB each); single-batch diagnostics after a 256 MB read",
                       "algorithmic_bytes_per_step": acct["total"]},
            "step_hbm_gbs": acct["total"] / (total_ms / args.steps / 1e3) / 1e9,
            "step_frac_of_peak": acct["total"] / (total_ms / args.steps / 1e3) / 1e9 / hbm,
            "roofline": {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": hbm, "unit": "GB/s",
                         "frac": achieved / hbm, "peak_kind": kind, "traffic": None},
            "stage_ms": {"step": total_ms / args.steps, "single_batch_latency": statistics.mean(one_ms),
                         "selection_alone": statistics.mean(sel_ms), "gather_alone": statistics.mean(gather_ms)},
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
        for st in sets:
            del st["graph"]
        del sel_graph, gat_graph
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())

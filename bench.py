#!/usr/bin/env python
"""Benchmark of the constrained beam step (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg2] [--impl ours|reference]

A "step" is one beam-search step of every request of the configured batch:
logits rows [R*B, V] -> new beams.  Steps cycle through the catalog levels
(root, level 1, level 2, ...) carrying the beams forward, as in a real
3-token semantic-ID decode, and restart at the root after the last level.

metric: constrained beam-steps/s = requests x steps / time (whole job), plus
the achieved HBM bandwidth of the fused kernel against the measured copy
bandwidth in MEASURED_PEAKS.json.  Logits are synthetic N(0, sigma^2) from a
seeded torch.Generator, each step's logits (>= 1.2 GB) exceed the 126 MB L2,
so no flush is needed between iterations.

--gpus N (under torchrun): requests are sharded, no collective on the data
path; the time is the max over ranks of the device-timed region.  cfg1, cfg2
and cfg4: every rank runs its own batch of the configured size (weak
scaling).  cfg3: BASELINE's batch of 128 requests is split over the ranks
(strong scaling, 128 / N requests per rank).
--config cfg5 --gpus N (under torchrun): the vocabulary-sharded step instead:
every rank holds V/N logit columns of the same requests (by default the
strided split: rank k holds tokens k, k + N, ...) and the ranks exchange
per-row partials and per-request top-2B keys by NCCL all-gathers (strong
scaling: the job is fixed, per-rank bytes shrink with N); the line splits the
step's time into its phases and the two all-gathers.
--impl reference: the CPU restatement of the reference's step (the oracle
port) on the host cores, on the same chain of levels with beams carried
forward (all requests of cfg2; a stated sample of larger configurations).
"""
from __future__ import annotations

import argparse
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

from vllm_gr_ehaleva_b200.synthetic import CONFIGS, histories, initial_cum, make_catalog  # noqa: E402

METRIC = "constrained beam-steps/sec (requests x steps)"
UNIT = "req-steps/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="cfg2", choices=["cfg1", "cfg2", "cfg3", "cfg4", "cfg5"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--requests", type=int, default=None, help="override requests per GPU")
    ap.add_argument("--split", default="strided", choices=["strided", "contiguous"],
                    help="vocab-sharded cfg5: how the lm_head's columns are dealt to the ranks")
    ap.add_argument("--catalog-cache", default=None,
                    help="directory to keep built synthetic catalogs in (reused by later runs of the same call)")
    ap.add_argument("--component", default="step", choices=["step", "suffix_kv", "wire", "remux", "hook"],
                    help="suffix_kv: the suffix KV gather of the attention pass; wire: the step message (host); "
                         "remux: the worker's logprobs remux; hook: the worker-side step over cfg2 sessions")
    return ap.parse_args()


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ------------------------------------------------------------------ clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append([x.strip() for x in line.split(",")])

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for s in self.samples:
            try:
                sm.append(float(s[1]))
                mx = float(s[2])
                for n, v in zip(names, s[5:9]):
                    if v.lower().startswith("active"):
                        reasons.add(n)
            except Exception:
                continue
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ workload
# Configurations whose batch is split over the ranks (strong scaling); the
# others give every rank the configured batch (weak scaling).
STRONG = {"cfg3"}


def requests_per_rank(cfg_name: str, requests: int | None, world: int) -> int:
    if requests:
        return requests
    total = CONFIGS[cfg_name]["requests"]
    if cfg_name in STRONG:
        if total % world:
            raise SystemExit(f"{total} requests do not split over {world} ranks")
        return total // world
    return total


def catalog_for(cfg, cache_dir=None):
    """The configuration's synthetic catalog (seed 1), optionally kept in
    cache_dir between runs."""
    if cache_dir:
        import hashlib
        from vllm_gr_ehaleva_b200.catalog import CSRTrie
        from vllm_gr_ehaleva_b200.synthetic import SyntheticCatalog
        src = open(os.path.join(ROOT, "vllm_gr_ehaleva_b200", "synthetic.py"), "rb").read()
        key = hashlib.sha1(repr((cfg["items"], cfg["levels"], cfg["codebook"], cfg["vocab"], cfg["zipf"])).encode()
                           + src).hexdigest()[:16]
        path = os.path.join(cache_dir, f"catalog_{key}.npz")
        if os.path.exists(path):
            z = np.load(path)
            m = [int(v) for v in z["meta"]]
            return SyntheticCatalog(csr=CSRTrie(z["row_ptr"], z["child_tok"], z["child_node"]), vocab_size=m[0],
                                    levels=m[1], codebook=m[2], num_items=m[3], sid_begin=m[4], sid_end=m[5],
                                    start_node=m[6])
    cat = make_catalog(cfg["items"], cfg["levels"], cfg["codebook"], cfg["vocab"], cfg["zipf"], seed=1)
    if cache_dir:
        os.makedirs(cache_dir, exist_ok=True)
        tmp = path + f".{os.getpid()}.tmp.npz"
        np.savez(tmp, row_ptr=cat.csr.row_ptr, child_tok=cat.csr.child_tok, child_node=cat.csr.child_node,
                 meta=np.array([cat.vocab_size, cat.levels, cat.codebook, cat.num_items, cat.sid_begin,
                                cat.sid_end, cat.start_node], np.int64))
        os.replace(tmp, path)
    return cat


def build_workload(cfg_name: str, requests: int | None, device, world: int = 1, cache_dir=None):
    import torch
    from vllm_gr_ehaleva_b200.synthetic import logits_torch
    cfg = dict(CONFIGS[cfg_name])
    R = requests_per_rank(cfg_name, requests, world)
    B, V = cfg["beams"], cfg["vocab"]
    dtype = {"bf16": torch.bfloat16, "f32": torch.float32}[cfg["dtype"]]
    wl = {"cfg": cfg, "R": R, "B": B, "V": V, "dtype": dtype}
    if cfg["levels"]:
        cat = catalog_for(cfg, cache_dir)
        wl["catalog"] = cat
        wl["levels"] = cfg["levels"]
        wl["csr_dev"] = (torch.from_numpy(cat.csr.row_ptr).to(device), torch.from_numpy(cat.csr.child_tok).to(device),
                         torch.from_numpy(cat.csr.child_node).to(device))
    else:
        wl["catalog"] = None
        wl["levels"] = 2        # unconstrained: alternate two logits buffers
        wl["csr_dev"] = None
    nbuf = wl["levels"]
    rows = R * B
    if rows * V * 4 <= (4 << 30):
        wl["logits"] = [logits_torch(rows, V, cfg["sigma"], seed=100 + i, dtype=dtype, device=device)
                        for i in range(nbuf)]
    else:
        # large batches (cfg3 on few GPUs): drawn in blocks of rows so that the
        # float32 draw never holds more than 4 GB next to the kept buffers
        per = max(1, (4 << 30) // (V * 4))
        wl["logits"] = []
        for i in range(nbuf):
            buf = torch.empty((rows, V), dtype=dtype, device=device)
            for j, r0 in enumerate(range(0, rows, per)):
                r1 = min(rows, r0 + per)
                buf[r0:r1] = logits_torch(r1 - r0, V, cfg["sigma"], seed=100 + i + 1000 * j, dtype=dtype,
                                          device=device)
            wl["logits"].append(buf)
    return wl


def initial_state(wl, device):
    import torch
    R, B = wl["R"], wl["B"]
    cum = torch.from_numpy(initial_cum(R, B)).to(device)
    if wl["catalog"] is not None:
        node = torch.full((R, B), wl["catalog"].start_node, dtype=torch.int32, device=device)
        hist = torch.full((R, B, 1), wl["catalog"].sid_begin, dtype=torch.int32, device=device)
    else:
        node = torch.full((R, B), -1, dtype=torch.int32, device=device)
        hist = torch.from_numpy(histories(R, B, wl["cfg"]["hist"], wl["V"], seed=3)).to(device)
    return cum, node, hist


def pen_tables_launched(wl) -> bool:
    """The selecting kernel runs pen_table_kernel first for processed-mode
    steps with penalties (step_kwargs passes them in that mode)."""
    return step_kernel_name(wl) == "fused_select_ws_kernel" and wl["cfg"]["mode"] == "processed"


def step_kernel_name(wl) -> str:
    """The step kernel the library picks for this workload: the selecting
    warp-specialised kernel for steps without a catalog, else the
    warp-specialised one unless GR_BEAM_KERNEL=stream or the step applies
    penalties in the processed domain."""
    choice = os.environ.get("GR_BEAM_KERNEL", "auto")
    cfg = wl["cfg"]
    if choice == "stream":
        return "fused_step_kernel"
    if wl["catalog"] is None and choice != "ws":
        return "fused_select_ws_kernel"      # steps without a catalog: every row streamed
    # step_kwargs passes the penalty lists in the processed mode; histories are non-empty
    penalised = cfg["mode"] == "processed"
    if choice != "ws" and penalised:
        return "fused_step_kernel"
    return "fused_step_ws_kernel"


def step_kwargs(wl):
    cfg = wl["cfg"]
    kw = dict(beam_width=wl["B"], csr=wl["csr_dev"], vocab_size=wl["V"])
    if cfg["mode"] == "processed":
        R = wl["R"]
        kw.update(logprobs_mode="processed_logprobs", temperature=[cfg["temperature"]] * R,
                  repetition_penalty=[cfg["rep"]] * R, presence_penalty=[cfg["pres"]] * R,
                  frequency_penalty=[cfg["freq"]] * R, eos_token_id=None)
    return kw


def algorithmic_bytes(wl, node_np: np.ndarray, hist_len: int) -> int:
    """Algorithmic bytes of one step of R requests: every logit once, CSR rows of the
    distinct nodes, per-beam inputs and outputs, and the fork table read and write."""
    R, B, V = wl["R"], wl["B"], wl["V"]
    s = 2 if wl["cfg"]["dtype"] == "bf16" else 4
    total = R * B * V * s                       # every logit read once
    total += R * B * 12                         # cum, node, lse
    total += R * (2 * B * 12 + B * 16)          # candidates + selected beams
    total += R * (B * hist_len * 4 + B * (hist_len + 1) * 4)   # fork table read + write
    if wl["catalog"] is not None:
        deg = wl["catalog"].csr.degree
        for r in range(R):
            nodes = np.unique(node_np[r][node_np[r] >= 0])
            total += int(np.sum(8 + 8 * deg(nodes)))
    else:
        total += R * B * hist_len * 4           # penalty histories (same buffer as the fork table)
    return int(total)


# ------------------------------------------------------------------ our arm
def run_ours(args):
    import torch
    import torch.distributed as dist
    from vllm_gr_ehaleva_b200.sample import beam_step
    from vllm_gr_ehaleva_b200.sample.beam_search_sampler import Workspace

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    device = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(device)
    wl = build_workload(args.config, args.requests, device, world, args.catalog_cache)
    R, B = wl["R"], wl["B"]
    kw = step_kwargs(wl)
    ws = Workspace(device)
    levels = wl["levels"]
    cum0, node0, hist0 = initial_state(wl, device)
    stream = torch.cuda.current_stream(device)

    # state per level so that each timed step sees the catalog level it would in a decode
    def run_chain(n_steps, record=None, bytes_acc=None):
        cum, node, hist = cum0, node0, hist0
        lvl = 0
        for i in range(n_steps):
            if bytes_acc is not None:
                bytes_acc.append(algorithmic_bytes(wl, node.cpu().numpy(), hist.shape[2]))
            if record is not None:
                record[i][0].record(stream)
            out = beam_step(wl["logits"][lvl], cum, node, hist=hist, workspace=ws, **kw)
            if record is not None:
                record[i][1].record(stream)
            lvl += 1
            if lvl == levels:
                lvl = 0
                cum, node, hist = cum0, node0, hist0
            else:
                cum, node, hist = out.sel_score, out.sel_node, out.hist_out
                if wl["catalog"] is None:
                    hist = hist0      # unconstrained: keep the fixed-length penalty history
        return out

    # algorithmic bytes of one cycle of levels (host-side, outside timing)
    bytes_cycle = []
    run_chain(levels, bytes_acc=bytes_cycle)
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    clocks = ClockSampler(device.index if world == 1 else local)
    clocks.start()
    time.sleep(0.5)          # let nvidia-smi start sampling before the timed region
    # the warm-up steps run right before the timed ones (after the pause above,
    # so that the GPU is out of its idle state when the timing starts)
    out = run_chain(max(args.warmup, 3))
    torch.cuda.synchronize()
    err = int(out.err.item())
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    out = run_chain(args.steps, record=events)
    t1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    elapsed_ms = t0.elapsed_time(t1)
    per_step_ms = [a.elapsed_time(b) for a, b in events]
    err |= int(out.err.item())
    if world > 1:
        t = torch.tensor([elapsed_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms = float(t.item())

    # roofline of the fused kernel: algorithmic bytes / device time of each step
    steps_bytes = [bytes_cycle[i % levels] for i in range(args.steps)]
    avg_launch_ms = float(np.mean(per_step_ms))
    per_level_ms = [round(float(np.mean(per_step_ms[i::levels])), 5) for i in range(min(levels, args.steps))]
    per_level_range = [[round(float(np.min(per_step_ms[i::levels])), 5), round(float(np.max(per_step_ms[i::levels])), 5)]
                       for i in range(min(levels, args.steps))]
    # all bytes of the timed steps over their summed device time
    achieved = float(np.sum(steps_bytes)) / (float(np.sum(per_step_ms)) * 1e-3) / 1e9
    peak, peak_kind = peaks()

    # ---- end to end through the public API with host buffers
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, wl, kw, ws, device, world)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(wl, budget_s=15.0)

    value = world * R * args.steps / (elapsed_ms * 1e-3)
    res = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": round(elapsed_ms / args.steps, 5),
        "higher_is_better": True, "scaling": "strong" if args.config in STRONG else "weak", "vs_baseline": None,
        "dtype": wl["cfg"]["dtype"], "data": "synthetic (seeded N(0, sigma^2) logits, Zipf catalog)",
        "config": {"workload": args.config, "requests_per_gpu": R, "requests_total": world * R,
                   "beam_width": B, "vocab": wl["V"],
                   "catalog_items": None if wl["catalog"] is None else wl["catalog"].num_items,
                   "levels": wl["cfg"]["levels"], "logprobs_mode": wl["cfg"]["mode"],
                   "parallelism": f"request-sharded x{world}" if world > 1 else "single GPU",
                   "l2": "inputs larger than L2 (>= 1.2 GB logits per step), no flush"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "traffic": None,
                     "kernel": f"gr::{step_kernel_name(wl)} (timed as the whole step: row_meta + [pen_table] + step kernel + merge)",
                     "algorithmic_bytes_per_launch": int(np.mean(steps_bytes)),
                     "avg_launch_ms": round(avg_launch_ms, 5), "per_level_ms": per_level_ms,
                     "per_level_ms_min_max": per_level_range,
                     "per_level_bytes": [int(b) for b in bytes_cycle]},
        # row_meta_kernel + the step kernel + merge_kernel per step, and
        # pen_table_kernel before the selecting kernel when penalties apply
        "gpu_launches": (4 if pen_tables_launched(wl) else 3) * args.steps,
        "clocks": clk,
        "device_errors": err,
    }
    if e2e is not None:
        res["e2e"] = e2e
    if cpu is not None:
        res["cpu_baseline"] = cpu
    # DRAM traffic per launch from the committed ncu summary (same kernel, same workload)
    for name in (f"fused_step_{args.config}.md", f"fused_select_{args.config}.md"):
        prof = os.path.join(ROOT, "profiles", name)
        if os.path.exists(prof) and R == CONFIGS[args.config]["requests"]:
            with open(prof) as f:
                for line in f:
                    if line.startswith(f"traffic_bytes_per_launch_{args.config}:"):
                        res["roofline"]["traffic"] = int(line.split(":")[1])
    if rank == 0:
        print(json.dumps(res), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_e2e(args, wl, kw, ws, device, world):
    """Same metric through the public API with host (pinned) input and output buffers:
    every step copies its logits host->device and reads the new beams back."""
    import torch
    from vllm_gr_ehaleva_b200.sample import beam_step
    R, B = wl["R"], wl["B"]
    # one pinned host copy of a step's logits, sent again every step (the
    # inputs' values do not change the work; one buffer keeps large batches
    # within host memory)
    host_logits = wl["logits"][0].cpu().pin_memory()
    dev_buf = torch.empty_like(wl["logits"][0])
    cum0, node0, hist0 = initial_state(wl, device)
    levels = wl["levels"]
    stream = torch.cuda.current_stream(device)
    host_out = {k: torch.empty((R, B), dtype=dt).pin_memory()
                for k, dt in (("sel_score", torch.float32), ("sel_token", torch.int32), ("sel_parent", torch.int32))}
    steps = max(3, min(args.steps, 10))

    def one(i, cum, node, hist):
        dev_buf.copy_(host_logits, non_blocking=True)
        out = beam_step(dev_buf, cum, node, hist=hist, workspace=ws, **kw)
        for k in host_out:
            host_out[k].copy_(getattr(out, k), non_blocking=True)
        return out

    def chain(n):
        cum, node, hist = cum0, node0, hist0
        for i in range(n):
            out = one(i, cum, node, hist)
            if (i + 1) % levels == 0:
                cum, node, hist = cum0, node0, hist0
            else:
                cum, node, hist = out.sel_score, out.sel_node, (out.hist_out if wl["catalog"] is not None else hist0)
        return out

    chain(levels)
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    chain(steps)
    t1.record(stream)
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1)
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    h2d = wl["logits"][0].numel() * wl["logits"][0].element_size()
    d2h = sum(v.numel() * v.element_size() for v in host_out.values())
    return {"value": round(world * R * steps / (ms * 1e-3), 2), "unit": UNIT, "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": int(d2h), "steps": steps}


# ------------------------------------------------------------------ CPU arms
def cpu_sample_inputs(wl_cfg, n_requests: int, seed: int = 0):
    """Host copy of one root-level step of `n_requests` requests (the costliest level)."""
    from oracle.restated import bf16_bits_to_f32, f32_to_bf16_bits
    cfg = wl_cfg
    B, V = cfg["beams"], cfg["vocab"]
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((n_requests, B, V), dtype=np.float32) * np.float32(cfg["sigma"]))
    if cfg["dtype"] == "bf16":
        x = bf16_bits_to_f32(f32_to_bf16_bits(x))
    return x


def cpu_step_time(cfg, cat, n_req: int, threads: int, budget_s: float):
    """Time the oracle port on n_req requests of one root-level step, rows spread
    over `threads` host threads.  Returns (seconds, requests done)."""
    from concurrent.futures import ThreadPoolExecutor
    from oracle import restated as O
    B, V = cfg["beams"], cfg["vocab"]
    x = cpu_sample_inputs(cfg, n_req)
    cum = initial_cum(n_req, B)
    if cat is not None:
        node = np.full((n_req, B), cat.start_node, np.int32)
        csr = O.CSR(cat.csr.row_ptr, cat.csr.child_tok, cat.csr.child_node)
        hist = np.full((n_req, B, 1), cat.sid_begin, np.int32)
        kw = {}
    else:
        node = np.full((n_req, B), -1, np.int32)
        csr = None
        hist = histories(n_req, B, cfg["hist"], V, seed=3)
        kw = dict(logprobs_mode=O.PROCESSED, temperature=[cfg["temperature"]] * n_req,
                  rep_penalty=[cfg["rep"]] * n_req, pres_penalty=[cfg["pres"]] * n_req,
                  freq_penalty=[cfg["freq"]] * n_req)

    def one(r):
        return O.beam_step(x[r:r + 1], cum[r:r + 1], node[r:r + 1], csr, beam_width=B, vocab_size=V,
                           hist_in=hist[r:r + 1], **{k: (v[r:r + 1] if isinstance(v, list) else v) for k, v in kw.items()})

    t0 = time.perf_counter()
    done = 0
    with ThreadPoolExecutor(max_workers=threads) as ex:
        futs = [ex.submit(one, r) for r in range(n_req)]
        for f in futs:
            f.result()
            done += 1
    return time.perf_counter() - t0, done


def cpu_baseline(wl, budget_s=15.0):
    cfg = wl["cfg"]
    threads = len(os.sched_getaffinity(0))
    n_req = max(1, min(wl["R"], threads))
    secs, done = cpu_step_time(cfg, wl["catalog"], n_req, threads, budget_s)
    return {"value": round(done / secs, 4), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{done} requests x 1 root-level step of {wl['cfg']['beams']} beams (oracle/restated.py, "
                      f"one request per thread)", "cpu_model": cpu_model()}


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


def cpu_chain_logits(cfg, n_req: int, threads: int, seed: int = 0):
    """Host logits of n_req requests in the storage dtype (bf16 as its bit
    patterns), drawn one request per task outside any timing."""
    from concurrent.futures import ThreadPoolExecutor
    from oracle.restated import f32_to_bf16_bits
    B, V = cfg["beams"], cfg["vocab"]

    def draw(r):
        rng = np.random.default_rng(seed * 100003 + r)
        x = (rng.standard_normal((B, V), dtype=np.float32) * np.float32(cfg["sigma"]))
        return f32_to_bf16_bits(x) if cfg["dtype"] == "bf16" else x.astype(np.float32)

    with ThreadPoolExecutor(max_workers=threads) as ex:
        return list(ex.map(draw, range(n_req)))


def run_reference(args):
    """Reference arm: the oracle port of the reference's CPU step (reference
    arithmetic: float64 normaliser and score sums, as the reference's Python
    loops) on all host threads, one request per task.  A step is one beam step
    of the sampled requests at the next catalog level, the beams carried
    forward from the previous step as in the GPU arm (root, level 1, ...,
    then the root again); the bf16 -> float32 conversion of the logits is
    inside the timed step (vLLM's logits.float()), their generation is not."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from concurrent.futures import ThreadPoolExecutor
    from oracle import restated as O
    cfg = dict(CONFIGS[args.config])
    R = cfg["requests"]
    B, V = cfg["beams"], cfg["vocab"]
    threads = len(os.sched_getaffinity(0))
    # every request of cfg2 / cfg1 / cfg5; a sample of at least 32 requests (one per task) for the larger batches
    n_req = min(R, max(32, threads))
    cat = catalog_for(cfg, args.catalog_cache) if cfg["levels"] else None
    levels = cfg["levels"] if cat is not None else 2
    xs = cpu_chain_logits(cfg, n_req, threads)
    csr = O.CSR(cat.csr.row_ptr, cat.csr.child_tok, cat.csr.child_node) if cat is not None else None
    kw = {}
    if cfg["mode"] == "processed":
        kw = dict(logprobs_mode=O.PROCESSED, temperature=[cfg["temperature"]], rep_penalty=[cfg["rep"]],
                  pres_penalty=[cfg["pres"]], freq_penalty=[cfg["freq"]])

    def initial():
        cum = initial_cum(n_req, B)
        if cat is not None:
            return ([cum[r:r + 1] for r in range(n_req)], [np.full((1, B), cat.start_node, np.int32)] * n_req,
                    [np.full((1, B, 1), cat.sid_begin, np.int32)] * n_req)
        hist = histories(n_req, B, cfg["hist"], V, seed=3)
        return ([cum[r:r + 1] for r in range(n_req)], [np.full((1, B), -1, np.int32)] * n_req,
                [hist[r:r + 1] for r in range(n_req)])

    state = initial()

    def one(r):
        x = O.bf16_bits_to_f32(xs[r]) if cfg["dtype"] == "bf16" else xs[r]
        return O.beam_step(x[None], state[0][r], state[1][r], csr, beam_width=B, vocab_size=V,
                           hist_in=state[2][r], **kw)

    def step(i, ex):
        nonlocal state
        outs = list(ex.map(one, range(n_req)))
        if (i + 1) % levels == 0:
            state = initial()
        else:
            keep_hist = cat is None      # unconstrained: the fixed-length penalty history
            state = ([o["sel_score"] for o in outs], [o["sel_node"] for o in outs],
                     state[2] if keep_hist else [o["hist_out"] for o in outs])

    warm = max(args.warmup, 3)
    with ThreadPoolExecutor(max_workers=threads) as ex:
        for i in range(warm):                  # untimed steps warm the pool and the caches
            step(i, ex)
        state = initial()
        t0 = time.perf_counter()
        for i in range(args.steps):
            step(i, ex)
        secs = time.perf_counter() - t0
    value = n_req * args.steps / secs
    sample = (f"{n_req} of {R} requests" if n_req < R else f"all {R} requests") + \
             f" x {args.steps} steps, levels cycling over {levels} (oracle/restated.py, one request per task)"
    cfg_line = {"workload": args.config, "requests_per_gpu": R, "requests_total": R, "beam_width": B, "vocab": V,
                "catalog_items": None if cat is None else cat.num_items, "levels": cfg["levels"],
                "logprobs_mode": cfg["mode"], "parallelism": "single GPU",
                "l2": "inputs larger than L2 (>= 1.2 GB logits per step), no flush"}
    res = {"impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": 0,
           "steps": args.steps, "warmup": warm, "ms_per_step": round(1e3 * secs / args.steps, 3),
           "higher_is_better": True, "scaling": "strong" if args.config in STRONG else "weak", "vs_baseline": None,
           "dtype": cfg["dtype"], "data": "synthetic (seeded N(0, sigma^2) logits, Zipf catalog)",
           "config": cfg_line,
           "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": threads, "kind": "port",
                            "sample": sample, "cpu_model": cpu_model()},
           "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(res), flush=True)


def run_sharded(args):
    """Vocabulary-sharded step (cfg5) on N GPUs: each rank V/N columns, NCCL all-gathers.
    With the strided split (default) rank k holds the columns of tokens k, k + N,
    k + 2N, ... (the lm_head's rows dealt round robin once), so every rank gets
    about 1/N of each trie node's children; --split contiguous gives rank k the
    slice [k V/N, (k + 1) V/N)."""
    import datetime

    import torch
    import torch.distributed as dist
    from vllm_gr_ehaleva_b200.sharded import ShardedStepper
    from vllm_gr_ehaleva_b200.synthetic import logits_torch

    world = int(os.environ["WORLD_SIZE"])
    rank = int(os.environ["RANK"])
    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    cfg = dict(CONFIGS[args.config])
    R, B, V = args.requests or cfg["requests"], cfg["beams"], cfg["vocab"]
    if V % world:
        raise SystemExit(f"vocab {V} does not split over {world} ranks")
    VL = V // world
    strided = args.split == "strided"
    voff, vstride = (rank, world) if strided else (rank * VL, 1)
    cat = catalog_for(cfg, args.catalog_cache)
    csr = tuple(torch.from_numpy(a).to(device) for a in (cat.csr.row_ptr, cat.csr.child_tok, cat.csr.child_node))
    levels = cfg["levels"]
    logits = [logits_torch(R * B, VL, cfg["sigma"], seed=1000 + 17 * lvl + rank, dtype=torch.bfloat16, device=device)
              for lvl in range(levels)]
    cum0 = torch.from_numpy(initial_cum(R, B)).to(device)
    node0 = torch.full((R, B), cat.start_node, dtype=torch.int32, device=device)
    hist0 = torch.full((R, B, 1), cat.sid_begin, dtype=torch.int32, device=device)
    stream = torch.cuda.current_stream(device)
    # one persistent stepper per fork-table length (the table grows by one token per level)
    steppers = [ShardedStepper(num_requests=R, num_beams=B, beam_width=B, vocab_size=V, vocab_local=VL,
                               vocab_offset=voff, vocab_stride=vstride, num_shards=world, csr=csr,
                               hist_len=1 + lvl, device=device)
                for lvl in range(levels)]

    def chain(n, marks=None):
        cum, node, hist = cum0, node0, hist0
        for i in range(n):
            out = steppers[i % levels].step(logits[i % levels], cum, node, hist,
                                            marks=None if marks is None else marks[i])
            if (i + 1) % levels == 0:
                cum, node, hist = cum0, node0, hist0
            else:
                cum, node, hist = out.sel_score, out.sel_node, out.hist_out
        return out

    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    out = chain(max(args.warmup, 3))          # warm-up right before the timed steps
    torch.cuda.synchronize()
    err = int(out.err.item())
    dist.barrier()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    out = chain(args.steps)
    t1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    err |= int(out.err.item())
    t = torch.tensor([t0.elapsed_time(t1)], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    step_ms = ms / args.steps
    # phases timed apart in a second pass of the same steps (events between the
    # phases, max over ranks of each phase's mean)
    marks = [[torch.cuda.Event(enable_timing=True) for _ in range(6)] for _ in range(args.steps)]
    dist.barrier()
    chain(args.steps, marks)
    torch.cuda.synchronize()
    names = ["lse_partials", "allgather_partials", "shard_candidates", "allgather_keys", "merge"]
    phase = torch.tensor([float(np.mean([m[i].elapsed_time(m[i + 1]) for m in marks])) for i in range(5)],
                         device=device)
    dist.all_reduce(phase, op=dist.ReduceOp.MAX)
    phases_ms = {n: round(float(v), 5) for n, v in zip(names, phase.tolist())}
    local_bytes = R * B * VL * 2          # this rank's logits, read once per step
    peak, peak_kind = peaks()
    # the HBM-bound phase is the lse-partials stream: its bytes over its own time
    achieved = local_bytes / (phases_ms["lse_partials"] * 1e-3) / 1e9
    res = {
        "metric": METRIC, "value": round(R * args.steps / (ms * 1e-3), 2), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": round(step_ms, 5),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0, sigma^2) logits, Zipf catalog)",
        "config": {"workload": args.config, "requests": R, "beam_width": B, "vocab": V, "vocab_per_rank": VL,
                   "split": args.split,
                   "parallelism": f"vocab-sharded x{world} (NCCL all-gathers, {args.split} columns)",
                   "l2": "per-rank logits larger than L2, no flush"},
        "phases_ms": phases_ms,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind, "traffic": None,
                     "kernel": "lse-partials stream of this rank's columns (phase 1)",
                     "algorithmic_bytes_per_launch": local_bytes},
        "gpu_launches": 8 * args.steps,
        "clocks": clk, "device_errors": err,
    }
    if rank == 0:
        print(json.dumps(res), flush=True)
    dist.barrier()
    dist.destroy_process_group()


# ------------------------------------------------------------------ suffix KV gather
def suffix_layout(R, B, shared, steps, rng):
    """slot_mapping / slot_mapping_out of R mega-decode requests laid out as
    the reference's metadata builder does (beam_attn.py:319-413): per request
    `shared` uncached prefix tokens plus B beams x `steps` decode tokens; beam 0's
    suffix is its own tokens (prefix tail included), beam b > 0 reads the prefix
    tail then its own.  Slots are a random permutation of the cache."""
    per_req = shared + B * steps
    n_src = R * per_req
    smo = []
    for r in range(R):
        base = r * per_req
        smo.extend(range(base, base + shared + steps))
        for b in range(1, B):
            smo.extend(range(base, base + shared))
            own = base + shared + b * steps
            smo.extend(range(own, own + steps))
    return n_src, np.asarray(smo, np.int32)


def run_suffix_kv(args):
    import torch
    from vllm_gr_ehaleva_b200.attention import extract_suffix_kv
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    R, B, H, D, block = 64, 128, 8, 128, 16
    rng = np.random.default_rng(7)
    lines = []
    for name, shared in (("decode", 0), ("shared_tail", 24)):
        steps = 8
        n_src, smo_np = suffix_layout(R, B, shared, steps, rng)
        n_slots = ((n_src + block - 1) // block) * block
        slots = torch.from_numpy(rng.permutation(n_slots)[:n_src].astype(np.int64)).to(device)
        smo = torch.from_numpy(smo_np).to(device)
        n = int(smo.numel())
        k = torch.randn(n_slots // block, block, H, D, device=device).to(torch.bfloat16)
        v = torch.randn(n_slots // block, block, H, D, device=device).to(torch.bfloat16)
        row = H * D * 2
        moved = 2 * n * row * 2                 # K and V rows, each read once and written once
        hbm = 2 * (n_src + n) * row             # distinct source rows read + rows written (shared rows hit L2)
        stream = torch.cuda.current_stream(device)

        def timed(fn, iters):
            for _ in range(max(args.warmup, 3)):
                fn()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(iters):
                fn()
            e1.record(stream)
            torch.cuda.synchronize()
            return e0.elapsed_time(e1) / iters

        iters = min(args.steps, 200)
        ms = timed(lambda: extract_suffix_kv(k, v, slots, smo, n), iters)
        flat_k, flat_v = k.view(-1, H, D), v.view(-1, H, D)
        ms_torch = timed(lambda: (flat_k[slots[smo.long()]], flat_v[slots[smo.long()]]), iters)
        ok, ov = extract_suffix_kv(k, v, slots, smo, n)
        exact = bool(torch.equal(ok, flat_k[slots[smo.long()]]) and torch.equal(ov, flat_v[slots[smo.long()]]))
        # CPU baseline: the oracle's NumPy gather on a bounded sample of the same layout
        from oracle import suffix_kv as osk
        ns = min(n, 8192)
        kc, vc = k.float().cpu().numpy(), v.float().cpu().numpy()
        sm_np = slots.cpu().numpy()
        t0 = time.perf_counter()
        reps = 0
        while time.perf_counter() - t0 < 2.0:
            osk.gather(kc, vc, sm_np, smo_np, ns)
            reps += 1
        cpu_gbs = reps * 2 * ns * row * 2 / (time.perf_counter() - t0) / 1e9
        peak, peak_kind = peaks()
        gbs = moved / (ms * 1e-3) / 1e9
        hbm_gbs = hbm / (ms * 1e-3) / 1e9
        lines.append({
            "metric": "suffix KV gather bytes moved per second", "layout": name, "value": round(gbs, 1),
            "unit": "GB/s", "ms_per_call": round(ms, 5), "tokens": n, "bytes_per_call": moved,
            "exact_vs_torch_index": exact, "torch_index_gbs": round(moved / (ms_torch * 1e-3) / 1e9, 1),
            "dtype": "bf16", "config": {"requests": R, "beams": B, "shared_tail": shared, "steps": steps,
                                         "kv_heads": H, "head_dim": D, "block_size": block,
                                         "l2": "cache and outputs larger than L2, no flush"},
            "roofline": {"bound": "hbm", "achieved": round(hbm_gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(hbm_gbs / peak, 4), "peak_kind": peak_kind, "hbm_bytes_per_call": hbm},
            "cpu_baseline": {"value": round(cpu_gbs, 2), "unit": "GB/s", "cores": 1, "kind": "port",
                             "sample": f"{ns} tokens (oracle/suffix_kv.py NumPy gather, fp32 copy of the cache)"},
        })
    # suffix-pass metadata for the shared_tail layout: the device builder
    # (host records + copy + kernel, synchronised) against the reference
    # builder's Python loops (oracle/suffix_kv.py restates them)
    from oracle import suffix_kv as osk
    from vllm_gr_ehaleva_b200.attention import build_suffix_metadata
    shared, steps = 24, 8
    mega = [dict(prefix_len=shared, cache_len=0, beam_width=B, steps=steps)] * R
    q_starts = list(range(0, (shared + B * steps) * R + 1, shared + B * steps))
    for _ in range(3):
        build_suffix_metadata(mega, q_starts, block, device)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(50):
        m = build_suffix_metadata(mega, q_starts, block, device)
    torch.cuda.synchronize()
    dev_ms = (time.perf_counter() - t0) / 50 * 1e3
    t0 = time.perf_counter()
    for _ in range(3):
        ref = osk.suffix_metadata(mega, q_starts, block)
    py_ms = (time.perf_counter() - t0) / 3 * 1e3
    same = bool(np.array_equal(m["suffix_slot_mapping_out"].cpu().numpy(), ref[1]))
    lines.append({"metric": "suffix-pass metadata build time", "layout": "shared_tail", "value": round(dev_ms, 4),
                  "unit": "ms", "higher_is_better": False, "suffix_tokens": int(m["suffix_total_tokens"]),
                  "python_builder_ms": round(py_ms, 3), "matches_python_builder": same,
                  "config": {"requests": R, "beams": B, "shared_tail": shared, "steps": steps},
                  "note": "device: host records + one copy + gr_suffix_metadata, wall clock with a sync per call; "
                          "python: the reference builder's loops (oracle/suffix_kv.py), one host core"})
    for line in lines:
        print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ step message (host)
def run_wire(args):
    """Build + encode + decode + the core's token list for one mega-request step
    message: the int32 form (vllm_gr_ehaleva_b200.wire, from the step's parent
    indices and fork table) against the reference's per-beam string ids and token
    lists (restated in oracle/wire_ref.py).  Host only."""
    import msgspec
    from oracle import wire_ref
    from vllm_gr_ehaleva_b200 import wire
    rng = np.random.default_rng(3)
    for B, steps in ((128, 3), (512, 4), (1024, 3)):
        prefix = list(range(100, 164))
        parents = rng.integers(0, B, B).astype(np.int32)
        toks = rng.integers(127488, 152064, (B, steps)).astype(np.int32)
        prev_ids = [f"req-prev0000-beam-{j}" for j in range(B)]
        beams = [prefix + t for t in toks.tolist()]
        fork_info = list(zip(parents.tolist(), toks[:, -1].tolist()))

        def ours():
            f = wire.build_step_fork("sess", "req-next0000", "req-prev0000", B, parents, toks, len(prefix))
            g = wire.decode(wire.encode(f))
            return wire.mega_token_ids(g, prefix)

        def ref():
            u = wire_ref.build("sess", fork_info, prev_ids, beams, "req-next0000", len(prefix))
            v = msgspec.msgpack.decode(msgspec.msgpack.encode(u), type=wire_ref.RefStepUpdate)
            return wire_ref.mega_token_ids(v, prefix)

        def t(fn, n=200):
            fn()
            t0 = time.perf_counter()
            for _ in range(n):
                fn()
            return (time.perf_counter() - t0) / n * 1e3

        assert np.array_equal(ours(), np.asarray(ref()))
        f = wire.build_step_fork("sess", "req-next0000", "req-prev0000", B, parents, toks, len(prefix))
        u = wire_ref.build("sess", fork_info, prev_ids, beams, "req-next0000", len(prefix))
        print(json.dumps({"metric": "mega-request step message: build + encode + decode + core token list",
                          "beams": B, "steps": steps, "value": round(t(ours), 4), "unit": "ms",
                          "higher_is_better": False, "bytes": len(wire.encode(f)),
                          "reference_format_ms": round(t(ref), 4),
                          "reference_format_bytes": len(msgspec.msgpack.encode(u)),
                          "note": "host, one core; SamplingParams excluded from both"}), flush=True)


# ------------------------------------------------------------------ logprobs remux
def run_remux(args):
    """gr_remux_logprobs against per-request torch slices / pads / cat (the
    reference's way, restated in oracle/remux.py), 64 mega requests x 128 rows
    x K = 129 (logprobs = beam width, plus the sampled token), CUDA events."""
    import torch
    from oracle import remux as orx
    from vllm_gr_ehaleva_b200.engine import remux_logprobs_tensors
    dev = torch.device("cuda", 0)
    ws = [128] * 64
    K = 129
    rows = sum(ws)
    lps = torch.randn(rows, K, device=dev)
    ids = torch.randint(0, 150000, (rows, K), device=dev, dtype=torch.int32)
    ranks = torch.randint(1, 99, (rows,), device=dev, dtype=torch.int32)
    st = torch.randint(0, 150000, (rows, 1), device=dev, dtype=torch.int32)
    cfg = [(i, 0, w) for i, w in enumerate(ws)]
    max_dim = max(ws) * K

    def timed(fn, iters=100):
        for _ in range(5):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(iters):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / iters

    ours = timed(lambda: remux_logprobs_tensors(cfg, max_dim, K, lps, ids, ranks, st))
    ref = timed(lambda: orx.remux_torch(ws, max_dim, K, lps, ids, ranks, st))
    a = remux_logprobs_tensors(cfg, max_dim, K, lps, ids, ranks, st)
    b = orx.remux_torch(ws, max_dim, K, lps, ids, ranks, st)
    same = all(bool(torch.equal(x, y)) for x, y in zip(a, b))
    moved = rows * K * 8 + rows * 8 + len(ws) * max_dim * 12
    print(json.dumps({"metric": "logprobs remux per step", "value": round(ours, 4), "unit": "ms",
                      "higher_is_better": False, "reference_way_ms": round(ref, 4), "exact": same,
                      "bytes_per_call": moved, "achieved_gbs": round(moved / (ours * 1e-3) / 1e9, 1),
                      "config": {"requests": len(ws), "rows_per_request": 128, "K": K},
                      "note": "ours: host offsets + two small copies + one kernel; reference way: torch "
                              "slices / pads / cat per request (oracle/remux.py)"}), flush=True)


# ------------------------------------------------------------------ worker-side step
def run_hook(args):
    """cfg2's root level through WorkerBeamHook (32 sessions of 128 beams in the
    worker's row layout, the same state every call) against one direct step
    call over the same rows."""
    import torch
    from vllm_gr_ehaleva_b200.engine import WorkerBeamHook
    from vllm_gr_ehaleva_b200.sample import beam_step
    from vllm_gr_ehaleva_b200.sample.beam_search_sampler import Workspace
    dev = torch.device("cuda", 0)
    wl = build_workload("cfg2", None, dev)
    R, B, V = wl["R"], wl["B"], wl["V"]
    cat = wl["catalog"]
    cum0 = torch.from_numpy(initial_cum(R, B)).to(dev)
    node0 = torch.full((R, B), cat.start_node, dtype=torch.int32, device=dev)
    logits = wl["logits"][0]
    cfg = []
    for r in range(R):
        cfg.append((f"s{r}", r, B))
    hook = WorkerBeamHook(vocab_size=V, csr=wl["csr_dev"], device=dev)
    ws = Workspace(dev)

    for r in range(R):
        hook.start(f"s{r}", B, cum0[r], node0[r])
    first = {"ids": tuple(f"s{r}" for r in range(R)), "cum": cum0, "node": node0,
             "hist": torch.zeros((R, B, 0), dtype=torch.int32, device=dev)}

    def via_hook():
        # every iteration steps the same root-level state (the sessions point back at it)
        for r in range(R):
            s = hook.sessions[f"s{r}"]
            s._batch, s._idx = first, r
        return hook.step(logits, cfg)

    def direct():
        return beam_step(logits, cum0, node0, beam_width=B, csr=wl["csr_dev"], vocab_size=V, workspace=ws)

    def timed(fn, iters=50):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(iters):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / iters

    h = timed(via_hook)
    d = timed(direct)
    a, b = via_hook(), direct()
    same = all(bool(torch.equal(a[f"s{r}"].sel_token, b.sel_token[r])) for r in range(R))
    print(json.dumps({"metric": "worker-side step (root level of cfg2, 32 sessions x 128 beams)", "unit": "ms",
                      "value": round(h, 4), "higher_is_better": False, "direct_step_ms": round(d, 4),
                      "same_beams": same, "note": "hook: run grouping + one step call on the rows + the "
                                                  "sessions' state update; direct: one step call"}), flush=True)


def main():
    args = parse()
    if args.component == "hook":
        run_hook(args)
        return
    if args.component == "remux":
        run_remux(args)
        return
    if args.component == "suffix_kv":
        run_suffix_kv(args)
        return
    if args.component == "wire":
        run_wire(args)
        return
    if args.impl == "reference":
        run_reference(args)
    elif "shards" in CONFIGS[args.config] and int(os.environ.get("WORLD_SIZE", "1")) > 1:
        run_sharded(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

#!/usr/bin/env python
"""Benchmark of the B200 store's train step (and the forward gather).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload ("train step", one step per data-parallel batch, per GPU):
  dim-64 fp32 table warmed with 10,000,000 int64 keys (splitmix64 sequence),
  batches of 65,536 keys: 95 % Zipf(alpha=1.05) over the warmed keys, 5 %
  never-seen keys inserted on miss; gradients N(0, sigma=1e-3) fp32 per row;
  step = lookup_or_insert -> accumulate_gradients -> optimizer_step(1) with
  Adagrad(lr=0.01, eps=1e-8, initial_accumulator_value=0.1); keys sharded over
  the GPUs by the hash partitioner (N > 1: keys, rows and gradients cross
  NVLink through the library's peer-memory exchange kernels).
  Weak scaling: 65,536 keys per GPU per step.
  Accumulation (--accumulation): "atomic" (default; per-key fp32 sums with
  vector reductions, updates within 1e-5 of the ordered sum) or "ordered"
  (each key's rows summed in arrival order, bit-exact with the reference).

Also reported (rank 0, 1 GPU): the forward-lookup workload - dim-32 fp32
store warmed with 1,000,000 uint64 keys, 400 batches of 4,096 keys Zipf(1.1).

One JSON line is printed by rank 0. `value` is keys/s over all GPUs with the
inputs resident in HBM; `e2e` is the same step through the public API with
host (pinned) inputs and outputs copied inside the timed region.
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
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

DIM = 64
BATCH = 65_536
NUM_KEYS = 10_000_000
FWD_KEYS, FWD_DIM, FWD_BATCH, FWD_BATCHES = 1_000_000, 32, 4096, 400
WIDE_KEYS, WIDE_DIM, WIDE_BATCH, WIDE_BATCHES = 200_000_000, 256, 262_144, 40
KEY_BYTES, M_BYTES = 8, 16
FALLBACK_HBM_GBS = 6650.0
# Kernels of one train step (lookup_or_insert -> accumulate_gradients ->
# optimizer_step), by accumulation mode.
STEP_KERNELS = {
    "ordered": ["k_lookup_or_insert", "k_accumulate", "k_group_fix", "k_group_alloc",
                "k_group_place", "k_group_apply", "k_group_hot"],
    "atomic": ["k_lookup_or_insert", "k_acc_atomic", "k_acc_apply"],
}
# value = train-step keys/s; the forward-lookup figure rides in "forward_lookup".
METRIC = "forward_lookup Mkeys/s & train-step keys/s at 1/2/4/8 B200; % of HBM peak"


def args_parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--num-keys", type=int, default=NUM_KEYS)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-forward", action="store_true")
    p.add_argument("--wide-keys", type=int, default=WIDE_KEYS,
                   help="keys of the wide-row forward store (weight-only, dim 256 bf16); 0 skips it")
    p.add_argument("--eager", action="store_true", help="time eager API calls instead of CUDA graphs")
    p.add_argument("--transport", choices=["p2p", "collective"], default="p2p",
                   help="N > 1: peer-memory exchange kernels, or NCCL all-to-all (eager)")
    p.add_argument("--loopback", action="store_true",
                   help="N = 1: route the step through a one-rank peer-memory exchange (its kernels on one GPU)")
    p.add_argument("--no-dedupe", action="store_true",
                   help="N > 1, p2p: route every position's key (no sender-side dedupe and pre-reduction)")
    p.add_argument("--accumulation", choices=["atomic", "ordered"], default="atomic",
                   help="how accumulate_gradients sums each key's rows: per-key fp32 sums with vector "
                        "reductions (atomic) or kept rows summed in arrival order at the step (ordered)")
    p.add_argument("--capacity", action="store_true",
                   help="N >= 8, p2p: after the train step, run the 1.5e9-key capacity configuration "
                        "(~160 GB per GPU)")
    p.add_argument("--configs-only", action="store_true",
                   help="N > 1: run only the sharded DLRM configuration and, on 8 GPUs, the capacity "
                        "configuration (no train step of the headline workload)")
    p.add_argument("--dlrm", action="store_true",
                   help="N > 1, p2p: after the train step, run the DLRM configuration sharded (26 tables up to "
                        "4e7 rows, fast_range, global batch of 8,192 samples)")
    p.add_argument("--bag-only", type=int, default=0, metavar="SAMPLES",
                   help="run only the DLRM-shaped embedding-bag step with this many samples per batch "
                        "(a small case for profiling) and print its JSON")
    return p.parse_args()


def measured_hbm():
    f = REPO / "MEASURED_PEAKS.json"
    try:
        d = json.loads(f.read_text())
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


# ---------------------------------------------------------------------------
# Clocks
# ---------------------------------------------------------------------------


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML every 1 ms while
    the timed region runs (read-only queries); summary() keeps the samples
    taken between mark_start() and mark_end()."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"),
               ("hw_power_brake", "nvmlClocksEventReasonHwPowerBrakeSlowdown"))

    def __init__(self, index: int):
        self.index = index
        self.samples: list[tuple[float, float, int]] = []
        self.t0 = self.t1 = None
        self.max_mhz = None
        self._stop = threading.Event()
        self.nv = None

    def __enter__(self):
        try:
            import pynvml as nv

            nv.nvmlInit()
            self.nv = nv
            self.h = nv.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM))
            self.thread = threading.Thread(target=self._run, daemon=True)
            self.thread.start()
        except Exception:
            self.nv = None
        return self

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                sm = float(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                rs = int(nv.nvmlDeviceGetCurrentClocksEventReasons(self.h))
                self.samples.append((time.perf_counter(), sm, rs))
            except Exception:
                pass
            time.sleep(0.001)

    def mark_start(self):
        self.t0 = time.perf_counter()

    def mark_end(self):
        self.t1 = time.perf_counter()

    def __exit__(self, *exc):
        self._stop.set()
        if self.nv is not None:
            self.thread.join(timeout=2)
            try:
                self.nv.nvmlShutdown()
            except Exception:
                pass

    def summary(self):
        if self.nv is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "source": "unavailable"}
        t0 = self.t0 if self.t0 is not None else float("-inf")
        t1 = self.t1 if self.t1 is not None else float("inf")
        win = [x for x in self.samples if t0 <= x[0] <= t1]
        where = "timed region"
        if not win and self.samples:
            # a short timed region may fall between two samples: take the
            # nearest ones around it
            win = [x for x in self.samples if t0 - 0.05 <= x[0] <= t1 + 0.05]
            where = "timed region +- 50 ms"
        reasons = set()
        for _, _, rs in win:
            for name, attr in self.REASONS:
                if rs & int(getattr(self.nv, attr, 0)):
                    reasons.add(name)
        sm = [x[1] for x in win]
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(sm), "source": f"nvml every 1 ms, {where}"}


# ---------------------------------------------------------------------------
# Our arm
# ---------------------------------------------------------------------------


def dist_setup(args):
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device(f"cuda:{local}"))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def owned_keys(keys_i64: np.ndarray, world: int, rank: int) -> np.ndarray:
    """The warm keys rank `rank` owns under the hash partitioner (GPU kernel)."""
    if world == 1:
        return keys_i64
    import torch

    import sparse_embedding_b200 as se

    d = torch.from_numpy(keys_i64).cuda()
    ids = se.HashPartitioner(num_shards=world).partition(d)
    return d[ids.to(torch.int64) == rank].cpu().numpy()


def run_ours(args):
    import torch

    import sparse_embedding_b200 as se
    from sparse_embedding_b200 import _native as N
    from sparse_embedding_b200.workloads import ForwardWorkload, TrainWorkload

    world, rank, local = dist_setup(args)
    K, W = args.steps, args.warmup
    wl = TrainWorkload(num_keys=args.num_keys, batch=BATCH, dim=DIM, rank=rank)
    warm = wl.warm_keys()
    mine = owned_keys(warm, world, rank)
    # Room for every row the run can create (5 % new keys per batch, twice
    # over), plus the headroom an insert call checks for while it is being
    # captured: the bound of the rows in use carries the previous call's
    # room for one batch from every rank, and the captured call asks for the
    # same again.
    cap = int(len(mine) + (W + 4 * K + 8) * BATCH * 0.1 + (2 * world + 1) * BATCH)
    store = se.EmbeddingStore(
        se.EmbeddingConfig(dims=[DIM], key_dtype="int64", device=local, initial_capacity=cap,
                           accumulation=args.accumulation),
        optimizer_config=se.Adagrad(lr=0.01, eps=1e-8, initial_accumulator_value=0.1))
    for chunk in np.array_split(mine, max(1, len(mine) // 1_000_000)):
        store.lookup_or_insert(torch.from_numpy(chunk).cuda(), DIM)
    torch.cuda.synchronize()
    api = store
    if world > 1 or args.loopback:
        from sparse_embedding_b200.sharded import ShardedEmbeddingStore

        api = ShardedEmbeddingStore(store, "sparse_embedding.hash", transport=args.transport,
                                    max_keys_per_rank=BATCH, dedupe=not args.no_dedupe)

    keys_np, _ = wl.make_batches(W + 2 * K, start_step=0)
    keys_d = torch.from_numpy(keys_np).cuda()
    gen = torch.Generator(device="cuda").manual_seed(1234 + rank)
    grads_d = torch.randn((W + 2 * K, BATCH, DIM), generator=gen, device="cuda") * 1e-3
    uniq = [int(np.unique(keys_np[W + K + s]).size) for s in range(K)]

    def step(s):
        k = keys_d[s]
        api.lookup_or_insert(k, DIM)
        api.accumulate_gradients(k, grads_d[s])
        api.optimizer_step(1)

    for s in range(W):
        step(s)
    torch.cuda.synchronize()
    barrier(world)

    lib = N.lib()
    # Every timed step is a CUDA graph captured from the same API calls (one
    # graph per batch), so the timed region holds the kernels and not the
    # Python launch path; on several GPUs the peer-memory exchange kernels
    # synchronise the ranks inside the graphs. The NCCL transport needs
    # host-side splits and runs eager. Two timed passes over different batches:
    # pass 1 gives `value` (no instrumentation); pass 2 repeats it with the
    # store's CUDA events around every kernel, on the launching stream, for
    # the per-kernel durations of the roofline.
    use_graphs = not args.eager and (world == 1 or args.transport == "p2p")

    def timed_pass(first, profiled):
        store.profile(profiled)
        graphs = []
        launches0 = lib.se_kernel_launch_count()
        if use_graphs:
            pool = torch.cuda.graph_pool_handle()
            for s in range(K):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, pool=pool, capture_error_mode="relaxed"):
                    step(first + s)
                graphs.append(g)
            torch.cuda.synchronize()
        captured = lib.se_kernel_launch_count() - launches0
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clocks:
            torch.cuda.synchronize()
            barrier(world)
            clocks.mark_start()
            start.record()
            for s in range(K):
                if use_graphs:
                    graphs[s].replay()
                else:
                    step(first + s)
            end.record()
            torch.cuda.synchronize()
            clocks.mark_end()
            barrier(world)
        launches = captured if use_graphs else lib.se_kernel_launch_count() - launches0
        store.profile(False)
        del graphs
        return max_over_ranks(start.elapsed_time(end) / 1e3, world), launches, clocks

    elapsed, launches, clocks = timed_pass(W, False)
    value = world * BATCH * K / elapsed
    elapsed_prof, _, _ = timed_pass(W + K, True)

    # Per-kernel device time inside the timed region.
    names = list(STEP_KERNELS[args.accumulation])
    if (world > 1 and args.transport == "p2p") or args.loopback:
        names += ["k_ex_dedupe", "k_ex_scatter_keys", "k_ex_owner", "k_ex_rows_out", "k_ex_prereduce",
                  "k_ex_scatter_rows", "k_ex_scatter_grads"]
    times = {}
    for nm in names:
        ms, cnt = store.profile_read(nm)
        times[nm] = (ms, cnt)
    peak, peak_kind = measured_hbm()
    R = DIM * 4
    n_new = int(round(BATCH * wl.new_fraction))
    # Algorithmic bytes per launch (what the step must move, per unit):
    #   lookup_or_insert: K + M + R (row read) + R (out write) per key, plus
    #                     R (param) + R (accumulator) initialised per new key;
    #   accumulate:       K + R (key and gradient row read) per gradient row;
    #   optimizer:        per unique key 2R (param read + write) + 2R (Adagrad
    #                     accumulator read + write); the reduced gradient is
    #                     on chip (ordered: registers) or in L2 (atomic sums).
    mean_u = sum(uniq) / len(uniq)
    rows_per_owner = BATCH  # weak scaling: each owner receives ~BATCH rows per step
    acc_name, apply_members = (("k_acc_atomic", ["k_acc_apply"]) if args.accumulation == "atomic"
                               else ("k_accumulate", ["k_group_apply", "k_group_hot"]))
    units = {
        "k_lookup_or_insert": (["k_lookup_or_insert" if "k_ex_owner" not in names else "k_ex_owner"],
                               rows_per_owner * (KEY_BYTES + M_BYTES + 2 * R) + n_new * 2 * R),
        acc_name: ([acc_name], rows_per_owner * (KEY_BYTES + R)),
        "+".join(apply_members): (apply_members, mean_u * 4 * R),
    }
    kern = []
    total_ms = sum(t[0] for t in times.values())
    for nm, (ms, cnt) in times.items():
        kern.append({"kernel": nm, "launches": cnt, "ms_total": round(ms, 4),
                     "share": round(ms / total_ms, 4) if total_ms else None})
    rooflines = []
    for label, (members, nbytes) in units.items():
        ms = sum(times[m][0] for m in members)
        cnt = times[members[0]][1]
        if not cnt:
            continue
        per = ms / cnt / 1e3
        rooflines.append({"kernel": label, "ms_total": ms, "algorithmic_bytes_per_launch": int(nbytes),
                          "achieved_gbs": round(nbytes / per / 1e9, 1)})
    dom = max(rooflines, key=lambda k: k["ms_total"])
    # DRAM bytes (read + write) per launch, copied from ncu --set full
    # captures of the same kernels on the same 65,536-key batch shape with a
    # 2M-key table (the 10M-key table is above the capture-size rule); not
    # measured by this run. Cold-cache replays: each capture starts with an
    # empty L2, so hot keys' rows and the accumulation tables miss once.
    dram = {"k_group_apply+k_group_hot": 23.881e6 + 6.710e6, "k_accumulate": 22.183e6 + 0.011e6,
            "k_lookup_or_insert": 9.486e6 + 0.055e6, "k_acc_atomic": 26.442e6, "k_acc_apply": 20.491e6 + 0.079e6}
    local_store = world == 1 and not args.loopback  # the captured kernels are the local store's
    traffic = dram.get(dom["kernel"]) if local_store else None
    roofline = {"bound": "hbm", "kernel": dom["kernel"], "achieved": dom["achieved_gbs"], "peak": peak,
                "unit": "GB/s", "frac": round(dom["achieved_gbs"] / peak, 4), "traffic": traffic,
                "traffic_source": ("copied, not measured in this run: ncu dram__bytes_read.sum + "
                                   "dram__bytes_write.sum of one cold-cache launch of this kernel, 2M-key table, "
                                   "same 65,536-key batch shape") if traffic else None,
                "peak_source": peak_kind, "per_kernel": rooflines}
    step_bytes = units["k_lookup_or_insert"][1] + BATCH * (KEY_BYTES + R) + mean_u * 4 * R
    step_roof = {"algorithmic_bytes_per_step_per_gpu": int(step_bytes),
                 "achieved_gbs_per_gpu": round(step_bytes * K / (elapsed) / 1e9, 1)}
    step_roof["frac_of_peak"] = round(step_roof["achieved_gbs_per_gpu"] / peak, 4)

    # e2e through the public API from pinned host memory: every step copies
    # its keys and gradients host -> device and reads its rows back device ->
    # host, inside the timed region. The copies run on their own streams
    # (copy engines, both PCIe directions at once), so step s+1's inputs and
    # step s-1's rows move while step s computes; the device buffers and the
    # pinned output buffers are double-buffered.
    keys_e, grads_e = wl.make_batches(K + 1, start_step=10_000)
    kh = [torch.from_numpy(keys_e[s]).pin_memory() for s in range(K + 1)]
    gh = [torch.from_numpy(grads_e[s]).pin_memory() for s in range(K + 1)]
    comp = torch.cuda.current_stream()
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    kd = [torch.empty(BATCH, dtype=torch.int64, device="cuda") for _ in range(2)]
    gd = [torch.empty((BATCH, DIM), dtype=torch.float32, device="cuda") for _ in range(2)]
    out_h = [torch.empty((BATCH, DIM), dtype=torch.float32).pin_memory() for _ in range(2)]
    ev_in = [torch.cuda.Event() for _ in range(K + 1)]
    ev_comp = [torch.cuda.Event() for _ in range(K + 1)]

    def e2e_step(s):
        b = s % 2
        with torch.cuda.stream(s_in):
            if s >= 2:
                s_in.wait_event(ev_comp[s - 2])  # step s-2 is done with buffers b
            kd[b].copy_(kh[s], non_blocking=True)
            gd[b].copy_(gh[s], non_blocking=True)
            ev_in[s].record(s_in)
        comp.wait_event(ev_in[s])
        rows = api.lookup_or_insert(kd[b], DIM)
        if isinstance(rows, tuple):
            rows = rows[0]
        api.accumulate_gradients(kd[b], gd[b])
        api.optimizer_step(1)
        ev_comp[s].record(comp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_comp[s])
            out_h[b].copy_(rows.view(BATCH, DIM), non_blocking=True)
            rows.record_stream(s_out)

    e2e_step(0)
    torch.cuda.synchronize()
    barrier(world)
    t0 = time.perf_counter()
    for s in range(1, K + 1):
        e2e_step(s)
    torch.cuda.synchronize()
    e2e_el = max_over_ranks(time.perf_counter() - t0, world)
    e2e_value = world * BATCH * K / e2e_el

    # The link's own bound: the same pinned copies, streams and buffers with
    # no kernels between them (each step's rows read back from a device
    # buffer of the same size).
    rows_d = [torch.empty((BATCH, DIM), dtype=torch.float32, device="cuda") for _ in range(2)]

    def copy_step(s):
        b = s % 2
        with torch.cuda.stream(s_in):
            kd[b].copy_(kh[s], non_blocking=True)
            gd[b].copy_(gh[s], non_blocking=True)
        with torch.cuda.stream(s_out):
            out_h[b].copy_(rows_d[b], non_blocking=True)

    copy_step(0)
    torch.cuda.synchronize()
    barrier(world)
    t0 = time.perf_counter()
    for s in range(1, K + 1):
        copy_step(s)
    torch.cuda.synchronize()
    copy_el = max_over_ranks(time.perf_counter() - t0, world)
    e2e = {"value": e2e_value, "unit": "keys/s", "h2d_bytes_per_step": BATCH * (KEY_BYTES + R) * world,
           "d2h_bytes_per_step": BATCH * R * world,
           "pipeline": "H2D, compute and D2H on separate streams, double-buffered",
           "link_bound": {"value": world * BATCH * K / copy_el, "unit": "keys/s",
                          "h2d_gbs_per_gpu": round(BATCH * (KEY_BYTES + R) * K / copy_el / 1e9, 1),
                          "d2h_gbs_per_gpu": round(BATCH * R * K / copy_el / 1e9, 1),
                          "note": "the same copies with no kernels: the PCIe ceiling of e2e"}}

    large = mut = uniq = bag = None
    if world == 1 and not args.no_forward:
        large = large_batch_bench(store, torch, args.num_keys, peak)
        mut = mutation_bench(store, torch, args.num_keys, peak)
        uniq = unique_bench(se, torch, args.num_keys)
        bag = dlrm_bag_bench(se, torch, peak)

    fwd = wide = None
    if world == 1 and not args.no_forward:
        fwd = forward_bench(se, torch, N)
        if args.wide_keys > 0:
            wide = forward_wide_bench(se, torch, N, args.wide_keys)
    if world > 1 and not args.no_forward and args.wide_keys > 0 and args.transport == "p2p":
        if api is not store:  # the train step's exchange is done
            api.close()
            api = store
        wide = forward_wide_sharded_bench(se, torch, world, rank, local, args.wide_keys)
    dlrm = None
    if args.dlrm and world > 1 and args.transport == "p2p":
        if api is not store:
            api.close()
            api = store
        dlrm = dlrm_sharded_bench(se, torch, world, rank, local, peak)
    finding = encode_keys_finding(se, torch, world) if rank == 0 and not args.no_forward else None
    capacity = None
    if args.capacity and world >= 8 and args.transport == "p2p":
        # the capacity table needs the device's memory: the train step's store goes first
        if api is not store:
            api.close()
        del step, e2e_step, keys_d, grads_d
        store = api = None
        torch.cuda.empty_cache()
        capacity = capacity_bench(se, torch, world, rank, local)

    result = {
        "metric": METRIC,
        "value": value, "unit": "keys/s", "n_gpus": world, "steps": K, "warmup": W,
        # the headline figures in one place, ahead of the long per-kernel lists
        "summary": {"train_step_keys_per_s": value, "train_step_us": elapsed / K * 1e6,
                    "train_step_frac_of_hbm": step_roof["frac_of_peak"],
                    "e2e_keys_per_s": e2e_value, "accumulation": args.accumulation},
        "ms_per_step": elapsed / K * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": train_config(args, world),
        "execution": {"accumulation": args.accumulation,
                      "transport": (args.transport if world > 1 else ("p2p-loopback" if args.loopback else "none")),
                      "dedupe": bool((world > 1 or args.loopback) and args.transport == "p2p" and not args.no_dedupe)},
        "timing": ("CUDA graph replay per step (captured from the public API calls)" if use_graphs
                   else "eager API calls"),
        "profiled_pass_ms_per_step": elapsed_prof / K * 1e3,
        "roofline": roofline, "step_roofline": step_roof, "kernels": kern,
        "e2e": e2e, "clocks": clocks.summary(), "gpu_launches": int(launches),
    }
    if fwd:
        result["forward_lookup"] = fwd
        result["summary"]["forward_lookup_mkeys_per_s"] = round(fwd["value"], 1)
        result["summary"]["forward_lookup_us_per_call"] = round(fwd["us_per_call"], 2)
    if wide:
        result["forward_wide"] = wide
        result["summary"]["forward_wide_mkeys_per_s"] = round(wide["value"], 1)
        result["summary"]["forward_wide_frac_of_hbm"] = wide.get("frac", wide.get("hbm_frac"))
        if "nvlink_frac" in wide:
            result["summary"]["forward_wide_nvlink_frac"] = wide["nvlink_frac"]
    if dlrm:
        result["dlrm_sharded"] = dlrm
        result["summary"]["dlrm_sharded_ids_per_s"] = dlrm["value"]
    if finding:
        result["encode_keys_fast_range"] = finding
    if capacity:
        result["capacity"] = capacity
        if "value" in capacity:
            result["summary"]["capacity_keys_per_s"] = capacity["value"]
    if large:
        result["train_step_large_batch"] = large
    if mut:
        result["mutation"] = mut
    if uniq:
        result["unique"] = uniq
    if bag:
        result["embedding_bag"] = bag
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(seconds=20.0)
    if api is not store and api is not None:
        api.close()
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return result if rank == 0 else None


def forward_bench(se, torch, N):
    from sparse_embedding_b200.workloads import ForwardWorkload

    fw = ForwardWorkload(num_keys=FWD_KEYS, dim=FWD_DIM, batch=FWD_BATCH)
    store = se.EmbeddingStore(se.EmbeddingConfig(dims=[FWD_DIM], key_dtype="uint64", enable_optimizer=False,
                                                 initial_capacity=FWD_KEYS))
    warm = torch.from_numpy(fw.warm_keys()).cuda()
    store.lookup_or_insert(warm, FWD_DIM)
    batches = torch.from_numpy(fw.batches(FWD_BATCHES)).cuda()
    out = torch.empty(FWD_BATCH * FWD_DIM, dtype=torch.float32, device="cuda")
    lib = N.lib()
    st = torch.cuda.current_stream().cuda_stream
    import ctypes

    def run(i):
        N.check(lib.se_forward_lookup_dim(store._h, batches[i].data_ptr(), FWD_BATCH, FWD_DIM, out.data_ptr(),
                                          ctypes.c_void_p(st)))
    for i in range(10):
        run(i)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    # eager: one API call (and kernel launch) per batch
    a.record()
    for i in range(FWD_BATCHES):
        run(i)
    b.record()
    torch.cuda.synchronize()
    el_eager = a.elapsed_time(b) / 1e3
    # graph-replayed: the 400 calls captured once into one CUDA graph (their
    # launches queue back to back), replayed; per-call time = replay / 400
    g = torch.cuda.CUDAGraph()
    s_cap = torch.cuda.Stream()
    s_cap.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s_cap):
        st_cap = s_cap.cuda_stream
        with torch.cuda.graph(g, stream=s_cap, capture_error_mode="relaxed"):
            for i in range(FWD_BATCHES):
                N.check(lib.se_forward_lookup_dim(store._h, batches[i].data_ptr(), FWD_BATCH, FWD_DIM,
                                                  out.data_ptr(), ctypes.c_void_p(st_cap)))
    torch.cuda.current_stream().wait_stream(s_cap)
    g.replay()
    torch.cuda.synchronize()
    a.record()
    g.replay()
    b.record()
    torch.cuda.synchronize()
    el = a.elapsed_time(b) / 1e3
    del g
    # kernel time from the store's per-kernel events (a separate eager pass)
    store.profile(True)
    for i in range(FWD_BATCHES):
        run(i)
    torch.cuda.synchronize()
    store.profile(False)
    kms, kcnt = store.profile_read("k_lookup")
    peak, _ = measured_hbm()
    per_key = KEY_BYTES + M_BYTES + 2 * FWD_DIM * 4
    kern_gbs = per_key * FWD_BATCH / (kms / kcnt / 1e3) / 1e9
    return {"workload": "dim 32 fp32, 1M warmed uint64 keys, 400 batches x 4,096 keys Zipf(1.1)",
            "value": FWD_BATCH * FWD_BATCHES / el / 1e6, "unit": "Mkeys/s", "timing": "CUDA graph of the 400 calls",
            "us_per_call": el / FWD_BATCHES * 1e6,
            "eager": {"value": FWD_BATCH * FWD_BATCHES / el_eager / 1e6, "us_per_call": el_eager / FWD_BATCHES * 1e6},
            "kernel_us": kms / kcnt * 1e3,
            "kernel_achieved_gbs": round(kern_gbs, 1), "kernel_frac": round(kern_gbs / peak, 4),
            "note": "4,096-key batches are latency bound (one short kernel per call); the tables fit in L2 partly"}


def large_batch_bench(store, torch, num_keys, peak):
    """The same train step on the same table with 8x larger batches
    (524,288 keys, same key and gradient distributions): how the step's
    kernels use HBM once the batch is large enough to leave the latency
    floor. Eager API calls (each step is several hundred microseconds)."""
    from sparse_embedding_b200.workloads import TrainWorkload

    big = 8 * BATCH
    wl = TrainWorkload(num_keys=num_keys, batch=big, dim=DIM, rank=0)
    steps = 12
    keys_np, grads_np = wl.make_batches(steps + 2, start_step=50_000)
    keys = torch.from_numpy(keys_np).cuda()
    grads = torch.from_numpy(grads_np).cuda()
    del grads_np
    uniq = [int(np.unique(keys_np[2 + s]).size) for s in range(steps)]
    # room for the new keys of every batch plus one batch of headroom, so no
    # arena growth falls inside the timed steps (a training loop pays it once)
    store.reserve(store.total_size() + int((2 * steps + 4) * big * wl.new_fraction) + 2 * big, DIM)

    def step(s):
        store.lookup_or_insert(keys[s], DIM)
        store.accumulate_gradients(keys[s], grads[s])
        store.optimizer_step(1)
    for s in range(2):
        step(s)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for s in range(2, steps + 2):
        step(s)
    b.record()
    torch.cuda.synchronize()
    el = a.elapsed_time(b) / 1e3
    # per-kernel times from a second, instrumented pass over the same batches
    store.profile(True)
    for s in range(2, steps + 2):
        step(s)
    torch.cuda.synchronize()
    per_kernel = {}
    for nm in STEP_KERNELS["atomic" if store._config.accumulation == "atomic" else "ordered"]:
        ms, cnt = store.profile_read(nm)
        if cnt:
            per_kernel[nm] = round(ms / cnt * 1e3, 1)
    store.profile(False)
    R = DIM * 4
    n_new = int(round(big * wl.new_fraction))
    step_bytes = big * (KEY_BYTES + M_BYTES + 2 * R) + n_new * 2 * R + big * (KEY_BYTES + R) \
        + sum(uniq) / len(uniq) * 4 * R
    gbs = step_bytes * steps / el / 1e9
    return {"workload": "train step as above with 524,288-key batches (8x), same table", "batch": big,
            "value": big * steps / el, "unit": "keys/s", "us_per_step": el / steps * 1e6,
            "algorithmic_bytes_per_step": int(step_bytes), "achieved_gbs": round(gbs, 1),
            "frac": round(gbs / peak, 4), "timing": "eager API calls, CUDA events",
            "kernel_us": per_kernel}


def mutation_bench(store, torch, num_keys, peak):
    """Mutation API on the bench's table (dim 64 fp32 Adagrad, num_keys warmed
    keys): contains, assign and erase of 65,536 distinct present keys per
    call, then the erased keys inserted again (their rows come back from the
    free stack). Device-resident keys and values; call times from CUDA events
    around the calls, kernel times from the store's per-kernel events."""
    from sparse_embedding_b200.workloads import splitmix64_sequence

    rng = np.random.default_rng(7)
    calls = 8
    idx = rng.choice(num_keys, size=(calls + 1) * BATCH, replace=False)
    keys = torch.from_numpy(splitmix64_sequence(idx).view(np.int64).reshape(calls + 1, BATCH)).cuda()
    vals = torch.randn((BATCH, DIM), device="cuda") * 0.01
    R = DIM * 4
    ops = [  # (name, call, kernel, algorithmic bytes per key)
        ("contains", lambda i: store.contains(keys[i]), "k_contains", KEY_BYTES + M_BYTES + 1),
        ("assign", lambda i: store.assign(keys[i], vals), "k_assign", KEY_BYTES + M_BYTES + 2 * R),
        ("erase", lambda i: store.erase(keys[i]), "k_erase", KEY_BYTES + M_BYTES + 4 + 4),
        # insert again: probe, claim, param + Adagrad state init, row out
        ("reinsert", lambda i: store.lookup_or_insert(keys[i], DIM), "k_lookup_or_insert",
         KEY_BYTES + M_BYTES + 3 * R),
    ]
    for _, fn, _, _ in ops:  # warm-up on the extra batch (erase then insert again)
        fn(calls)
    torch.cuda.synchronize()
    out = {}
    for profiled in (False, True):
        store.profile(profiled)
        for name, fn, kname, per_key in ops:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for i in range(calls):
                fn(i)
            b.record()
            torch.cuda.synchronize()
            if not profiled:
                out[name] = {"us_per_call": round(a.elapsed_time(b) / calls * 1e3, 1),
                             "keys_per_s": BATCH * calls / (a.elapsed_time(b) / 1e3)}
            else:
                ms, cnt = store.profile_read(kname)
                if cnt == 0:
                    continue
                kus = ms / cnt * 1e3
                gbs = per_key * BATCH / (kus / 1e6) / 1e9
                out[name].update({"kernel": kname, "kernel_us": round(kus, 1),
                                  "algorithmic_bytes_per_key": per_key,
                                  "kernel_achieved_gbs": round(gbs, 1), "kernel_frac": round(gbs / peak, 4)})
    store.profile(False)
    assert store.total_size() >= num_keys
    return {"workload": "65,536 distinct present keys per call on the train-step table, 8 calls each",
            "ops": out,
            "note": "assign checks the batch for repeated keys on the device (k_assign_dups, a scratch hash "
                    "set) and reads the verdict back before it returns, since the reference raises before it "
                    "mutates anything (validate_unique_mutation_batch); the call time includes that wait"}


def unique_bench(se, torch, num_keys):
    """se.unique (distinct keys, inverse, first positions, counts) of
    device-resident batches shaped like the train step's: 65,536 and
    524,288 int64 keys, Zipf(1.05) + 5% new. Per call, CUDA events around the
    call (which waits for the distinct count)."""
    from sparse_embedding_b200.workloads import TrainWorkload

    out = {}
    for batch in (BATCH, 8 * BATCH):
        wl = TrainWorkload(num_keys=num_keys, batch=batch, dim=DIM, rank=0)
        keys_np, _ = wl.make_batches(6, start_step=90_000)
        keys = torch.from_numpy(keys_np).cuda()
        for i in range(2):
            se.unique(keys[i], return_first_indices=True, return_counts=True)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for i in range(2, 6):
            u = se.unique(keys[i], return_first_indices=True, return_counts=True)[0]
        b.record()
        torch.cuda.synchronize()
        us = a.elapsed_time(b) / 4 * 1e3
        out[str(batch)] = {"us_per_call": round(us, 1), "keys_per_s": batch / (us / 1e6),
                           "unique_keys": int(u.numel())}
    return {"workload": "unique with inverse, first positions and counts of train-step batches (int64, "
                        "Zipf 1.05 + 5% new), device-resident", "batches": out}


def dlrm_bag_bench(se, torch, peak, samples: int = 8192, capacity: int = 0):
    """DLRM-shaped embedding-bag step on one GPU: 26 tables' pre-mixed u64
    keys in one dim-128 fp32 store with Adam(1e-3); `samples` samples x 26
    tables x max(1, Poisson(20)) ids (~4.3M ids per step at 8,192 samples)
    drawn Zipf(1.2) over each table's rows (1e3..4e7 rows per table,
    log-uniform, seeded; generated on the device); step = embedding_bag with
    insert -> embedding_bag_backward of N(0, 1e-3) pooled gradients ->
    optimizer_step(1). Eager calls, CUDA events."""
    from sparse_embedding_b200.workloads import DlrmWorkload

    wl = DlrmWorkload(batch=samples)
    dim = wl.dim
    steps, warm = 4, 2
    batches = []
    for s in range(warm + steps):
        # the first warm-up batch is 10% larger, so the store's step buffers
        # (sized by the largest window so far) are grown before the timed steps
        src = DlrmWorkload(batch=samples + samples // 10) if s == 0 else wl
        k, o, _, g = src.device_bags(s, torch)
        batches.append((k, o, g))
    ids = [int(b[0].numel()) for b in batches[warm:]]
    uniq = [int(torch.unique(b[0].view(torch.int64)).numel()) for b in batches[warm:]]
    if capacity <= 0:  # every distinct key of all the batches, with room
        capacity = int(1.2 * sum(int(torch.unique(b[0].view(torch.int64)).numel()) for b in batches)) + (1 << 20)
    store = se.EmbeddingStore(se.EmbeddingConfig(dims=[dim], key_dtype="uint64", initial_capacity=capacity),
                              optimizer_config=se.Adam(lr=1e-3))

    def step(b):
        k, o, g = b
        store.embedding_bag(k, o, dim, insert=True)
        store.embedding_bag_backward(k, o, g)
        store.optimizer_step(1)
    for b in batches[:warm]:
        step(b)
    torch.cuda.synchronize()
    a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for b in batches[warm:]:
        step(b)
    e.record()
    torch.cuda.synchronize()
    el = a.elapsed_time(e) / 1e3
    store.profile(True)
    for b in batches[warm:]:
        step(b)
    torch.cuda.synchronize()
    kern = {}
    for nm in ["k_bag_insert", "k_bag_pool", "k_accumulate", "k_group_fix", "k_group_alloc", "k_group_place",
               "k_group_apply", "k_group_hot"]:
        ms, cnt = store.profile_read(nm)
        if cnt:
            kern[nm] = round(ms / cnt * 1e3, 1)
    store.profile(False)
    R = dim * 4
    nb = wl.batch * wl.tables
    # each distinct row read once, a row number per id, the pooled rows written
    pool_bytes = sum(uniq) / len(uniq) * R + sum(ids) / len(ids) * 4 + nb * R
    pool_gbs = pool_bytes / (kern.get("k_bag_pool", float("nan")) / 1e6) / 1e9
    out = {"workload": f"DLRM-shaped bag step: 26 tables, {samples:,} samples, dim 128 fp32, Adam; "
                       "rows per table 1e3..4e7 (seeded log-uniform), ids generated on the device",
           "ids_per_step": int(sum(ids) / len(ids)), "unique_ids_per_step": int(sum(uniq) / len(uniq)),
           "bags_per_step": nb, "us_per_step": round(el / steps * 1e6, 1),
           "value": sum(ids) / el, "unit": "ids/s", "kernel_us": kern, "rows": store.total_size(),
           "k_bag_pool": {"algorithmic_bytes": int(pool_bytes), "achieved_gbs": round(pool_gbs, 1),
                          "frac": round(pool_gbs / peak, 4)}}
    del store
    torch.cuda.empty_cache()
    return out


def forward_wide_bench(se, torch, N, num_keys):
    """Weight-only inference store: int32 keys 0..num_keys-1, dim 256 bf16
    rows from the initializer; forward_lookup of 262,144-key batches uniform
    over the keys (the table is far larger than L2, so every row comes from
    HBM). Algorithmic bytes per key: key 4 + directory 16 + row read 512 +
    row write 512."""
    import ctypes

    from sparse_embedding_b200.workloads import InferenceWorkload

    wl = InferenceWorkload(num_keys=num_keys, dim=WIDE_DIM, batch=WIDE_BATCH)
    store = se.EmbeddingStore(se.EmbeddingConfig(dims=[WIDE_DIM], key_dtype="int32", value_dtype="bfloat16",
                                                 enable_optimizer=False, initial_capacity=num_keys))
    chunk = 1 << 22
    for s0 in range(0, num_keys, chunk):
        keys = torch.arange(s0, min(s0 + chunk, num_keys), dtype=torch.int32, device="cuda")
        store.lookup_or_insert(keys, WIDE_DIM)
    torch.cuda.synchronize()
    batches = torch.from_numpy(wl.batches(WIDE_BATCHES)).cuda()
    out = torch.empty(WIDE_BATCH * WIDE_DIM, dtype=torch.bfloat16, device="cuda")
    lib = N.lib()
    st = torch.cuda.current_stream().cuda_stream

    def run(i):
        N.check(lib.se_forward_lookup_dim(store._h, batches[i].data_ptr(), WIDE_BATCH, WIDE_DIM, out.data_ptr(),
                                          ctypes.c_void_p(st)))
    for i in range(3):
        run(i)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(WIDE_BATCHES):
        run(i)
    b.record()
    torch.cuda.synchronize()
    el = a.elapsed_time(b) / 1e3
    peak, _ = measured_hbm()
    per_key = 4 + M_BYTES + 2 * WIDE_DIM * 2
    gbs = per_key * WIDE_BATCH * WIDE_BATCHES / el / 1e9
    del store
    torch.cuda.empty_cache()
    return {"workload": f"weight-only dim 256 bf16, {num_keys:,} int32 keys, {WIDE_BATCHES} batches x "
                        f"262,144 keys uniform (table {num_keys * 512 / 1e9:.0f} GB >> L2)",
            "value": WIDE_BATCH * WIDE_BATCHES / el / 1e6, "unit": "Mkeys/s",
            "us_per_call": el / WIDE_BATCHES * 1e6, "algorithmic_bytes_per_key": per_key,
            "achieved_gbs": round(gbs, 1), "frac": round(gbs / peak, 4), "peak_gbs": peak}


NVLINK_PEER_GBS = 770.0  # measured peer copy per direction per GPU on this pool's B200s


def forward_wide_sharded_bench(se, torch, world, rank, local, num_keys):
    """The weight-only inference store sharded over the GPUs (hash
    partitioner: rank r holds the int32 keys whose murmur fmix32 & (N-1) is
    r, num_keys / N rows of dim 256 bf16 each), forward_lookup of 262,144-key
    batches per GPU uniform over all keys, through the peer-memory exchange:
    keys to their owners, rows back over NVLink (the row all-to-all). Weak
    scaling; time = max over ranks. Per key: HBM 4 + 16 + 512 (owner's row
    read) + 512 (row written), NVLink (4 + 512) x (N - 1) / N."""
    from sparse_embedding_b200.sharded import ShardedEmbeddingStore
    from sparse_embedding_b200.workloads import InferenceWorkload

    owned = num_keys // world + num_keys // (world * 16) + 1_000_000
    store = se.EmbeddingStore(se.EmbeddingConfig(dims=[WIDE_DIM], key_dtype="int32", value_dtype="bfloat16",
                                                 enable_optimizer=False, initial_capacity=owned, device=local))
    part = se.HashPartitioner(num_shards=world)
    chunk = 1 << 23
    for s0 in range(0, num_keys, chunk):
        keys = torch.arange(s0, min(s0 + chunk, num_keys), dtype=torch.int32, device="cuda")
        mine = keys[part.filter(keys, rank)]
        if mine.numel():
            store.lookup_or_insert(mine, WIDE_DIM)
    torch.cuda.synchronize()
    api = ShardedEmbeddingStore(store, "sparse_embedding.hash", transport="p2p", max_keys_per_rank=WIDE_BATCH,
                                dedupe=False)
    wl = InferenceWorkload(num_keys=num_keys, dim=WIDE_DIM, batch=WIDE_BATCH, seed=0x1BF + rank)
    batches = torch.from_numpy(wl.batches(WIDE_BATCHES)).cuda()
    out = torch.empty((WIDE_BATCH, WIDE_DIM), dtype=torch.bfloat16, device="cuda")
    ex = api.exchange(WIDE_DIM)
    for i in range(3):
        ex.lookup(batches[i], insert=False, out=out)
    torch.cuda.synchronize()
    barrier(world)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(WIDE_BATCHES):
        ex.lookup(batches[i], insert=False, out=out)
    b.record()
    torch.cuda.synchronize()
    el = max_over_ranks(a.elapsed_time(b) / 1e3, world)
    api.check()
    api.close()
    del store
    torch.cuda.empty_cache()
    peak, _ = measured_hbm()
    per_key = 4 + M_BYTES + 2 * WIDE_DIM * 2
    link_per_key = (4 + WIDE_DIM * 2) * (world - 1) / world
    keys_per_gpu_s = WIDE_BATCH * WIDE_BATCHES / el
    hbm_gbs = per_key * keys_per_gpu_s / 1e9
    link_gbs = link_per_key * keys_per_gpu_s / 1e9
    return {"workload": f"weight-only dim 256 bf16, {num_keys:,} int32 keys hash-sharded over {world} GPUs, "
                        f"{WIDE_BATCHES} batches x 262,144 keys per GPU uniform, rows returned over NVLink",
            "value": world * keys_per_gpu_s / 1e6, "unit": "Mkeys/s (all GPUs)", "us_per_batch": el / WIDE_BATCHES * 1e6,
            "hbm_gbs_per_gpu": round(hbm_gbs, 1), "hbm_frac": round(hbm_gbs / peak, 4),
            "nvlink_gbs_per_gpu_per_direction": round(link_gbs, 1),
            "nvlink_frac": round(link_gbs / NVLINK_PEER_GBS, 4),
            "nvlink_peak_source": "measured peer copy 770 GB/s per direction per GPU",
            "timing": "eager exchange calls, CUDA events, max over ranks"}


def encode_keys_finding(se, torch, world):
    """fast_range over the reference's encode_keys layout, measured: the
    share of each shard for 26 tables' ids (table id in the top 16 bits),
    for raw ids, and for the pre-mixed keys the DLRM step uses."""
    from sparse_embedding_b200.workloads import DlrmWorkload

    wl = DlrmWorkload(batch=512)
    keys, _, bag, _ = wl.device_bags(0, torch)
    table = bag % wl.tables
    # the raw ids behind the pre-mixed keys are not kept: draw ids of the same
    # tables uniformly below each table's row count
    rows = torch.as_tensor(wl.table_rows(), dtype=torch.int64, device="cuda")
    raw_ids = (torch.rand(table.numel(), device="cuda", dtype=torch.float64) * rows[table]).to(torch.int64)
    encoded = torch.zeros_like(raw_ids)
    for t in range(wl.tables):
        sel = table == t
        encoded[sel] = DlrmWorkload.encode_keys_like(raw_ids[sel], t)
    part = se.FastRangePartitioner(num_shards=max(world, 8))

    def shares(k):
        p = part.partition(k).to(torch.int64)
        h = torch.bincount(p, minlength=part.num_shards).double()
        return [round(float(x), 4) for x in (h / h.sum()).tolist()]

    return {"shards": part.num_shards, "ids": int(table.numel()),
            "encode_keys_16bit_prefix": shares(encoded.view(torch.uint64)),
            "raw_ids": shares(raw_ids.view(torch.uint64)),
            "premixed_fmix64": shares(keys),
            "note": "fast_range(key, n) = (key * n) >> 64 keeps the top bits: table ids < 2^16 / n in the top 16 "
                    "bits, and ids < 2^64 / n, all land on shard 0; the step's pre-mixed keys spread evenly"}


def dlrm_sharded_bench(se, torch, world, rank, local, peak, samples: int = 8192, steps: int = 4, warm: int = 2):
    """The DLRM configuration at its stated scale: 26 tables with 1e3..4e7
    rows (log-uniform, seeded), dim 128 fp32, Adam(1e-3), fast_range
    partitioner over the GPUs; a global batch of `samples` samples split over
    the ranks (strong scaling), per (sample, table) max(1, Poisson(20)) ids
    drawn Zipf(1.2), generated on the device. Step per rank: sharded
    lookup_or_insert of its ids through the peer-memory exchange (sender-side
    dedupe, atomic accumulation) -> sum-pool per (sample, table) in torch ->
    pooled N(0, 1e-3) gradients broadcast back to each id ->
    accumulate_gradients -> optimizer_step(1). Time = max over ranks."""
    from sparse_embedding_b200.sharded import ShardedEmbeddingStore
    from sparse_embedding_b200.workloads import DlrmWorkload

    per_rank = max(1, samples // world)
    wl = DlrmWorkload(batch=per_rank, max_rows=40_000_000, rank=rank)
    dim = wl.dim
    batches = [wl.device_bags(s, torch) for s in range(warm + steps)]
    n_max = max(int(b[0].numel()) for b in batches)
    ids = sum(int(b[0].numel()) for b in batches[warm:]) / steps
    capacity = int(1.3 * n_max * (warm + steps)) + (1 << 20)  # rows this rank may own after all batches
    store = se.EmbeddingStore(se.EmbeddingConfig(dims=[dim], key_dtype="uint64", device=local,
                                                 initial_capacity=capacity, accumulation="atomic"),
                              optimizer_config=se.Adam(lr=1e-3))
    api = ShardedEmbeddingStore(store, "sparse_embedding.fast_range", transport="p2p",
                                max_keys_per_rank=n_max + n_max // 8, dedupe=True)

    def step(b):
        k, o, bag, g = b
        rows = api.lookup_or_insert(k, dim)
        pooled = torch.zeros((g.shape[0], dim), dtype=torch.float32, device="cuda").index_add_(0, bag, rows)
        grads = g.index_select(0, bag)
        api.accumulate_gradients(k, grads)
        api.optimizer_step(1)
        return pooled

    for b in batches[:warm]:
        step(b)
    torch.cuda.synchronize()
    barrier(world)
    a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for b in batches[warm:]:
        step(b)
    e.record()
    torch.cuda.synchronize()
    el = max_over_ranks(a.elapsed_time(e) / 1e3, world)
    api.check()
    held = store.total_size()
    api.close()
    total_ids = sum_over_ranks(ids, world)
    del store, api, batches
    torch.cuda.empty_cache()
    return {"workload": f"DLRM: 26 tables, rows 1e3..4e7 per table (seeded log-uniform), dim 128 fp32, Adam(1e-3), "
                        f"fast_range over {world} GPUs, global batch {per_rank * world:,} samples "
                        f"({per_rank:,} per GPU), max(1, Poisson(20)) ids per bag, Zipf(1.2), pre-mixed u64 keys",
            "value": total_ids * steps / el, "unit": "ids/s (all GPUs)", "ms_per_step": el / steps * 1e3,
            "ids_per_step_all_gpus": int(total_ids), "rows_held_rank0": int(held),
            "step": "sharded lookup_or_insert -> torch sum-pool -> pooled grads to ids -> accumulate -> Adam step",
            "timing": "eager calls, CUDA events, max over ranks", "scaling": "strong (global batch fixed)"}


def capacity_bench(se, torch, world, rank, local, total_keys: int = 1_500_000_000, steps: int = 10, warmup: int = 3):
    """The capacity configuration: one table of 1.5e9 uint64 keys
    splitmix64(i), dim 64 fp32 with Adam m / v state and a u32 step per row
    (784 B per row: ~147 GB per B200 at 8 GPUs), modulo partitioner; each
    rank generates its keys on the device and inserts the ones it owns
    (after checking its free memory); then full train steps of 262,144 keys
    per GPU (99 % Zipf(1.05) over all keys + 1 % new keys, grads N(0, 1e-3),
    Adam) through the peer-memory exchange with sender-side dedupe and atomic
    accumulation. Runs only where every rank has the memory (8 B200s);
    otherwise reports why it was skipped. Time = max over ranks."""
    import torch.distributed as dist

    from sparse_embedding_b200.sharded import ShardedEmbeddingStore
    from sparse_embedding_b200.workloads import CapacityWorkload

    dim, stride = 64, 784
    own = total_keys // world
    cap = int(own * 1.02) + 8 * 262_144
    dir_bytes = 64 * (1 << (int(cap / 3.5) + 1).bit_length())
    need = cap * stride + dir_bytes + cap * 12 + (6 << 30)  # slabs, directory, row arrays, work buffers
    free, _ = torch.cuda.mem_get_info()
    ok = torch.tensor([1 if free > need else 0], dtype=torch.int32, device="cuda")
    if world > 1:
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    if not int(ok.item()):
        return {"skipped": f"needs ~{need / 1e9:.0f} GB per GPU over {world} GPUs; {free / 1e9:.0f} GB free "
                           f"on rank {rank}"}
    wl = CapacityWorkload(num_keys=total_keys, dim=dim, rank=rank)
    store = se.EmbeddingStore(se.EmbeddingConfig(dims=[dim], key_dtype="uint64", device=local, initial_capacity=cap,
                                                 accumulation="atomic"),
                              optimizer_config=se.Adam(lr=1e-3))
    part = se.ModuloPartitioner(num_shards=world)
    t0 = time.perf_counter()
    chunk = 1 << 26
    for s0 in range(0, total_keys, chunk):
        keys = wl.device_keys(s0, min(chunk, total_keys - s0), torch)
        # boolean indexing has no CUDA kernel for uint64: select on the int64 view
        mine = keys.view(torch.int64)[part.filter(keys, rank)].view(torch.uint64)
        if mine.numel():
            store.lookup_or_insert(mine, dim)
        del keys, mine
    torch.cuda.synchronize()
    warm_s = max_over_ranks(time.perf_counter() - t0, world)
    held = store.total_size()
    api = ShardedEmbeddingStore(store, "sparse_embedding.modulo", transport="p2p", max_keys_per_rank=wl.batch,
                                dedupe=True)

    def one(step):
        k, g = wl.device_batch(step, torch)
        torch.cuda.synchronize()
        return k, g

    for s in range(warmup):
        k, g = one(s)
        api.lookup_or_insert(k, dim)
        api.accumulate_gradients(k, g)
        api.optimizer_step(1)
    batches = [one(warmup + s) for s in range(steps)]
    torch.cuda.synchronize()
    barrier(world)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for k, g in batches:
        api.lookup_or_insert(k, dim)
        api.accumulate_gradients(k, g)
        api.optimizer_step(1)
    b.record()
    torch.cuda.synchronize()
    el = max_over_ranks(a.elapsed_time(b) / 1e3, world)
    api.check()
    api.close()
    used = torch.cuda.mem_get_info()
    del api, store, batches
    torch.cuda.empty_cache()
    return {"workload": f"{total_keys:,} uint64 keys splitmix64(i), dim 64 fp32 + Adam m/v + u32 step "
                        f"({stride} B per row), modulo over {world} GPUs; 262,144-key batches per GPU, 99% "
                        "Zipf(1.05) + 1% new, Adam, exchange with sender-side dedupe, atomic accumulation",
            "value": world * wl.batch * steps / el, "unit": "keys/s (all GPUs)", "ms_per_step": el / steps * 1e3,
            "keys_held_rank0": int(held), "device_bytes_in_use_rank0": int(used[1] - used[0]),
            "warm_seconds": round(warm_s, 2), "timing": "eager API calls, CUDA events, max over ranks",
            "zipf_sampler": "continuous inverse CDF, rank -> fmix64(rank) mod n (no stored permutation)"}


# ---------------------------------------------------------------------------
# CPU baseline / reference arm: the oracle port on the host cores
# ---------------------------------------------------------------------------


def cpu_train(num_keys: int, steps: int, seconds: float, threads: int, warmup: int = 1):
    from oracle import oracle as O
    from sparse_embedding_b200.workloads import TrainWorkload

    wl = TrainWorkload(num_keys=num_keys, batch=BATCH, dim=DIM)
    s = O.OracleStore([DIM], key_dtype="int64", optimizer="adagrad", lr=0.01, eps=1e-8, initial_accumulator=0.1,
                      threads=threads)
    s.reserve(num_keys + 200_000, DIM)
    s.lookup_or_insert(wl.warm_keys(), DIM)
    warmup = max(1, int(warmup))
    keys, grads = wl.make_batches(steps + warmup)

    def one(b):
        s.lookup_or_insert(keys[b], DIM)
        s.accumulate_gradients(keys[b], grads[b], DIM)
        s.optimizer_step(1)
    for b in range(warmup):  # untimed
        one(b)
    done, t0 = 0, time.perf_counter()
    for b in range(warmup, warmup + steps):
        one(b)
        done += 1
        if time.perf_counter() - t0 > seconds:
            break
    el = time.perf_counter() - t0
    return BATCH * done / el, done


def cpu_info(threads: int) -> dict:
    """The host CPU the baseline ran on: model name, widest vector ISA it
    offers, logical CPUs available to this process, threads used."""
    model, flags = "unknown", set()
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name") and model == "unknown":
                model = line.split(":", 1)[1].strip()
            elif line.startswith("flags") and not flags:
                flags = set(line.split(":", 1)[1].split())
    except OSError:
        pass
    isa = "AVX-512" if "avx512f" in flags else ("AVX2" if "avx2" in flags else "SSE")
    return {"cpu_model": model, "cpu_isa": isa, "logical_cpus": len(os.sched_getaffinity(0)),
            "threads_used": threads,
            "code": "oracle port of the reference store flow, g++ -O2 -march=x86-64-v3 (AVX2 level), "
                    "-ffp-contract=off; the reference's own compiled kernels pin its results in the tests"}


def cpu_baseline(seconds: float):
    from oracle import oracle as O

    threads = O.cpu_count()
    value, done = cpu_train(NUM_KEYS, 50, seconds, threads)
    return {"value": value, "unit": "keys/s", "cores": threads, "kind": "port", **cpu_info(threads),
            "sample": f"{done} train steps of 65,536 keys on the 10M-key dim-64 Adagrad table (oracle port, "
                      f"{threads} threads; insert-on-miss single-threaded as in the reference)"}


def train_config(args, world: int) -> dict:
    """The workload both arms run (the GPU arm adds its execution keys)."""
    return {"workload": "single-table train step: dim 64 fp32, 10M warmed int64 keys, 65,536-key "
                        "batches per GPU Zipf(1.05) + 5% new keys, grads N(0,1e-3), Adagrad(lr 0.01, "
                        "eps 1e-8, init_acc 0.1), hash partitioner",
            "num_keys": args.num_keys, "dim": DIM, "batch_per_gpu": BATCH, "parallelism": f"key-sharded x{world}",
            "l2": "inputs larger than L2: 5.1 GB table, fresh batch each step"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    from oracle import oracle as O

    threads = O.cpu_count()
    K, W = args.steps, args.warmup
    value, done = cpu_train(args.num_keys, K, 120.0, threads, warmup=W)
    return {"impl": "reference", "metric": METRIC, "value": value, "unit": "keys/s", "n_gpus": args.gpus, "steps": done,
            "warmup": max(1, W), "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": train_config(args, args.gpus),
            "cpu_baseline": {"value": value, "unit": "keys/s", "cores": threads, "kind": "port", **cpu_info(threads),
                             "sample": f"{done} steps of 65,536 keys (oracle port of the reference store flow; "
                                       "the reference store itself does not build here)"},
            "e2e": {"value": value, "unit": "keys/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def run_configs(args):
    """The sharded DLRM configuration, then (8 GPUs) the capacity one, each
    on a fresh store; rank 0 returns their lines."""
    import torch

    import sparse_embedding_b200 as se

    world, rank, local = dist_setup(args)
    peak, _ = measured_hbm()
    out = {"metric": "configuration runs (DLRM sharded, capacity)", "n_gpus": world, "data": "synthetic"}
    if world > 1:
        out["dlrm_sharded"] = dlrm_sharded_bench(se, torch, world, rank, local, peak)
        torch.cuda.empty_cache()
        if rank == 0:  # on record before the capacity run
            print(json.dumps({"dlrm_sharded": out["dlrm_sharded"], "n_gpus": world}), flush=True)
    if world >= 8:
        out["capacity"] = capacity_bench(se, torch, world, rank, local)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return out if rank == 0 else None


def main():
    args = args_parse()
    if args.bag_only > 0 and args.impl == "ours":
        import torch

        import sparse_embedding_b200 as se

        peak, _ = measured_hbm()
        print(json.dumps(dlrm_bag_bench(se, torch, peak, samples=args.bag_only)), flush=True)
        return
    if args.configs_only and args.impl == "ours":
        out = run_configs(args)
    elif args.impl == "reference":
        out = run_reference(args)
    else:
        out = run_ours(args)
    if out is not None:
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()

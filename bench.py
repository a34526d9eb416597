"""Benchmark of the B200 token sampler on the north-star headline workload.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (per GPU, weak scaling): B=256 rows x V=151936 fp32 logits ``randn*3``,
T=0.7, top-k 50, top-p 0.9, repetition 1.1, presence 0.5, frequency 0.3, 1024
uniform history ids per row, one caller uniform per row (synthetic, seeded; the
reference publishes no benchmark data).

One step = one ``ns_sample`` launch over one batch.  ``value`` is sampled
tokens/s over all ranks with inputs resident in HBM, timed with CUDA events
around CUDA-graph replays totalling exactly K launches (graphs of up to
GRAPH_LAUNCHES launches) that rotate over 3 logits buffers (467 MB in total,
> the 126 MB L2), max over ranks.  ``e2e`` is the same
metric through the public ``B200Sampler.select_batch`` call with the logits
in pinned host memory and the histories as Python lists (H2D copies, packing
and the ids' D2H read inside the timed region).

``--impl reference`` times the CPU restatement of the reference sampler
(``oracle/``) on the host cores, on a bounded sample of rows per step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "nano-inference_b200"))
sys.path.insert(0, REPO)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "sampled tokens/sec and logits HBM GB/s vs peak at B=256,V=151936"
UNIT = "tokens/s"
N_BUFFERS = 3
GRAPH_LAUNCHES = 500
# DRAM bytes (read + write) of one headline launch of the sampling kernel,
# from the ncu capture summarised in profiles/sample_kernel_headline_B256.md
# (dram__bytes_read.sum + dram__bytes_write.sum of one launch, same workload).
NCU_TRAFFIC_BYTES = 156778752 + 6206464


def _peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def algorithmic_bytes(B: int, V: int, H: int, esz: int = 4) -> int:
    """Logits once + history ids + 36 B/row (6 fp32 params, uniform, int64 id)."""
    return B * V * esz + B * H * 4 + B * 36


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if self.proc is None or not self.path:
            return None
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        try:
            for line in open(self.path):
                f = [v.strip() for v in line.split(",")]
                if len(f) < 9:
                    continue
                sm.append(float(f[1]))
                mx.append(float(f[2]))
                for n, v in zip(names, f[5:9]):
                    if v.lower() == "active":
                        reasons.add(n)
        except Exception:
            return None
        finally:
            try:
                os.unlink(self.path)
            except OSError:
                pass
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(world, v: float) -> float:
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# CPU arm: the oracle restatement of the reference sampler
# ---------------------------------------------------------------------------
def cpu_port_tokens_per_s(w, rows: int, steps: int = 1, threads: int = 1):
    from concurrent.futures import ThreadPoolExecutor
    from oracle import sampler_oracle as O
    x = w.logits.numpy()
    u = w.uniforms.numpy()

    def one(b):
        return O.sample_row(x[b], w.histories[b], w.params[b], float(u[b])).token

    t0 = time.perf_counter()
    for _ in range(steps):
        if threads > 1:
            with ThreadPoolExecutor(threads) as ex:
                list(ex.map(one, range(rows)))
        else:
            for b in range(rows):
                one(b)
    dt = time.perf_counter() - t0
    return rows * steps / dt, dt


def run_reference(args, world, rank):
    """The CPU reference arm: rows of the headline workload through the numpy
    restatement, all host threads across rows.  A step is one round of
    `threads` rows; the run stops after the requested steps or a ~90 s budget,
    whichever comes first, and reports both counts."""
    if rank != 0:
        return
    from b200_sampler.workloads import headline
    w = headline()
    threads = os.cpu_count() or 1
    rows = min(w.batch, threads)
    cpu_port_tokens_per_s(w, rows, 1, threads)                      # warm-up round
    _, t_round = cpu_port_tokens_per_s(w, rows, 1, threads)
    steps_run = int(max(1, min(args.steps, 90.0 / max(t_round, 1e-6))))
    for _ in range(min(args.warmup, 1)):
        cpu_port_tokens_per_s(w, rows, 1, threads)
    rate, dt = cpu_port_tokens_per_s(w, rows, steps_run, threads)
    cfg = {"workload": w.notes, "sample_rows_per_step": rows, "rows_per_step_full": w.batch,
           "steps_requested": args.steps, "steps_run": steps_run}
    line = {"impl": "reference", "metric": METRIC, "value": rate, "unit": UNIT, "n_gpus": args.gpus,
            "steps": steps_run, "warmup": args.warmup, "ms_per_step": w.batch / rate * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded randn*3 logits, uniform histories)", "config": cfg,
            "cpu_baseline": {"value": rate, "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": f"{rows} of {w.batch} rows of the headline workload per step, "
                                       f"{steps_run} steps, numpy restatement of Sampler.select_batch, "
                                       f"{threads} threads"},
            "e2e": {"value": rate, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def run_e2e(args, world, w, dev, stream):
    from b200_sampler import B200Sampler
    B, V, H = w.batch, w.vocab, w.history_len
    sampler = B200Sampler(device=dev, seed=1)
    host_logits = w.logits.pin_memory()
    hists = w.histories
    u_host = w.uniforms
    e2e_steps = max(1, min(args.steps, 10))
    with torch.cuda.stream(stream):
        for _ in range(2):
            sampler.select_batch(host_logits, hists, w.params, uniforms=u_host)
        barrier(world)
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            ids = sampler.select_batch(host_logits, hists, w.params, uniforms=u_host)
        dt = time.perf_counter() - t0
    dt = max_over_ranks(world, dt)
    assert len(ids) == B
    return {"value": B * world * e2e_steps / dt, "unit": UNIT,
            "h2d_bytes_per_step": B * V * 4 + B * H * 4 + (B + 1) * 8 + B * 24 + B * 4,
            "d2h_bytes_per_step": B * 8, "steps": e2e_steps,
            "path": "B200Sampler.select_batch(pinned host logits, List[List[int]] histories) -> List[int]"}


def run_ours(args, world, rank, local):
    from b200_sampler.sampler import DeviceBatch
    from b200_sampler.workloads import headline

    dev = torch.device("cuda", local)
    w = headline(seed=rank)
    B, V, H = w.batch, w.vocab, w.history_len
    db = DeviceBatch(w.histories, w.params, dev, uniforms=w.uniforms)
    bufs = [w.logits.to(dev)]
    for i in range(1, N_BUFFERS):
        bufs.append((w.logits.roll(i, dims=1)).to(dev))
    out = torch.empty(B, dtype=torch.int64, device=dev)
    stream = torch.cuda.Stream(dev)

    # correctness gate on the benchmarked inputs (first rows only)
    with torch.cuda.stream(stream):
        rc = db.launch(bufs[0], out, stream)
    stream.synchronize()
    assert rc == 0, rc
    assert int(out.min()) >= 0, "a row failed"

    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 3)):
            assert db.launch(bufs[i % N_BUFFERS], out, stream) == 0
    stream.synchronize()

    # CUDA graphs of up to GRAPH_LAUNCHES launches rotating over the buffers;
    # `reps` replays of the full graph plus one of the remainder make K steps
    def capture(n):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(n):
                db.launch(bufs[i % N_BUFFERS], out, torch.cuda.current_stream(dev))
        return g
    per = min(args.steps, GRAPH_LAUNCHES)
    reps, rem = divmod(args.steps, per)
    g = capture(per)
    g_rem = capture(rem) if rem else None
    with torch.cuda.stream(stream):
        g.replay()                                   # graph warm-up
        if g_rem is not None:
            g_rem.replay()
    stream.synchronize()

    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize(dev)
    with ClockSampler(local) as clk:
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(reps):
                g.replay()
            if g_rem is not None:
                g_rem.replay()
            e1.record(stream)
        stream.synchronize()
    barrier(world)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1)
    ms_max = max_over_ranks(world, ms)
    ms_per_step = ms_max / args.steps
    tokens_per_s = B * world / (ms_per_step / 1e3)

    peak, peak_kind = _peaks()
    alg = algorithmic_bytes(B, V, H)
    achieved = alg / (ms / args.steps / 1e3) / 1e9
    del g, g_rem

    # ---- end to end through the public API, host buffers ----
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, world, w, dev, stream)

    line = {"metric": METRIC, "value": tokens_per_s, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded randn*3 logits, uniform histories)",
            "config": {"workload": w.notes, "global_batch": B * world, "rows_per_gpu": B, "vocab": V,
                       "parallelism": f"rows sharded, {world} GPU(s), no collective",
                       "l2": f"{N_BUFFERS} rotating logits buffers ({N_BUFFERS * B * V * 4 / 1e6:.0f} MB) > L2",
                       "timing": f"CUDA graphs ({per} launches x {reps} replays"
                                 f"{f' + {rem}' if rem else ''}), CUDA events, max over ranks"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": NCU_TRAFFIC_BYTES, "peak_kind": peak_kind,
                         "algorithmic_bytes_per_launch": alg,
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, one launch "
                                           "(profiles/sample_kernel_headline_B256.md)"},
            "gpu_launches": args.steps}
    if e2e is not None:
        line["e2e"] = e2e
    clocks = clk.summary()
    if clocks is not None:
        line["clocks"] = clocks
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        # bounded sample: rows of the same workload until ~10 s of single-thread work
        probe, _ = cpu_port_tokens_per_s(w, 2, 1, 1)
        rows = int(max(2, min(w.batch, probe * 10.0)))
        reps_c = int(max(1, min(100, 10.0 * probe / rows)))
        rate, dtc = cpu_port_tokens_per_s(w, rows, reps_c, 1)
        line["cpu_baseline"] = {"value": rate, "unit": UNIT, "cores": 1, "kind": "port",
                                "sample": f"{rows} of {w.batch} rows of the headline workload x {reps_c} "
                                          f"({dtc:.1f} s), numpy restatement of Sampler.select_batch, 1 thread"}
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_vp(args, world, rank, local):
    """vocab-parallel sampling, B=128 rows of V=151936 fp32
    split into `world` contiguous slices; per step ns_vp_local on this rank's
    slice, then the exchange of the candidate records -- `peer`: ns_vp_signal
    and ns_vp_merge_peers, which reads every rank's record in place over
    NVLink; `gather`: an NCCL all-gather and ns_vp_merge.  Total work is fixed
    as N grows (strong scaling); tokens/s counts the B rows once."""
    import ctypes
    import torch.distributed as dist
    from b200_sampler import _lib
    from b200_sampler.params import SamplingParams, pack_params
    from b200_sampler.vocab_parallel import PeerExchange, _ptr_array, gather_records
    from b200_sampler.workloads import make_logits, make_uniforms

    dev = torch.device("cuda", local)
    B, V, K = 128, 151936, 50
    w = (V + world - 1) // world
    off = rank * w
    width = min(w, V - off)
    full = make_logits(0, B, V, 3.0)
    bufs = [full[:, off:off + width].contiguous().to(dev)]
    for i in range(1, N_BUFFERS):
        bufs.append(full.roll(i, dims=1)[:, off:off + width].contiguous().to(dev))
    params = [SamplingParams(temperature=0.8, top_k=K, top_p=0.95)] * B
    p = torch.from_numpy(pack_params(params)).to(dev)
    pp = p.data_ptr()
    u = make_uniforms(1, B).to(dev)
    cap = K + 16
    n = ctypes.c_int64()
    lib = _lib.load()
    assert lib.ns_vp_record_int64s(B, cap, ctypes.byref(n)) == 0
    rec = torch.empty(n.value, dtype=torch.int64, device=dev)
    out = torch.empty(B, dtype=torch.int64, device=dev)
    vp_ws_bytes = _lib.workspace_bytes(B, width, 0)
    vp_ws = torch.empty(vp_ws_bytes, dtype=torch.uint8, device=dev)
    side = torch.cuda.Stream(dev)
    peer = args.vp_transport == "peer"
    if peer:
        ex = PeerExchange(lib, None, world, rank, dev)
        ex.ensure(int(n.value), side)
        flags_arg, _k1 = _ptr_array([ex.flags(r) for r in range(world)])
        recs_arg = [_ptr_array([ex.record(r, par) for r in range(world)]) for par in (0, 1)]

    def step(i):
        # step i writes record buffer i % 2: every run of steps alternates
        x = bufs[i % N_BUFFERS]
        rp = ex.record(rank, i & 1) if peer else rec.data_ptr()
        rc = lib.ns_vp_local(x.data_ptr(), _lib.NS_DTYPE_F32, B, width, width, off, V, None, None, 0,
                             pp, pp + 4 * B, pp + 8 * B, None, None, None, cap, rp,
                             vp_ws.data_ptr(), vp_ws_bytes, side.cuda_stream)
        assert rc == 0
        if peer:
            rc = lib.ns_vp_signal(flags_arg, world, rank, ex.counter(), side.cuda_stream)
            assert rc == 0
            rc = lib.ns_vp_merge_peers(recs_arg[i & 1][0], world, ex.flags(rank), ex.counter(), B, cap, V,
                                       pp, pp + 4 * B, pp + 8 * B, u.data_ptr(), 0, 0,
                                       out.data_ptr(), side.cuda_stream)
        else:
            g = gather_records(rec) if world > 1 else rec
            rc = lib.ns_vp_merge(g.data_ptr(), world, B, cap, V, pp, pp + 4 * B, pp + 8 * B, u.data_ptr(), 0, 0,
                                 out.data_ptr(), side.cuda_stream)
        assert rc == 0

    with torch.cuda.stream(side):
        for i in range(max(args.warmup, 3) + (max(args.warmup, 3) & 1)):   # even: the graphs start on buffer 0
            step(i)
    torch.cuda.synchronize(dev)
    assert int(out.min()) >= 0

    # CUDA graphs of up to 100 steps (every rank captures the same collectives;
    # an even count keeps the record buffers alternating across replays)
    per = min(args.steps, 100)
    per -= per & 1 if per > 1 else 0
    reps, rem = divmod(args.steps, per)

    def capture(nsteps):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            for i in range(nsteps):
                step(i)
        return g
    g = capture(per)
    g_rem = capture(rem) if rem else None
    with torch.cuda.stream(side):
        g.replay()
    torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize(dev)
    with ClockSampler(local) as clk:
        with torch.cuda.stream(side):
            e0.record(side)
            for _ in range(reps):
                g.replay()
            if g_rem is not None:
                g_rem.replay()
            e1.record(side)
        torch.cuda.synchronize(dev)
    barrier(world)
    del g, g_rem  # graphs holding NCCL calls go before the process group
    if peer:
        ex.release(side)
    ms = max_over_ranks(world, e0.elapsed_time(e1))
    ms_per_step = ms / args.steps
    peak, peak_kind = _peaks()
    local_bytes = B * width * 4
    line = {"metric": "vocab-parallel sampled tokens/sec at B=128,V=151936 (BASELINE config 4)",
            "value": B / (ms_per_step / 1e3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded randn*3 logits)",
            "config": {"workload": f"B={B} V={V} fp32 split into {world} slices of <= {w}; T=0.8 k={K} p=0.95",
                       "record_bytes_per_rank": int(n.value) * 8,
                       "transport": ("peer: records read in place over NVLink by the merge kernel after a "
                                     "flag signal" if peer else "gather: NCCL all-gather of the records"),
                       "timing": f"CUDA graphs of local + exchange + merge ({per} steps x {reps}"
                                 f"{f' + {rem}' if rem else ''}), CUDA events, max over ranks"},
            "roofline": {"bound": "hbm", "achieved": local_bytes / (ms_per_step / 1e3) / 1e9, "peak": peak,
                         "unit": "GB/s", "frac": local_bytes / (ms_per_step / 1e3) / 1e9 / peak,
                         "traffic": None, "peak_kind": peak_kind, "algorithmic_bytes_per_launch": local_bytes},
            "gpu_launches": (3 if peer else 2) * args.steps}
    clocks = clk.summary()
    if clocks is not None:
        line["clocks"] = clocks
    if rank == 0:
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end leg (profiling runs)")
    ap.add_argument("--vp-transport", default="peer", choices=["peer", "gather"],
                    help="vp mode: records read in place over NVLink (peer) or all-gathered (gather)")
    ap.add_argument("--mode", default="rows", choices=["rows", "vp"],
                    help="rows: the headline (rows sharded); vp: vocab-parallel config 4")
    args = ap.parse_args()
    world, rank, local = (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
                          int(os.environ.get("LOCAL_RANK", "0")))
    if args.impl == "reference":
        run_reference(args, world, rank)
        return
    world, rank, local = dist_setup(args.gpus)
    try:
        if args.mode == "vp":
            run_vp(args, world, rank, local)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()

"""Benchmark of the B200 token sampler on the north-star headline workload.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload headline|c1|c2|c3|topp095|softmax|k240] [--mode rows|vp]

Headline workload: B=256 rows x V=151936 fp32 logits ``randn*3``, T=0.7,
top-k 50, top-p 0.9, repetition 1.1, presence 0.5, frequency 0.3, 1024
uniform history ids per row, one caller uniform per row (synthetic, seeded;
the reference publishes no benchmark data).  ``--workload`` selects the other
benchmark configurations and modes (``b200_sampler.workloads.WORKLOADS``).

One step = one ``ns_sample`` launch over the batch.  With N GPUs the one
batch is sharded by rows (strong scaling: rank r samples rows
[r B / N, (r + 1) B / N)); a second, labelled measurement gives every rank the
full batch (weak scaling).  ``value`` is sampled tokens/s of the whole batch
with inputs resident in HBM: CUDA-graph replays of exactly K launches that
rotate over logits buffers totalling >= 2x the L2 (3 at the headline), timed with
CUDA events on the launching stream and bracketed by a barrier and a device
synchronisation; the K-step region is repeated until >= 1 s has elapsed and
the median repeat (max over ranks) is reported.  ``e2e`` is the same metric
through the public ``B200Sampler.select_batch`` call with the logits in pinned
host memory and the histories as Python lists (H2D copies, packing and the
ids' D2H read inside the timed region).

``cpu_baseline`` (rank 0, N=1): the reference's own torch
``Sampler.select_batch`` (installed unmodified under baseline/_ref by
baseline/install_reference.py), else the numpy restatement in ``oracle/``,
on a bounded sample of the workload's rows with all host threads.  The same
leg checks every row of the benchmarked launch against the oracle and fails
the run on a mismatch.

``--impl reference`` times that reference sampler on the full batch per step
(all host threads), steps bounded by a ~60 s budget.
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
N_BUFFERS = 3          # at least this many rotating logits buffers ...
L2_MULTIPLE = 2        # ... and together at least this many times the device's L2


def n_buffers(dev, bytes_per_buffer: int) -> int:
    """Rotating input buffers whose total is >= L2_MULTIPLE x the L2, so no
    timed launch finds its logits in L2 (a small per-GPU shard would
    otherwise fit it)."""
    import math
    l2 = int(getattr(torch.cuda.get_device_properties(dev), "L2_cache_size", 126 << 20))
    return max(N_BUFFERS, int(math.ceil(L2_MULTIPLE * l2 / max(bytes_per_buffer, 1))))


GRAPH_LAUNCHES = 500
MIN_TIMED_S = 1.0
REF_BUDGET_S = 60.0
# DRAM bytes (read + write) of one headline launch of the sampling kernel as
# ncu counted them (dram__bytes_read.sum + dram__bytes_write.sum of one launch
# of the headline workload, captured with --clock-control none on a B200 of
# this pool).  A recorded constant, not measured by this script; it describes
# --workload headline only.
NCU_TRAFFIC_BYTES = 156781056 + 4289792
NCU_TRAFFIC_SOURCE = ("recorded constant: ncu dram__bytes_read.sum + dram__bytes_write.sum of one headline "
                      "launch (sample_kernel<fp32>, B=256), not measured by this run")


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


def metric_for(workload: str) -> str:
    return METRIC if workload == "headline" else f"sampled tokens/sec and logits HBM GB/s vs peak, workload {workload}"


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
# CPU legs: the reference's own torch sampler, or the numpy restatement
# ---------------------------------------------------------------------------
def reference_sampler():
    """(Sampler instance, its SamplingParams class, None) from the unmodified
    reference under baseline/_ref, or (None, None, reason)."""
    ref = os.path.join(REPO, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "nano_inference")):
        return None, None, "baseline/_ref holds no reference install (run baseline/install_reference.py)"
    if ref not in sys.path:
        sys.path.insert(0, ref)
    try:
        from nano_inference.core.sampling import SamplingParams as RefParams
        from nano_inference.sampling import Sampler
    except Exception as e:  # pragma: no cover - depends on the install
        return None, None, f"import failed: {type(e).__name__}: {e}"
    return Sampler(), RefParams, None


def _ref_params(RefParams, params):
    # the reference's SamplingParams has no presence / frequency penalty
    # (core/sampling.py); those are dropped in its arm
    return [RefParams(temperature=float(p.temperature), top_k=int(p.top_k), top_p=float(p.top_p),
                      repetition_penalty=float(p.repetition_penalty)) for p in params]


def cpu_rate(w, rows: int, steps: int, threads: int):
    """Tokens/s of the reference torch sampler (or the numpy port) over the
    first `rows` rows of workload `w`, `steps` times; returns (rate, seconds,
    kind, note).  Each step's select_batch gets a fresh copy of the logits
    (the reference writes them in place), made outside the timed span."""
    torch.set_num_threads(threads)
    sampler, RefParams, why = reference_sampler()
    if sampler is not None:
        ps = _ref_params(RefParams, w.params[:rows])
        hs = w.histories[:rows]
        src = w.logits[:rows]
        dt = 0.0
        for _ in range(steps):
            x = src.clone()
            t0 = time.perf_counter()
            sampler.select_batch(x, hs, ps)
            dt += time.perf_counter() - t0
        return rows * steps / dt, dt, "reference", "reference Sampler.select_batch (sampling/sampler.py:36-91)"
    from concurrent.futures import ThreadPoolExecutor
    from oracle import sampler_oracle as O
    x = w.logits.float().numpy()
    u = w.uniforms.numpy()

    def one(b):
        return O.sample_row(x[b], w.histories[b], w.params[b], float(u[b])).token

    t0 = time.perf_counter()
    for _ in range(steps):
        with ThreadPoolExecutor(threads) as ex:
            list(ex.map(one, range(rows)))
    dt = time.perf_counter() - t0
    return rows * steps / dt, dt, "port", f"numpy restatement in oracle/ ({why})"


def parity_gate(w, ids):
    """Every row of the benchmarked launch against the oracle: greedy rows
    bit-exact, sampled rows equal unless the oracle marks them exempt (a
    top-p cumsum or inverse-CDF step within 1e-6 of its threshold) and the id
    is one of its alternatives."""
    from oracle import sampler_oracle as O
    ref = O.sample_batch(w.logits.float().numpy(), w.histories, w.params, uniforms=w.uniforms.numpy())
    bad, exempt = [], 0
    for b, r in enumerate(ref):
        if r.error:
            if ids[b] >= 0:
                bad.append(b)
        elif ids[b] != r.token:
            if r.exempt and ids[b] in r.allowed:
                exempt += 1
            else:
                bad.append(b)
    return {"rows": len(ref), "mismatch": len(bad), "exempt": exempt, "ok": not bad,
            "first_bad": bad[:8], "oracle": "oracle/sampler_oracle.py"}


def run_reference(args, world, rank):
    """The reference arm: the full batch of the workload through the
    reference's own torch sampler per step (all host threads), steps bounded
    by a ~60 s budget.  Rank 0 only."""
    if rank != 0:
        return
    from b200_sampler.workloads import WORKLOADS
    w = WORKLOADS[args.workload]()
    threads = os.cpu_count() or 1
    B = w.batch
    _, t1, kind, note = cpu_rate(w, B, 1, threads)                    # warm-up step (also sizes the run)
    steps_run = int(max(1, min(args.steps, REF_BUDGET_S // max(t1, 1e-6))))
    rate, dt, kind, note = cpu_rate(w, B, steps_run, threads)
    cfg = {"workload": w.notes, "global_batch": B, "rows_per_step": B, "same_config": True,
           "steps_requested": args.steps, "steps_run": steps_run, "threads": threads}
    if kind == "reference" and any(p.presence_penalty or p.frequency_penalty for p in w.params):
        cfg["note"] = "the reference has no presence/frequency penalty; its arm applies repetition only"
    line = {"impl": "reference", "metric": metric_for(args.workload), "value": rate, "unit": UNIT,
            "n_gpus": args.gpus, "steps": steps_run, "warmup": 1, "ms_per_step": dt / steps_run * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32" if w.logits.element_size() == 4 else "bf16", "data": "synthetic (seeded)", "config": cfg,
            "cpu_baseline": {"value": rate, "unit": UNIT, "cores": threads, "kind": kind,
                             "sample": f"all {B} rows per step x {steps_run} steps ({dt:.1f} s), {note}, "
                                       f"{threads} threads"},
            "e2e": {"value": rate, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def timed_repeats(world, dev, stream, run_k):
    """CUDA-event time (ms) of run_k(), which enqueues exactly K steps on
    `stream`, bracketed by a barrier and a device synchronisation on both
    sides.  Repeated until >= MIN_TIMED_S has elapsed (the count agreed over
    ranks); returns the median repeat and all repeats, each the max over
    ranks."""
    import math

    def once():
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        barrier(world)
        torch.cuda.synchronize(dev)
        with torch.cuda.stream(stream):
            e0.record(stream)
            run_k()
            e1.record(stream)
        stream.synchronize()
        barrier(world)
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1)

    first = once()
    n = int(max(2, math.ceil(MIN_TIMED_S * 1e3 / max(first, 1e-3))))
    n = int(max_over_ranks(world, float(n)))
    ms = [first] + [once() for _ in range(n - 1)]
    ms = [max_over_ranks(world, m) for m in ms]
    return statistics.median(ms), ms


def measure_rows(args, world, dev, w, r0, r1, clk=None):
    """Device time per step of ns_sample over rows [r0, r1) of workload w:
    warm-up launches, then CUDA graphs of exactly K launches rotating over
    logits buffers totalling >= L2_MULTIPLE x the L2.  Returns (median ms per
    step, repeats, ids of the first launch on the unrotated logits, (graph
    launches, replays, remainder, buffers))."""
    from b200_sampler.sampler import DeviceBatch
    rows = slice(r0, r1)
    db = DeviceBatch(w.histories[r0:r1], w.params[r0:r1], dev, uniforms=w.uniforms[rows])
    base = w.logits[rows]
    nb = n_buffers(dev, base.numel() * base.element_size())
    bufs = [base.to(dev)] + [base.roll(i, dims=1).to(dev) for i in range(1, nb)]
    out = torch.empty(r1 - r0, dtype=torch.int64, device=dev)
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        rc = db.launch(bufs[0], out, stream)
    stream.synchronize()
    assert rc == 0, rc
    first_ids = out.cpu().tolist()
    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 3)):
            assert db.launch(bufs[i % nb], out, stream) == 0
    stream.synchronize()

    def capture(n):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(n):
                db.launch(bufs[i % nb], out, torch.cuda.current_stream(dev))
        return g
    per = min(args.steps, GRAPH_LAUNCHES)
    reps, rem = divmod(args.steps, per)
    g = capture(per)
    g_rem = capture(rem) if rem else None

    def run_k():
        for _ in range(reps):
            g.replay()
        if g_rem is not None:
            g_rem.replay()
    with torch.cuda.stream(stream):
        run_k()                                      # graph warm-up
    stream.synchronize()
    if clk is not None:
        with clk:
            ms, all_ms = timed_repeats(world, dev, stream, run_k)
    else:
        ms, all_ms = timed_repeats(world, dev, stream, run_k)
    del g, g_rem
    return ms / args.steps, [m / args.steps for m in all_ms], first_ids, (per, reps, rem, nb)


def run_e2e(args, world, w, dev, r0, r1):
    from b200_sampler import B200Sampler
    B, V, H = r1 - r0, w.vocab, w.history_len
    sampler = B200Sampler(device=dev, seed=1)
    host_logits = w.logits[r0:r1].contiguous().pin_memory()
    hists = w.histories[r0:r1]
    params = w.params[r0:r1]
    u_host = w.uniforms[r0:r1].contiguous()
    e2e_steps = max(1, min(args.steps, 10))
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        for _ in range(2):
            sampler.select_batch(host_logits, hists, params, uniforms=u_host)
        barrier(world)
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            ids = sampler.select_batch(host_logits, hists, params, uniforms=u_host)
        dt = time.perf_counter() - t0
    dt = max_over_ranks(world, dt)
    assert len(ids) == B
    esz = w.logits.element_size()
    return {"value": w.batch * e2e_steps / dt if world > 1 else B * e2e_steps / dt, "unit": UNIT,
            "h2d_bytes_per_step": B * V * esz + sum(len(h) for h in hists) * 4 + (B + 1) * 8 + B * 24 + B * 4,
            "d2h_bytes_per_step": B * 8, "steps": e2e_steps,
            "path": "B200Sampler.select_batch(pinned host logits, List[List[int]] histories) -> List[int]"}


def run_ours(args, world, rank, local):
    from b200_sampler.workloads import WORKLOADS

    dev = torch.device("cuda", local)
    w = WORKLOADS[args.workload]()
    B, V, H = w.batch, w.vocab, w.history_len
    esz = w.logits.element_size()
    r0, r1 = rank * B // world, (rank + 1) * B // world
    clk = ClockSampler(local)
    ms_step, all_ms, first_ids, (per, reps, rem, nb) = measure_rows(args, world, dev, w, r0, r1, clk)
    tokens_per_s = B / (ms_step / 1e3)
    # roofline of the dominant kernel: algorithmic bytes of the rows this
    # rank launched over the launch's average device time (max over ranks)
    peak, peak_kind = _peaks()
    alg = algorithmic_bytes(r1 - r0, V, H, esz)
    achieved = alg / (ms_step / 1e3) / 1e9

    weak = None
    if world > 1:
        ms_w, _, _, _ = measure_rows(args, world, dev, w, 0, B)
        weak = {"value": B * world / (ms_w / 1e3), "unit": UNIT, "ms_per_step": ms_w,
                "global_batch": B * world, "rows_per_gpu": B, "scaling": "weak",
                "note": "every rank samples its own full copy of the batch"}

    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, world, w, dev, r0, r1)

    line = {"metric": metric_for(args.workload), "value": tokens_per_s, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32" if esz == 4 else "bf16",
            "data": "synthetic (seeded)",
            "config": {"workload": w.notes, "name": args.workload, "global_batch": B, "rows_per_gpu": r1 - r0,
                       "vocab": V,
                       "parallelism": f"one batch sharded by rows over {world} GPU(s), no collective",
                       "l2": f"{nb} rotating logits buffers ({nb * (r1 - r0) * V * esz / 1e6:.0f} MB per GPU, "
                             f">= {L2_MULTIPLE}x the L2): no timed launch finds its logits in L2",
                       "timing": f"CUDA graphs ({per} launches x {reps} replays{f' + {rem}' if rem else ''}) "
                                 f"= K steps per repeat, {len(all_ms)} repeats >= {MIN_TIMED_S:.0f} s, median "
                                 f"repeat, CUDA events, max over ranks",
                       "ms_per_step_repeats": [round(m, 6) for m in all_ms]},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind,
                         "traffic": NCU_TRAFFIC_BYTES if (args.workload == "headline" and world == 1) else None,
                         "traffic_source": NCU_TRAFFIC_SOURCE if (args.workload == "headline" and world == 1)
                         else "not recorded for this workload",
                         "algorithmic_bytes_per_launch": alg},
            "gpu_launches": args.steps}
    if weak is not None:
        line["weak_scaling"] = weak
    if e2e is not None:
        line["e2e"] = e2e
    clocks = clk.summary()
    if clocks is not None:
        line["clocks"] = clocks
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        # parity of every row of the benchmarked launch, then the CPU sampler
        # on a bounded sample (~10-30 s) at all host threads
        gate = parity_gate(w, first_ids)
        line["parity"] = gate
        threads = os.cpu_count() or 1
        rows = min(B, 16)
        _, t1, _, _ = cpu_rate(w, rows, 1, threads)
        rows = int(min(B, max(rows, rows * 10.0 / max(t1, 1e-6))))
        rate, dtc, kind, note = cpu_rate(w, rows, 1, threads)
        line["cpu_baseline"] = {"value": rate, "unit": UNIT, "cores": threads, "kind": kind,
                                "sample": f"{rows} of {B} rows of the workload, one select_batch "
                                          f"({dtc:.1f} s), {note}, {threads} threads"}
        if not gate["ok"]:
            print(json.dumps(line), flush=True)
            raise SystemExit(f"parity gate failed: {gate}")
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_vp(args, world, rank, local):
    """Benchmark configuration 4: vocab-parallel sampling, B=128 rows of V=151936 fp32
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
    nb = n_buffers(dev, B * width * 4)   # this rank's slices, >= L2_MULTIPLE x the L2 in total
    bufs = [full[:, off:off + width].contiguous().to(dev)]
    for i in range(1, nb):
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
        x = bufs[i % nb]
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

    def run_k():
        for _ in range(reps):
            g.replay()
        if g_rem is not None:
            g_rem.replay()
    with ClockSampler(local) as clk:
        ms, all_ms = timed_repeats(world, dev, side, run_k)
    del g, g_rem  # graphs holding NCCL calls go before the process group
    if peer:
        ex.release(side)
    ms_per_step = ms / args.steps
    peak, peak_kind = _peaks()
    local_bytes = B * width * 4
    line = {"metric": "vocab-parallel sampled tokens/sec at B=128,V=151936 (benchmark configuration 4)",
            "value": B / (ms_per_step / 1e3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded randn*3 logits)",
            "config": {"workload": f"B={B} V={V} fp32 split into {world} slices of <= {w}; T=0.8 k={K} p=0.95",
                       "record_bytes_per_rank": int(n.value) * 8,
                       "l2": f"{nb} rotating logits slices per GPU ({nb * B * width * 4 / 1e6:.0f} MB, "
                             f">= {L2_MULTIPLE}x the L2)",
                       "transport": ("peer: records read in place over NVLink by the merge kernel after a "
                                     "flag signal" if peer else "gather: NCCL all-gather of the records"),
                       "timing": f"CUDA graphs of local + exchange + merge ({per} steps x {reps}"
                                 f"{f' + {rem}' if rem else ''}) = K steps per repeat, {len(all_ms)} repeats "
                                 f">= {MIN_TIMED_S:.0f} s, median repeat, CUDA events, max over ranks"},
            "roofline": {"bound": "hbm", "achieved": local_bytes / (ms_per_step / 1e3) / 1e9, "peak": peak,
                         "unit": "GB/s", "frac": local_bytes / (ms_per_step / 1e3) / 1e9 / peak,
                         "traffic": None, "peak_kind": peak_kind, "algorithmic_bytes_per_launch": local_bytes},
            "gpu_launches": (3 if peer else 2) * args.steps}
    clocks = clk.summary()
    if clocks is not None:
        line["clocks"] = clocks
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_decode(args, world, rank, local):
    """Benchmark configuration 5: an end-to-end decode loop.  A Qwen3-0.6B-shaped
    model (28 layers, hidden 1024, 16 query / 8 KV heads, head_dim 128,
    vocab 151936; transformers' Qwen3 with random-init bf16 weights), batch
    64, 128-token random prompts, 256 decode steps, each sampled through
    ``B200Sampler.select_batch_tensor`` with top-k 20 / top-p 0.8 / T 0.7 and
    the growing histories.  The sampler reads ``logits[:, -1, :]`` of the
    model's bf16 [B, S, V] output in place (row stride S x V) -- the
    reference stacks ``.float()`` copies of those rows
    (inferencer/torch_inferencer.py:242-251).  Reports decode tokens/s and
    the sampler's share of the step time (CUDA events around each call).
    One GPU; with N ranks each runs its own replica."""
    from transformers import Qwen3Config, Qwen3ForCausalLM
    from b200_sampler import B200Sampler
    from b200_sampler.params import SamplingParams

    dev = torch.device("cuda", local)
    B, P, steps = 64, 128, args.decode_steps
    cfg = Qwen3Config(vocab_size=151936, hidden_size=1024, intermediate_size=3072, num_hidden_layers=28,
                      num_attention_heads=16, num_key_value_heads=8, head_dim=128,
                      max_position_embeddings=P + steps + 8, tie_word_embeddings=True)
    torch.manual_seed(1234 + rank)
    with torch.device(dev):
        model = Qwen3ForCausalLM(cfg).to(torch.bfloat16).eval()
    g = torch.Generator().manual_seed(99 + rank)
    prompt = torch.randint(0, cfg.vocab_size, (B, P), generator=g)
    params = [SamplingParams(temperature=0.7, top_k=20, top_p=0.8)] * B
    sampler = B200Sampler(device=dev, seed=5 + rank)
    e_s = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    e_e = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]

    def generate(n_steps, timed):
        hist = [list(map(int, r)) for r in prompt]
        ids = prompt.to(dev)
        with torch.inference_mode():
            out = model(input_ids=ids, use_cache=True)
            pkv = out.past_key_values
            x = out.logits[:, -1, :]                     # [B, V] bf16 view, row stride P x V
            assert x.stride(1) == 1 and x.stride(0) == P * cfg.vocab_size
            for t in range(n_steps + 1):
                if timed:
                    e_s[t].record()
                nxt = sampler.select_batch_tensor(x, hist, params)
                if timed:
                    e_e[t].record()
                new = nxt.tolist()
                assert min(new) >= 0, new
                for b in range(B):
                    hist[b].append(new[b])
                if t == n_steps:
                    break
                out = model(input_ids=nxt[:, None], past_key_values=pkv, use_cache=True)
                pkv = out.past_key_values
                x = out.logits[:, -1, :]
        return hist

    def generate_device(n_steps, timed):
        """The same loop with the histories on the device: DeviceBatch reads
        them from a DeviceHistory and ns_hist_append adds each step's ids --
        no host lists, no per-step .tolist(); the ids feed the next step
        directly."""
        from b200_sampler.sampler import DeviceBatch, DeviceHistory
        dh = DeviceHistory([list(map(int, r)) for r in prompt], dev, reserve_steps=n_steps + 2)
        db = DeviceBatch(None, params, dev, seed=5 + rank, history=dh)
        nxt = torch.empty(B, dtype=torch.int64, device=dev)
        ids = prompt.to(dev)
        with torch.inference_mode():
            out = model(input_ids=ids, use_cache=True)
            pkv = out.past_key_values
            x = out.logits[:, -1, :]
            for t in range(n_steps + 1):
                if timed:
                    e_s[t].record()
                assert db.launch(x, nxt, offset=t) == 0
                dh.append(nxt)
                if timed:
                    e_e[t].record()
                if t == n_steps:
                    break
                out = model(input_ids=nxt[:, None].clone(), past_key_values=pkv, use_cache=True)
                pkv = out.past_key_values
                x = out.logits[:, -1, :]
        return dh

    # warm-up over every step: each decode step meets a new KV length, and
    # the eager model's first use of a shape is slow; both timed loops below
    # then run on warm shapes
    generate(steps, False)
    torch.cuda.synchronize(dev)
    barrier(world)
    t0 = time.perf_counter()
    hist = generate(steps, True)
    torch.cuda.synchronize(dev)
    dt = time.perf_counter() - t0
    sampler_ms = sum(a.elapsed_time(b) for a, b in zip(e_s, e_e))
    dt = max_over_ranks(world, dt)

    generate_device(4, False)                            # warm-up
    torch.cuda.synchronize(dev)
    barrier(world)
    t0 = time.perf_counter()
    dh = generate_device(steps, True)
    torch.cuda.synchronize(dev)
    dt_dev = max_over_ranks(world, time.perf_counter() - t0)
    sampler_ms_dev = sum(a.elapsed_time(b) for a, b in zip(e_s, e_e))
    dev_lists = dh.to_lists()
    assert min(min(r[P:]) for r in dev_lists) >= 0, "a device-history step reported a failed row"
    line = {"metric": "end-to-end decode tokens/sec, Qwen3-0.6B shape (benchmark configuration 5)",
            "value": B * world * (steps + 1) / dt, "unit": UNIT, "n_gpus": world, "steps": steps,
            "warmup": steps, "ms_per_step": dt / (steps + 1) * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (random-init weights, random prompts)",
            "config": {"workload": f"Qwen3-0.6B shape, B={B}, {P}-token prompts, {steps} decode steps, "
                                   "k=20 p=0.8 T=0.7, histories = prompt + outputs",
                       "model": "transformers Qwen3ForCausalLM (eager, DynamicCache), random init bf16",
                       "sampler_feed": "logits[:, -1, :] of the bf16 [B, S, V] output, in place via row_stride"},
            "sampler": {"ms_total": sampler_ms, "share_of_step_time": sampler_ms / 1e3 / dt,
                        "ms_per_call": sampler_ms / (steps + 1),
                        "note": "CUDA events around select_batch_tensor (host packing of the growing "
                                "histories, H2D, the kernel)"},
            "tokens_generated_per_row": len(hist[0]) - P,
            "device_history": {
                "value": B * world * (steps + 1) / dt_dev, "unit": UNIT, "ms_per_step": dt_dev / (steps + 1) * 1e3,
                "sampler_ms_total": sampler_ms_dev, "sampler_share_of_step_time": sampler_ms_dev / 1e3 / dt_dev,
                "sampler_ms_per_call": sampler_ms_dev / (steps + 1),
                "note": "DeviceBatch + DeviceHistory: histories stay on the device (ns_hist_append per step), "
                        "ids feed the next step without .tolist(); CUDA events around the launch and the append"}}
    if rank == 0:
        print(json.dumps(line), flush=True)


def main():
    from b200_sampler.workloads import WORKLOADS
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="headline", choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end leg (profiling runs)")
    ap.add_argument("--vp-transport", default="peer", choices=["peer", "gather"],
                    help="vp mode: records read in place over NVLink (peer) or all-gathered (gather)")
    ap.add_argument("--mode", default="rows", choices=["rows", "vp", "decode"],
                    help="rows: the workload sharded by rows; vp: vocab-parallel config 4; "
                         "decode: the config 5 decode loop")
    ap.add_argument("--decode-steps", type=int, default=256)
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
        elif args.mode == "decode":
            run_decode(args, world, rank, local)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()

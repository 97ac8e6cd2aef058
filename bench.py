#!/usr/bin/env python3
"""Benchmark of the B200 token sampler (the hot path of BASELINE.json).

Headline workload (config C3): one full-vocabulary sampling pass over
B=256 rows x V=262144 bf16 logits, top-k disabled, T=1, top-p 0.95, one draw
per row -- a streaming, HBM-bound pass.  `value` is sampled rows/s of the whole
job (all ranks; rows are independent, so N GPUs each sample their own 256 rows:
weak scaling, no collective on the data path).  Also reported:
  latency_b1   p50/p90 device us/step of config C1 (B=1 fp32, top-k 64, top-p 0.95)
  roofline     algorithmic bytes / mean launch time of the sampling kernel vs
               the measured HBM copy bandwidth (MEASURED_PEAKS.json)
  e2e          rows/s through g4s_sample_host from pinned host memory (PCIe in
               the timed region)
  cpu_baseline the reference algorithm (oracle port of DoSample) on host cores

`--impl reference` times the reference's own algorithm for the path (the C
oracle port: the Delphi reference cannot be built here) on all host cores, on
the same config and metric.
"""
import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "gemma4.pas_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "sampled rows/s at V=262144 B=256 (% HBM peak); p50 µs/step at B=1"
ROWS, VOCAB, SOFTCAP = 256, 262144, 30.0
BYTES_PER_ROW = VOCAB * 2  # bf16 logits read once
FALLBACK_HBM_GBS = 6650.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-c4", action="store_true", help="skip the config C4 (LM head) record")
    ap.add_argument("--no-c5", action="store_true", help="skip the config C5 record")
    ap.add_argument("--only", choices=["c4"], default=None,
                    help="run config C4 alone and print its record (for profiling)")
    return ap.parse_args()


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def load_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic():
    """DRAM bytes per launch of the full-path streaming kernel from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "full_etab_kernel_c3.md")
    try:
        m = re.search(r"dram_bytes_per_launch:\s*([0-9]+)", open(path).read())
        return int(m.group(1)) if m else None
    except OSError:
        return None


class Clocks:
    """SM clock and throttle reasons sampled every ~2 ms through NVML (read-only
    queries) in a background thread while the timed region runs; nvidia-smi at
    100 ms when NVML is unavailable."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4}

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.samples = []
        self.run = False
        self.thread = None
        self.proc = None
        self.nvml = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nvml = pynvml
            uuid = None
            try:
                import torch

                uuid = "GPU-" + str(torch.cuda.get_device_properties(gpu_index).uuid)
            except Exception:
                pass
            self.h = (pynvml.nvmlDeviceGetHandleByUUID(uuid) if uuid else
                      pynvml.nvmlDeviceGetHandleByIndex(gpu_index))
            self.smax = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.reasons_fn = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
        except Exception:
            self.nvml = None

    def _poll(self):
        nv = self.nvml
        while self.run:
            try:
                sm = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
                rs = self.reasons_fn(self.h)
                pw = nv.nvmlDeviceGetPowerUsage(self.h) / 1000.0
                self.samples.append((sm, rs, pw))
            except Exception:
                pass
            time.sleep(0.002)

    def start(self):
        if self.nvml is not None:
            import threading

            self.run = True
            self.thread = threading.Thread(target=self._poll, daemon=True)
            self.thread.start()
            return
        try:
            self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.idx), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.thread is not None:
            self.run = False
            self.thread.join()
            if not self.samples:
                return None
            reasons = sorted({n for _, rs, _ in self.samples for n, bit in self.REASONS.items() if rs & bit})
            return {"sm_mhz": statistics.median(s[0] for s in self.samples), "sm_max_mhz": self.smax,
                    "reasons": reasons, "samples": len(self.samples),
                    "power_w_max": max(s[2] for s in self.samples), "source": "NVML, 2 ms"}
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(5)
        except Exception:
            self.proc.kill()
        self.f.flush()
        rows = [[p.strip() for p in line.split(",")] for line in open(self.f.name)]
        os.unlink(self.f.name)
        rows = [r for r in rows if len(r) >= 7 and r[0].replace(".", "").isdigit()]
        if not rows:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        return {"sm_mhz": statistics.median(float(r[0]) for r in rows), "sm_max_mhz": max(float(r[1]) for r in rows),
                "reasons": sorted({names[i] for r in rows for i in range(4) if r[3 + i].lower() == "active"}),
                "samples": len(rows), "source": "nvidia-smi, 100 ms"}


def dist_setup(n):
    import torch

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n:
        raise SystemExit(f"--gpus {n} but WORLD_SIZE={world}")
    if n > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def allreduce_max(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def c3_config(world):
    """The headline workload, described identically by both arms of the bench."""
    return {"workload": "C3 full-vocab sampling, B=256 x V=262144 bf16 per GPU, top_k=0, T=1, top_p=0.95, softcap 30",
            "global_batch": ROWS * world, "seq_len": VOCAB,
            "parallelism": f"row-sharded x{world} (independent rows, no collective)",
            "l2": "4 rotating input sets of 128 MiB (512 MiB > 126 MB L2)",
            "timing": "K steps per timed window (CUDA graphs of up to 250 calls, each replayed once untimed); "
                      "the window is repeated (15 times at K = 20) and its median reported; CUDA events, max over "
                      "ranks"}


def cpu_reference(rows_bf16, u, nthreads, min_cpu_s=10.0):
    """The reference algorithm (oracle port of DoSample, fp32 transcription) on host
    threads; repeats the sample until ~min_cpu_s of CPU work.  Returns rows/s."""
    from oracle import oracle as O

    p = O.params(1.0, 0, 0.95)
    done, t0 = 0, time.perf_counter()
    while True:
        O.sample_batch(rows_bf16, O.DTYPE_BF16, p, SOFTCAP, u, O.VARIANT_F32, O.TIE_HEAP, nthreads)
        done += rows_bf16.shape[0]
        el = time.perf_counter() - t0
        if el * nthreads >= min_cpu_s:
            return done / el, done, el


def one_core_us_per_row(rows_bf16, u):
    """The reference algorithm on one host thread: microseconds per C3 row."""
    from oracle import oracle as O

    p = O.params(1.0, 0, 0.95)
    O.sample_batch(rows_bf16[:1], O.DTYPE_BF16, p, SOFTCAP, u[:1], O.VARIANT_F32, O.TIE_HEAP, 1)
    t0 = time.perf_counter()
    O.sample_batch(rows_bf16, O.DTYPE_BF16, p, SOFTCAP, u, O.VARIANT_F32, O.TIE_HEAP, 1)
    return (time.perf_counter() - t0) * 1e6 / rows_bf16.shape[0]


def verify_c3(rows_bf16, u, got, nthreads):
    """Tokens of one C3 step against the oracle: equal to the fp64 restatement
    except draws within 1e-6 of a CDF boundary (counted); also how often the
    reference's own fp32 arithmetic (serial sums) picks another token."""
    import numpy as np

    from oracle import oracle as O

    p = O.params(1.0, 0, 0.95)
    t64 = O.sample_batch(rows_bf16, O.DTYPE_BF16, p, SOFTCAP, u, O.VARIANT_F64, O.TIE_LOWER, nthreads)
    t32 = O.sample_batch(rows_bf16, O.DTYPE_BF16, p, SOFTCAP, u, O.VARIANT_F32, O.TIE_LOWER, nthreads)
    boundary, bad = 0, 0
    for r in np.nonzero(got != t64)[0]:
        _, tr, _, _ = O.sample(O.as_f32(rows_bf16[r]), p, SOFTCAP, u[r], O.VARIANT_F64)
        if tr["boundary"] < 1e-6:
            boundary += 1
        else:
            bad += 1
    return {"rows": int(len(got)), "tokens_match_f64": int((got == t64).sum()), "boundary_rows": boundary,
            "mismatch_outside_band": bad, "ref_f32_vs_f64_rows": int((t32 != t64).sum())}


def run_reference(args, emit):
    """--impl reference: the reference's algorithm for the path on the host cores."""
    import numpy as np

    import synth

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    nthreads = host_threads()
    xb = synth.c3_logits(ROWS, step=0)
    u = synth.uniforms(ROWS * (args.steps + args.warmup), synth.SEEDS["c3"]).reshape(-1, ROWS)
    from oracle import oracle as O

    O.load()
    p = O.params(1.0, 0, 0.95)
    for w in range(args.warmup):
        O.sample_batch(xb[:nthreads], O.DTYPE_BF16, p, SOFTCAP, u[w][:nthreads], O.VARIANT_F32, O.TIE_HEAP, nthreads)
    t0 = time.perf_counter()
    for s in range(args.steps):
        O.sample_batch(xb, O.DTYPE_BF16, p, SOFTCAP, u[args.warmup + s], O.VARIANT_F32, O.TIE_HEAP, nthreads)
    el = time.perf_counter() - t0
    value = ROWS * args.steps / el
    line = {
        "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": el * 1e3 / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "impl": "reference",
        "config": c3_config(args.gpus),
        "cpu_baseline": {"value": value, "unit": "rows/s", "cores": nthreads, "kind": "port",
                         "sample": f"all {ROWS} rows per step, {args.steps} steps; C oracle port of "
                                   "TModel.DoSample (the Delphi reference does not build here)"},
        "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(line)


def run_c4(dev, peak, steps=20):
    """Config C4: LM head (64 x 2560 hidden, 262144 x 2560 Q4_0 weights, 377 MB)
    + top-K sampling, one g4s_lmhead_sample call per step; device time per step
    from a CUDA graph of `steps` calls (weights 377 MB > L2: streamed each step)."""
    import torch

    import g4sampler as g4
    import synth

    rows, H = 64, 2560
    h, blocks = synth.c4_inputs(rows, H, VOCAB)
    bd = torch.from_numpy(blocks).to(dev)
    nib = torch.empty(VOCAB * H // 2, dtype=torch.uint8, device=dev)
    sc = torch.empty(VOCAB * H // 32, dtype=torch.int16, device=dev)
    g4.q4_repack(bd.data_ptr(), VOCAB, H, nib.data_ptr(), sc.data_ptr())
    torch.cuda.synchronize()
    del bd
    hd = torch.from_numpy(h).to(dev)
    u = torch.from_numpy(synth.uniforms(rows, synth.SEEDS["c4"])).to(dev)
    out = torch.empty(rows, dtype=torch.int32, device=dev)
    s = g4.Sampler(dev.index or 0, rows, VOCAB)
    p = g4.make_params(1.0, 64, 0.95)
    cap = torch.cuda.Stream(device=dev)

    def call(st=None, mask=0):
        o = g4.Outputs()
        o.phase_mask = mask
        s.lmhead_sample(hd.data_ptr(), rows, H, nib.data_ptr(), sc.data_ptr(), VOCAB, p, SOFTCAP, u.data_ptr(),
                        out.data_ptr(), outputs=o, stream=st)

    def timed(mask):
        for _ in range(3):
            call(mask=mask)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=cap):
            for _ in range(steps):
                call(cap.cuda_stream, mask)
        g.replay()
        torch.cuda.synchronize()
        ts = []
        for _ in range(5):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()  # replay runs on the current stream
            g.replay()
            b.record()
            b.synchronize()
            ts.append(a.elapsed_time(b) * 1e3 / steps)
        del g
        return ts, out.cpu().numpy().copy()

    # default: top-K selection in the LM head's epilogue; unfused: the logits
    # written to memory and sampled by the top-K kernels
    ts, tok_fused = timed(0)
    ts_unfused, tok_unfused = timed(g4.PHASE_LMHEAD_UNFUSED)
    # agreement with the reference's own LM-head arithmetic on a few rows: the
    # fp32 CpuMatVecQ4 and the Q8_1 + DP4A path of its GPU shaders, each
    # followed by the oracle's DoSample
    from oracle import oracle as O

    cid = torch.full((rows, 64), -1, dtype=torch.int32, device=dev)
    o = g4.Outputs()
    o.cand_ids, o.cand_stride = cid.data_ptr(), 64
    s.lmhead_sample(hd.data_ptr(), rows, H, nib.data_ptr(), sc.data_ptr(), VOCAB, p, SOFTCAP, u.data_ptr(),
                    out.data_ptr(), outputs=o)
    torch.cuda.synchronize()
    s.close()
    tok, ids = out.cpu().numpy(), cid.cpu().numpy()
    uh = u.cpu().numpy()
    agree = {"rows": 0, "tokens_vs_f32": 0, "tokens_vs_q8": 0, "survivors_vs_f32": 0.0, "survivors_vs_q8": 0.0}
    for r in range(0, rows, 16):
        for name, lg in (("f32", O.matvec_q4_mt(blocks, h[r], VOCAB, H, host_threads())),
                         ("q8", O.matvec_q4q8(blocks, h[r], VOCAB, H, host_threads()))):
            t, _, rid, _ = O.sample(lg, O.params(1.0, 64, 0.95), SOFTCAP, uh[r], O.VARIANT_F32, O.TIE_LOWER)
            agree["tokens_vs_" + name] += int(t == tok[r])
            agree["survivors_vs_" + name] += len(set(rid.tolist()) & set(ids[r].tolist())) / 64.0
        agree["rows"] += 1
    us = statistics.median(ts)
    wbytes = VOCAB * (H // 32) * 18
    return {"us_per_step": us, "rows_per_s": rows / (us * 1e-6), "weight_gbs": wbytes / (us * 1e-6) / 1e9,
            "hbm_frac_of_peak": wbytes / (us * 1e-6) / 1e9 / peak,
            "tflops": 2.0 * rows * VOCAB * H / (us * 1e-6) / 1e12,
            "unfused_us_per_step": statistics.median(ts_unfused),
            "tokens_fused_equal_unfused": int((tok_fused == tok_unfused).sum()),
            "agreement_with_reference_lmhead": agree,
            "config": "C4: hidden 64 x 2560 fp32 -> LM head 262144 x 2560 Q4_0 (tcgen05 fp16 MMA, dequantized "
                      "weights in TMEM, fp32 accumulate) with top-K selection in its epilogue -> top_k 64, T=1, "
                      "top_p 0.95; median of 5 replays of a 20-call CUDA graph; unfused_us_per_step: the same "
                      "with the logits written to memory and sampled by the top-K kernels"}


def run_c5(rank, world, local, dev, peak, steps=50):
    """Config C5: 1024 fp32 rows x V=262144, per-row T, top-K, top-P.

    N = 1: plain g4s_sample on the whole rows (the one-GPU line of this batch).
    N > 1: the vocabulary-sharded mode: every rank holds a contiguous V/world
    slice of every row; per step the slice's top-K lists, two NCCL
    all-gathers, the merge and the draw (g4s_shard_sample).  The rows are the
    same on every rank (one seeded generator), so rank 0 also samples the
    whole rows unsharded on its own GPU and reports how many tokens agree
    (the merge is exact: all of them must).  Phase times come from separate
    timed runs of g4s_shard_lists and g4s_shard_merge on the same inputs;
    the exchange is the step minus the two.  Device time per step, max over
    ranks; two input buffers alternate (each slice >= 128 MiB at N <= 8)."""
    import numpy as np
    import torch

    import g4sampler as g4
    import synth

    rows = 1024
    full = synth.c5_logits(rows)  # identical on every rank
    c5p = synth.c5_params(rows)
    prm = g4.params_array(c5p)  # converted once, reused every step
    u = torch.from_numpy(synth.uniforms(rows, synth.SEEDS["c5"])).to(dev)
    out = torch.empty(rows, dtype=torch.int32, device=dev)
    # a stream of our own: the events below are recorded on it, and its handle
    # is non-zero (a NULL stream would mean the sampler context's own stream)
    cs = torch.cuda.Stream(device=dev)
    stream = cs.cuda_stream
    torch.cuda.set_stream(cs)

    def timed(fn, n):
        for i in range(3):
            fn(i)
        torch.cuda.synchronize()
        barrier(world)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        for i in range(n):
            fn(i)
        t1.record()
        torch.cuda.synchronize()
        return allreduce_max(t0.elapsed_time(t1), world) * 1e3 / n

    rec = {"world": world, "rows": rows}
    single = None
    if rank == 0:
        # the whole batch on one GPU (both N = 1 and the reference point at N > 1)
        xa = torch.from_numpy(full).to(dev)
        sets = [xa, xa.clone()]
        s1 = g4.Sampler(local, rows, VOCAB)

        def one(i):
            s1.sample(sets[i % 2].data_ptr(), g4.F32, rows, VOCAB, VOCAB, prm, SOFTCAP, u.data_ptr(), out.data_ptr(),
                      stream=stream)

        for i in range(3):
            one(i)
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        for i in range(steps):
            one(i)
        t1.record()
        torch.cuda.synchronize()
        us = t0.elapsed_time(t1) * 1e3 / steps
        one(0)
        torch.cuda.synchronize()
        single = out.cpu().numpy().copy()
        s1.close()
        del sets, xa
        rec["single_gpu"] = {"us_per_step": us, "rows_per_s": rows / (us * 1e-6),
                             "hbm_frac_of_peak": rows * VOCAB * 4 / (us * 1e-6) / 1e9 / peak}
    barrier(world)
    if world == 1:
        rec.update(rec.pop("single_gpu"))
        rec["config"] = ("C5 on one GPU: B=1024 x V=262144 fp32, per-row T~U[0.3,1.5], K in {1,20,64,200}, "
                         f"P~U[0.5,1]; g4s_sample, {steps} steps, CUDA events")
        return rec

    lo, hi = g4.shard_slices(VOCAB, world)[rank]
    n = hi - lo
    xs = torch.from_numpy(np.ascontiguousarray(full[:, lo:hi])).to(dev)
    del full
    sets = [xs, xs.clone()]
    sh = g4.Sampler(local, rows, n)
    uid = torch.zeros(g4.SHARD_UID_BYTES, dtype=torch.uint8, device=dev)
    if rank == 0:
        uid.copy_(torch.frombuffer(bytearray(g4.shard_unique_id()), dtype=torch.uint8))
    import torch.distributed as dist

    dist.broadcast(uid, 0)
    sh.shard_init(world, rank, VOCAB, bytes(uid.cpu().numpy().tobytes()))

    def step(i):
        sh.shard_sample(sets[i % 2].data_ptr(), g4.F32, rows, n, prm, SOFTCAP, u.data_ptr(), out.data_ptr(),
                        stream=stream)

    step(0)
    torch.cuda.synchronize()
    got = out.clone()
    allt = [torch.empty_like(got) for _ in range(world)]
    dist.all_gather(allt, got)
    ranks_agree = all(bool(torch.equal(allt[0], t)) for t in allt)
    us = timed(step, steps)
    # phases, each timed alone on the same inputs
    lists = torch.zeros((world, rows, g4.SHARD_LIST), dtype=torch.int64, device=dev)
    counts = torch.zeros((world, rows), dtype=torch.int32, device=dev)
    us_lists = timed(lambda i: sh.shard_lists(sets[i % 2].data_ptr(), g4.F32, rows, n, n, lo, VOCAB, prm, SOFTCAP,
                                              lists[rank].data_ptr(), counts[rank].data_ptr(), stream=stream), steps)
    dist.all_gather_into_tensor(lists.view(-1), lists[rank].contiguous().view(-1))
    dist.all_gather_into_tensor(counts.view(-1), counts[rank].contiguous().view(-1))
    us_merge = timed(lambda i: sh.shard_merge(lists.data_ptr(), counts.data_ptr(), world, rows, VOCAB, prm, SOFTCAP,
                                              u.data_ptr(), out.data_ptr(), stream=stream), steps)
    sh.close()
    if rank == 0:
        rec["tokens_match"] = int((got.cpu().numpy() == single).sum())
    rec["ranks_agree"] = ranks_agree
    rec.update({"rows_per_s": rows / (us * 1e-6), "us_per_step": us,
                "per_gpu_hbm_frac_of_peak": rows * n * 4 / (us * 1e-6) / 1e9 / peak,
                "phases_us": {"lists": us_lists, "merge": us_merge, "exchange": max(0.0, us - us_lists - us_merge)},
                "lists_hbm_frac_of_peak": rows * n * 4 / (us_lists * 1e-6) / 1e9 / peak,
                # each row's own slots (its top_k; 2 for a full-vocabulary row), packed, plus the counts
                "allgather_bytes_per_rank": sum(2 if (k <= 0 or k >= VOCAB) else k for _, k, _ in c5p) * 8 + rows * 4,
                "config": f"C5 sharded: B=1024 x V=262144 fp32, a {n}-id slice per rank; per-row T~U[0.3,1.5], "
                          "K in {1,20,64,200}, P~U[0.5,1]; lists -> ncclAllGather x2 -> merge; "
                          f"{steps} steps, host loop, CUDA events, max over ranks; phases timed alone"})
    return rec


def main():
    args = parse()
    # the one JSON line goes to the original stdout; everything else printed in
    # this process (libraries too, e.g. NCCL's version banner) goes to stderr
    json_fd = os.dup(1)
    sys.stdout.flush()
    os.dup2(2, 1)

    def emit(line):
        os.write(json_fd, (json.dumps(line) + "\n").encode())

    if args.impl == "reference":
        run_reference(args, emit)
        return
    import numpy as np
    import torch

    import g4sampler as g4
    import synth

    rank, world, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    K, W = args.steps, args.warmup
    peak, peak_kind = load_peak()
    if args.only == "c4":
        emit({"c4": run_c4(dev, peak)})
        return

    # ---- inputs: 4 rotating sets of C3 rows (4 x 128 MiB > 126 MB L2) ----
    base = synth.c3_logits(ROWS, step=rank)
    sets = [torch.from_numpy(np.roll(base, k, axis=0).view(np.int16).copy()).to(dev) for k in range(4)]
    u_all = torch.from_numpy(synth.uniforms(ROWS * (K + W), synth.SEEDS["c3"], 100 + rank)).to(dev).view(K + W, ROWS)
    out = torch.empty(ROWS, dtype=torch.int32, device=dev)
    s = g4.Sampler(local, ROWS, VOCAB, g4.FLAG_HOST_STAGING)
    p = g4.make_params(1.0, 0, 0.95)

    def step(i, stream=None):
        s.sample(sets[i % 4].data_ptr(), g4.BF16, ROWS, VOCAB, VOCAB, p, SOFTCAP, u_all[i].data_ptr(),
                 out.data_ptr(), stream=stream)

    torch.cuda.synchronize()
    for i in range(W):
        step(i)
    torch.cuda.synchronize()

    # The timed steps run from CUDA graphs of G consecutive g4s_sample calls: a
    # Python loop of ctypes calls cannot enqueue a ~50 us step as fast as the
    # GPU runs it, and per-call events would time the host.  Exactly K steps are
    # timed: the G-step graph is replayed K // G times, then a graph of the
    # remaining K % G steps.  Each graph is replayed once untimed first.
    cap = torch.cuda.Stream(device=dev)
    G = min(K, 250)

    def capture(nsteps, phase_mask=0):
        o = g4.Outputs()
        o.phase_mask = phase_mask
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=cap):
            for i in range(nsteps):
                j = W + i
                s.sample(sets[j % 4].data_ptr(), g4.BF16, ROWS, VOCAB, VOCAB, p, SOFTCAP, u_all[j % (K + W)].data_ptr(),
                         out.data_ptr(), stream=cap.cuda_stream, outputs=o)
        gr.replay()
        return gr

    def timed(graphs, clocks=None, reps=1):
        """The K steps `graphs` hold, timed `reps` times (each time exactly K
        steps between a barrier + synchronize on both sides, max over ranks);
        returns the median over the repetitions."""
        if clocks:
            clocks.start()
        runs = []
        for _ in range(reps):
            torch.cuda.synchronize()
            barrier(world)
            t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0.record()
            for gr in graphs:
                gr.replay()
            t1.record()
            torch.cuda.synchronize()
            barrier(world)
            runs.append(allreduce_max(t0.elapsed_time(t1), world))
        clk = clocks.stop() if clocks else None
        return statistics.median(runs), clk, runs

    g_main = capture(G)
    g_rest = capture(K % G) if K % G else None
    plan = [g_main] * (K // G) + ([g_rest] if g_rest else [])
    # short K (the driver's K = 20 is ~1 ms of work): repeat the K-step window
    # and take the median, so one scheduling hiccup or rank skew does not decide
    reps = max(1, min(15, int(20000 // max(K, 1))))
    total_ms_max, clk, rep_ms = timed(plan, Clocks(local), reps)
    value = world * ROWS * K / (total_ms_max / 1e3)
    tokens_ok = bool(((out >= 0) & (out < VOCAB)).all().item())
    # one step of the timed workload, checked against the oracle (rank 0)
    check = None
    if rank == 0:
        s.sample(sets[0].data_ptr(), g4.BF16, ROWS, VOCAB, VOCAB, p, SOFTCAP, u_all[0].data_ptr(), out.data_ptr())
        torch.cuda.synchronize()
        check = verify_c3(base, u_all[0].cpu().numpy(), out.cpu().numpy(), host_threads())
    # the dominant kernel alone: the same steps with only the streaming pass
    # (G4S_PHASE_FULL_STREAM_ONLY), for the roofline's achieved bandwidth
    gs_main = capture(G, 1)
    gs_rest = capture(K % G, 1) if K % G else None
    stream_ms, _, _ = timed([gs_main] * (K // G) + ([gs_rest] if gs_rest else []), None, reps)
    stream_us = stream_ms / K * 1e3
    achieved = ROWS * BYTES_PER_ROW / (stream_us * 1e-6) / 1e9
    del plan, g_main, g_rest, gs_main, gs_rest

    # ---- latency at B=1 (config C1: fp32, top_k 64, top_p 0.95) ----
    # (i) in a decode loop the sampler is one node of a captured step: device
    #     time per call inside a CUDA graph of 20 consecutive calls (each on a
    #     fresh row), p50/p90 over 200 replays; (ii) one call as a graph of its
    #     own (adds the graph launch, ~8 us on this box for a one-kernel graph).
    lat = None
    c2 = None
    if rank == 0:
        n1 = 20
        c1 = torch.from_numpy(np.stack([synth.c1_logits(i) for i in range(n1)])).to(dev)
        u1 = torch.from_numpy(synth.uniforms(n1, synth.SEEDS["c1"])).to(dev)
        p1 = g4.make_params(1.0, 64, 0.95)
        o1 = torch.empty(n1, dtype=torch.int32, device=dev)

        def call1(i, st=None):
            s.sample(c1[i].data_ptr(), g4.F32, 1, VOCAB, VOCAB, p1, SOFTCAP, u1[i:].data_ptr(), o1[i:].data_ptr(),
                     stream=st)

        for i in range(n1):
            call1(i)
        torch.cuda.synchronize()

        def replay_times(gr, reps):
            gr.replay()
            torch.cuda.synchronize()
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
            for e0, e1 in ev:
                e0.record()
                gr.replay()
                e1.record()
                e1.synchronize()
            return sorted(e0.elapsed_time(e1) * 1e3 for e0, e1 in ev)

        gl = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gl, stream=cap):
            for i in range(n1):
                call1(i, cap.cuda_stream)
        lt = [t / n1 for t in replay_times(gl, 200)]
        g1 = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g1, stream=cap):
            call1(0, cap.cuda_stream)
        ls = replay_times(g1, 200)
        # After a producer, as in a decode step: each call samples a row that a
        # kernel just wrote (a 1 MiB device copy standing in for the LM head),
        # so consecutive sampler calls cannot overlap each other.  The step's
        # latency is the graph [copy -> sample] x 20 minus the graph [copy] x 20.
        work = torch.empty(VOCAB, dtype=torch.float32, device=dev)

        def call_w(i, st):
            s.sample(work.data_ptr(), g4.F32, 1, VOCAB, VOCAB, p1, SOFTCAP, u1[i:].data_ptr(), o1[i:].data_ptr(),
                     stream=st)

        gp = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gp, stream=cap):
            for i in range(n1):
                work.copy_(c1[i])
                call_w(i, cap.cuda_stream)
        gq = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gq, stream=cap):
            for i in range(n1):
                work.copy_(c1[i])
        tq = statistics.median(replay_times(gq, 200)) / n1
        tp = sorted(t / n1 - tq for t in replay_times(gp, 200))
        lat = {"p50_us": tp[len(tp) // 2], "p90_us": tp[int(len(tp) * 0.9)],
               "pipelined_p50_us": lt[len(lt) // 2], "pipelined_p90_us": lt[int(len(lt) * 0.9)],
               "single_graph_p50_us": ls[len(ls) // 2], "single_graph_p90_us": ls[int(len(ls) * 0.9)],
               "producer_us": tq, "steps": 200 * n1,
               "config": "C1: B=1 x V=262144 fp32 (fresh row per call), top_k 64, T=1, top_p 0.95.  p50_us: one "
                         "step after a producer -- graph of 20 x [1 MiB copy writing the row -> g4s_sample] minus "
                         "graph of 20 x [copy], per step, p50/p90 over 200 replays; pipelined: 20 consecutive calls "
                         "in one graph (call i+1's launch overlaps call i); single_graph: one call per graph replay "
                         "(includes the graph launch)"}
        del gl, g1, gp, gq

        # ---- config C2: B=32 fp32 rows, T=0.7, top_k 40, top_p 0.9 (HBM-bound top-K) ----
        nset, k2 = 8, 200
        c2sets = [torch.from_numpy(synth.c2_logits(32, step=i)).to(dev) for i in range(nset)]
        u2 = torch.from_numpy(synth.uniforms(32, synth.SEEDS["c2"])).to(dev)
        o2 = torch.empty(32, dtype=torch.int32, device=dev)
        p2 = g4.make_params(0.7, 40, 0.9)
        for i in range(nset):
            s.sample(c2sets[i].data_ptr(), g4.F32, 32, VOCAB, VOCAB, p2, SOFTCAP, u2.data_ptr(), o2.data_ptr())
        torch.cuda.synchronize()
        g2 = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g2, stream=cap):
            for i in range(k2):
                s.sample(c2sets[i % nset].data_ptr(), g4.F32, 32, VOCAB, VOCAB, p2, SOFTCAP, u2.data_ptr(),
                         o2.data_ptr(), stream=cap.cuda_stream)
        t2 = statistics.median(replay_times(g2, 5)) / k2
        s.sample(c2sets[0].data_ptr(), g4.F32, 32, VOCAB, VOCAB, p2, SOFTCAP, u2.data_ptr(), o2.data_ptr())
        torch.cuda.synchronize()
        from oracle import oracle as O

        x2 = synth.c2_logits(32, step=0)
        u2h = u2.cpu().numpy()
        want2 = O.sample_batch(x2, O.DTYPE_F32, O.params(0.7, 40, 0.9), SOFTCAP, u2h, O.VARIANT_F32, O.TIE_LOWER,
                               host_threads())
        ties2 = sum(int(not np.array_equal(np.sort(O.topk(x2[r], 40, O.TIE_HEAP)), np.sort(O.topk(x2[r], 40, O.TIE_LOWER))))
                    for r in range(32))
        c2 = {"rows_per_s": 32 / (t2 * 1e-6), "us_per_step": t2,
              "tokens_match_oracle": int((o2.cpu().numpy() == want2).sum()), "heap_tie_rows": ties2,
              "hbm_frac_of_peak": 32 * VOCAB * 4 / (t2 * 1e-6) / 1e9 / peak,
              "config": "C2: B=32 x V=262144 fp32, T=0.7, top_k 40, top_p 0.9; 8 rotating input sets "
                        "(256 MiB > L2); 200 calls per CUDA graph, median of 5 replays"}
        del g2, c2sets

    c4 = run_c4(dev, peak) if rank == 0 and not args.no_c4 else None
    # ---- end to end through g4s_sample_host (pinned host memory, PCIe inside) ----
    e2e = None
    if not args.no_e2e:
        hb = torch.from_numpy(base.view(np.int16)).pin_memory()
        hn = hb.numpy().view(np.uint16)
        hu = synth.uniforms(ROWS, 7, rank)
        htok = torch.empty(ROWS, dtype=torch.int32).pin_memory().numpy()
        ke = max(3, min(K, 20))
        for _ in range(2):
            s.sample_host(hn, g4.BF16, p, SOFTCAP, hu, htok)
        barrier(world)
        t0 = time.perf_counter()
        for _ in range(ke):
            s.sample_host(hn, g4.BF16, p, SOFTCAP, hu, htok)
        el = allreduce_max(time.perf_counter() - t0, world)
        e2e = {"value": world * ROWS * ke / el, "unit": "rows/s",
               "h2d_bytes_per_step": ROWS * BYTES_PER_ROW + ROWS * 8, "d2h_bytes_per_step": ROWS * 4,
               "steps": ke, "timing": "host wall clock around synchronous g4s_sample_host calls"}

    # ---- CPU baseline: the reference algorithm on host cores (rank 0, N=1) ----
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        nt = host_threads()
        sample = base[:64]
        rps, done, el = cpu_reference(sample, synth.uniforms(64, 3), nt)
        us1 = one_core_us_per_row(base[:8], synth.uniforms(8, 4))
        cpu = {"value": rps, "unit": "rows/s", "cores": nt, "kind": "port",
               "us_per_row_1core": us1,
               "sample": f"{done} C3 rows ({64}-row sample repeated, {el:.1f} s wall on {nt} threads); "
                         "C oracle port of TModel.DoSample, fp32 transcription; us_per_row_1core: 8 rows on one "
                         "thread, as the reference's single-threaded DoSample"}

    s.close()
    c5 = run_c5(rank, world, local, dev, peak) if not args.no_c5 else None
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": total_ms_max / K, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": c3_config(world),
            "timed_windows_ms": rep_ms,
            "hbm_frac_of_peak": ROWS * BYTES_PER_ROW / (total_ms_max / K * 1e-3) / 1e9 / peak,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": profiled_traffic(),
                         "traffic_source": "static: dram__bytes_read + dram__bytes_write of one launch in the "
                                           "committed ncu capture (profiles/full_etab_kernel_c3.md), not measured "
                                           "in this run",
                         "kernel": "full_etab_kernel (bf16 weight-table streaming pass), timed alone (phase_mask = stream only), "
                                   "CUDA events over K launches",
                         "kernel_mean_us": stream_us,
                         "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json), burst copy",
                         "algorithmic_bytes_per_launch": ROWS * BYTES_PER_ROW,
                         "step_us": total_ms_max / K * 1e3,
                         "step_hbm_frac": ROWS * BYTES_PER_ROW / (total_ms_max / K * 1e-3) / 1e9 / peak},
            "latency_b1": lat,
            "c2": c2,
            "c4": c4,
            "c5": c5,
            "e2e": e2e,
            "cpu_baseline": cpu,
            "gpu_launches": 2 * K,
            "clocks": clk,
            "tokens_in_range": tokens_ok,
            "parity_c3": check,
        }
        emit(line)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()

#!/usr/bin/env python3
"""bench.py — batched Needle generation throughput on B200.

Workload (per GPU, weak scaling): 4096 independent requests with prompt
lengths uniform in [64, 512] and token ids uniform over the vocabulary,
64 greedy decode steps each under a constrained-decoding mask (every step a
random vocabulary bitmap with 5% of the entries allowed plus one forced
token).  The model is random-init at the shipped config dims (d=512, 8 Q /
4 KV heads, 12 encoder + 8 decoder layers, V=8192, INT4 group-32
projections), in the reference's SafeTensors format.  One step = prefill of
all prompts + the 64 decode steps.  Requests are sharded over ranks with no
collective (each rank owns its own 4096 requests).

  value  generated tokens/s, all ranks, inputs already in HBM, CUDA events on
         the batch's stream, max over ranks
  e2e    the same through needle_run_batch_ids with pinned host buffers:
         prompt ids + offsets + mask bitmaps in, token ids + lengths out
  --impl reference   the CPU oracle (a C++ restatement of the reference Rust
         path) on the host's cores, same metric, bounded request sample
"""
import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

MEASURED_PEAKS = os.path.join(ROOT, "MEASURED_PEAKS.json")
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
CLASS_NAMES = {1: "cross_attention", 2: "prefill_matmul", 3: "decode_matmul", 4: "head_mask_argmax",
               5: "encoder_attention", 6: "self_attention", 7: "elementwise"}
# classes whose algorithmic work is accounted (candidates for the roofline line)
ROOFLINE_CLASSES = (1, 2, 3, 4, 5)
# DRAM bytes (read + write) per algorithmic byte, from one ncu capture of the
# class's kernel on the 512-request case; a launch reads each encoder K/V row
# once, so its traffic grows in proportion to the rows and scales to the full
# launch.  cross_attention: profiles/cross_attn_decode_512req.md
DRAM_PER_ALG_BYTE = {1: 1.017}
METRIC = "generated tokens/s"


def pkg():
    from __graft_entry__ import _pkg

    return _pkg(), _pkg("needle_workload", "workload.py")


def peaks():
    try:
        p = json.load(open(MEASURED_PEAKS))
        return p, "measured"
    except Exception:
        return FALLBACK_PEAKS, "fallback"


def env_rank():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def workload(args, wl, rank):
    blob = wl.random_model(seed=args.seed)
    ids, off = wl.random_prompts(args.requests, args.min_len, args.max_len, 8192, seed=1000 + 7919 * rank + args.seed)
    masks = wl.random_masks(args.requests, args.max_new, 8192, args.mask_frac, seed=2000 + 7919 * rank + args.seed)
    return blob, ids, off, masks


def config_desc(args):
    return {
        "workload": (f"{args.requests} requests per GPU, prompt length U[{args.min_len},{args.max_len}], "
                     f"{args.max_new} greedy steps, {args.mask_frac:.0%} random vocab mask + 1 forced token; "
                     "random-init model at the shipped dims (d=512, 8/4 heads, 12+8 layers, V=8192, INT4 g32)"),
        "requests_per_gpu": args.requests,
        "prompt_len": [args.min_len, args.max_len],
        "max_new": args.max_new,
        "mask_fraction": args.mask_frac,
        "parallelism": "request-sharded, no collective",
        "l2": "inputs larger than L2 (encoder K/V about 19 GB per GPU)",
    }


_ORACLE = {}


def cpu_sample(args, blob, ids, off, masks, max_seconds):
    """Oracle (C++ restatement of the reference path) on this host's cores
    over a bounded prefix of the same requests -> (tokens/s, threads, n)."""
    import numpy as np
    import oracle

    threads = os.cpu_count() or 1
    key = id(blob)
    if _ORACLE.get("key") != key:
        _ORACLE.update(key=key, model=oracle.Model(data=blob))
    m = _ORACLE["model"]
    done_req, t_total = 0, 0.0
    n = min(args.requests, max(threads, 8))
    while done_req < args.requests:
        r1 = min(args.requests, done_req + n)
        sub_off = off[done_req:r1 + 1] - off[done_req]
        sub_ids = ids[int(off[done_req]):int(off[r1])]
        t0 = time.perf_counter()
        m.run_batch(sub_ids, sub_off, args.max_new, mask_bits=masks[done_req:r1], n_threads=threads)
        t_total += time.perf_counter() - t0
        done_req = r1
        if t_total >= max_seconds:
            break
    return done_req * args.max_new / t_total, threads, done_req, t_total


def run_reference(args):
    rank, world, _ = env_rank()
    if rank != 0:
        return 0
    import numpy as np  # noqa: F401

    _, wl = pkg()
    blob, ids, off, masks = workload(args, wl, 0)
    vals = []
    info = None
    for _ in range(args.warmup):
        cpu_sample(args, blob, ids, off, masks, args.cpu_seconds / 4)
    for _ in range(args.steps):
        v, threads, n, t = cpu_sample(args, blob, ids, off, masks, args.cpu_seconds)
        vals.append(v)
        info = (threads, n, t)
    value = statistics.mean(vals)
    threads, n, t = info
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * n * args.max_new / value,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_desc(args),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": f"first {n} of the {args.requests} requests per step ({t:.1f} s), one request "
                                   f"per host thread; the reference Rust path restated in C++ (oracle/)"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


L2_BYTES = 126e6


def _graph_ms(torch, launch, reps=5):
    """Capture launch(stream_handle) into a CUDA graph; mean ms per replay
    (CUDA events on the replaying stream, a synchronize on both sides)."""
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        launch(s.cuda_stream)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        launch(s.cuda_stream)
    with torch.cuda.stream(s):
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(reps):
            g.replay()
        e1.record(s)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    del g
    return ms


def _cpu_us(fn, budget_s=0.3, min_reps=3):
    fn()
    t0, n = time.perf_counter(), 0
    while n < min_reps or time.perf_counter() - t0 < budget_s:
        fn()
        n += 1
    return 1e6 * (time.perf_counter() - t0) / n


def op_suite(args, nb, wl, torch, np, pk, eng, blob):
    """The other INT4-path workloads, measured beside the headline line.

    int4_gemv   one INT4 matvec, x f32 [1, 512], W [N=2048, K=512] group-32
                (quant.rs:160-297): a chain of R launches over R distinct
                weight copies (R x 665,600 B > 2 x L2) captured in one CUDA
                graph, each launch a separate op; plain launches and
                programmatic-dependent ("overlap") launches.
    int4_sweep  M in {1, 8, 64, 512, 4096} x (N, K) in {(512,512), (2048,512),
                (512,2048), (8192,512)} through a prepared plan: CUDA-core
                matvec up to 8 rows, tcgen05 from 9 rows; chains of
                R ops on distinct weight and x copies (over 2 x L2 per replay).
    single_request  one request, 256-token prompt, 64 greedy steps, no mask,
                through needle_run_batch_ids (host buffers).
    mlp_block   ffn_forward over T = 256 tokens, d 512 -> 2048 -> 512, drelu.
    Each carries the oracle's single-thread time of the same work (cpu_us:
    the reference path restated in C++, AVX2 order)."""
    import oracle

    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    hbm, tcp = pk["hbm_gbs"], pk.get("bf16_tflops", 1590.0)
    out = {}

    def alg_bytes(M, N, K):
        return N * K / 2 + (K // 32) * N * 4 + M * K * 4 + M * N * 4

    # ── config 0: INT4 GEMV ──
    M, N, K = 1, 2048, 512
    x, packed, scales = wl.int4_case(M, N, K, seed=0)
    R = 512
    W = dev(np.broadcast_to(packed.reshape(1, -1), (R, packed.size)))
    S = dev(np.broadcast_to(scales.reshape(1, -1), (R, scales.size)))
    xd = dev(x)
    Y = torch.empty((R, N), device="cuda")
    G = scales.shape[0]

    def chain(overlap):
        def launch(st):
            for r in range(R):
                nb.int4_matmul(xd.data_ptr(), M, K, W[r].data_ptr(), S[r].data_ptr(), N, G, Y[r].data_ptr(),
                               stream=st, overlap=overlap)
        return launch

    ref = oracle.matmul(packed, scales, K, N, x, path=1)
    res = {"shape": [M, N, K], "copies": R, "bytes_per_op": alg_bytes(M, N, K)}
    for name, ov in (("plain", False), ("overlap", True)):
        ms = _graph_ms(torch, chain(ov))
        gbs = R * alg_bytes(M, N, K) / (ms / 1e3) / 1e9
        res[name] = {"us_per_op": 1e3 * ms / R, "GB/s": gbs, "frac_of_measured_hbm": gbs / hbm,
                     "frac_of_8TBs": gbs / 8000.0}
    got = Y[R - 1].cpu().numpy()
    res["max_abs_err_vs_oracle"] = float(np.max(np.abs(got - ref)))
    res["cpu_us"] = _cpu_us(lambda: oracle.matmul(packed, scales, K, N, x, path=1))
    out["int4_gemv"] = res
    del W, S, Y

    # ── config 4: shape sweep ──
    sweep = []
    for M in (1, 8, 64, 512, 4096):
        for (N, K) in ((512, 512), (2048, 512), (512, 2048), (8192, 512)):
            x, packed, scales = wl.int4_case(M, N, K, seed=M + N + K)
            G = scales.shape[0]
            per = packed.nbytes + scales.nbytes + x.nbytes
            R = int(min(1024, max(2, -(-2 * L2_BYTES // per))))
            Wd = dev(np.broadcast_to(packed.reshape(1, -1), (R, packed.size)))
            Sd = dev(np.broadcast_to(scales.reshape(1, -1), (R, scales.size)))
            Xd = dev(np.broadcast_to(x.reshape(1, -1), (R, x.size)))
            Yd = torch.empty((M, N), device="cuda")
            plans = [nb.Int4Plan(Wd[r].data_ptr(), Sd[r].data_ptr(), K, N, G, M) for r in range(R)]

            def launch(st, plans=plans, Xd=Xd, Yd=Yd, M=M):
                for r, pl in enumerate(plans):
                    pl.matmul(Xd[r].data_ptr(), M, Yd.data_ptr(), stream=st, overlap=M <= 8)
            ms = _graph_ms(torch, launch, reps=3)
            plans[0].status()
            t = ms / 1e3 / R
            rows = min(M, 64)
            cpu = _cpu_us(lambda: oracle.matmul(packed, scales, K, N, x[:rows], path=1), budget_s=0.2,
                          min_reps=1) * (M / rows)
            path = "tcgen05" if M > 8 else "cuda-core gemv"
            gbs = alg_bytes(M, N, K) / t / 1e9
            tfl = 2.0 * M * N * K / t / 1e12
            sweep.append({"M": M, "N": N, "K": K, "path": path, "us": 1e6 * t, "GB/s": gbs,
                          "frac_hbm": gbs / hbm, "TFLOP/s": tfl, "frac_bf16": tfl / tcp, "cpu_us": cpu,
                          "copies": R})
            for pl in plans:
                pl.close()
            del Wd, Sd, Xd, Yd
    out["int4_sweep"] = sweep
    torch.cuda.empty_cache()

    # ── config 1: one request ──
    ids, off = wl.random_prompts(1, 256, 256, 8192, seed=11)
    prompt = [ids.tolist()]
    eng.run_batch_ids(prompt, 64)
    times = []
    for _ in range(5):
        t0 = time.perf_counter()
        gpu_ids, _ = eng.run_batch_ids(prompt, 64)
        times.append(time.perf_counter() - t0)
    if _ORACLE.get("key") != id(blob):
        _ORACLE.update(key=id(blob), model=oracle.Model(data=blob))
    t0 = time.perf_counter()
    ref_ids = _ORACLE["model"].generate(ids, 64)[0]
    cpu_s = time.perf_counter() - t0
    ms = 1e3 * statistics.median(times)
    out["single_request"] = {"prompt": 256, "steps": 64, "ms": ms, "tokens/s": 64 / (ms / 1e3),
                             "cpu_ms": 1e3 * cpu_s, "cpu_cores": 1,
                             "first_tokens_match": bool(np.array_equal(np.asarray(gpu_ids[0][:8]),
                                                                       np.asarray(ref_ids[:8])))}

    # ── config 2: MLP block ──
    T, d, ff = 256, 512, 2048
    rng = np.random.default_rng(2)
    x = rng.standard_normal((T, d)).astype(np.float32)
    g, u, dn = wl.random_int4(rng, d, ff), wl.random_int4(rng, d, ff), wl.random_int4(rng, ff, d)
    gd, ud, dd = [dev(a) for a in g], [dev(a) for a in u], [dev(a) for a in dn]
    xd, od = dev(x), torch.empty((T, d), device="cuda")

    def mlp(st):
        for _ in range(8):
            nb.ffn_forward_noalloc(xd.data_ptr(), T, d, ff, [a.data_ptr() for a in gd], [a.data_ptr() for a in ud],
                                   [a.data_ptr() for a in dd], 0, od.data_ptr(), stream=st)
    ms = _graph_ms(torch, mlp) / 8
    ref0 = oracle.ffn_forward(g, u, dn, d, ff, x[0], 0)
    cpu = _cpu_us(lambda: [oracle.ffn_forward(g, u, dn, d, ff, x[t], 0) for t in range(16)], budget_s=0.3,
                  min_reps=1) * (T / 16)
    fl = 3 * 2.0 * T * d * ff
    out["mlp_block"] = {"T": T, "d": d, "d_ff": ff, "activation": "drelu", "us": 1e3 * ms,
                        "TFLOP/s": fl / (ms / 1e3) / 1e12, "cpu_us": cpu,
                        "max_abs_err_row0": float(np.max(np.abs(od[0].cpu().numpy() - ref0)))}
    return out


class Clocks:
    """nvidia-smi sampler for the timed region."""

    def __init__(self, device):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(device), f"--query-gpu={q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f,
                                      stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None

    def stop(self):
        if self.p is None:
            return None
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except Exception:
            self.p.kill()
        self.f.flush()
        rows = []
        for line in open(self.f.name):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 7:
                rows.append(parts)
        os.unlink(self.f.name)
        if not rows:
            return None
        sm = [float(r[0]) for r in rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[3 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--requests", type=int, default=4096, help="requests per GPU")
    ap.add_argument("--max-new", type=int, default=64)
    ap.add_argument("--min-len", type=int, default=64)
    ap.add_argument("--max-len", type=int, default=512)
    ap.add_argument("--mask-frac", type=float, default=0.05)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="CPU baseline sample budget")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-ops", action="store_true", help="skip the INT4 op / single-request / MLP measurements")
    ap.add_argument("--profile-run", action="store_true",
                    help="one untimed run of the workload and exit (for ncu launch lists)")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl != "reference":
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    if args.impl == "reference":
        return run_reference(args)

    import numpy as np
    import torch
    import torch.distributed as dist

    rank, world, local = env_rank()
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("gloo", timeout=timedelta(seconds=900))
    torch.cuda.set_device(local)
    nb, wl = pkg()

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    blob, ids, off, masks = workload(args, wl, rank)
    eng = nb.NeedleEngine.from_bytes(blob, "a\nb\n", device=local)
    batch = eng.prepare_batch(ids, off, args.max_new, masks, flags=0)
    stream = torch.cuda.ExternalStream(batch.stream, device=local)
    tokens_per_step = args.requests * args.max_new
    if args.profile_run:
        batch.run()
        batch.sync()
        print(json.dumps({"profile_run": True, "kernel_launches": batch.kernel_launches(),
                          "requests": args.requests}), flush=True)
        batch.close()
        eng.close()
        return 0

    # Per-kernel-class breakdown (one instrumented run each) to find the
    # dominant kernel, then warm-up runs.
    breakdown = {}
    for cls in CLASS_NAMES:
        batch.time_kernel(cls)
        batch.run()
        batch.sync()
        ms, n, fl, by = batch.kernel_timing()
        breakdown[CLASS_NAMES[cls]] = {"ms": ms, "launches": n, "flops": fl, "bytes": by}
    dom = max(ROOFLINE_CLASSES, key=lambda c: breakdown[CLASS_NAMES[c]]["ms"])
    batch.time_kernel(dom)
    for _ in range(args.warmup):
        batch.run()
    batch.sync()

    # ── timed region: device-resident inputs ──
    barrier()
    torch.cuda.synchronize()
    clocks = Clocks(local)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    launches = 0
    dom_ms = dom_n = dom_fl = dom_by = 0.0
    e0.record(stream)
    for _ in range(args.steps):
        batch.run()
        launches += batch.kernel_launches()
        # the last run's per-kernel events are read after the region
    e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    barrier()
    ms, n, fl, by = batch.kernel_timing()  # events of the last timed run
    dom_ms, dom_n, dom_fl, dom_by = ms, n, fl, by
    elapsed = e0.elapsed_time(e1)
    ms_step = max_over_ranks(elapsed / args.steps)
    value = world * tokens_per_step / (ms_step / 1e3)
    out_ids, lens = batch.results()
    assert int(lens.min()) == args.max_new

    # ── e2e: host buffers through needle_run_batch_ids ──
    e2e = None
    if not args.no_e2e:
        def pinned(a):
            t = torch.empty(a.shape, dtype={np.uint32: torch.int32, np.uint64: torch.int64}[a.dtype.type],
                            pin_memory=True)
            v = t.numpy().view(a.dtype)
            v[...] = a
            return t, v

        _, ids_p = pinned(ids)
        _, off_p = pinned(off)
        _, mask_p = pinned(masks)
        _, out_p = pinned(np.zeros((args.requests, args.max_new), np.uint32))
        _, lens_p = pinned(np.zeros(args.requests, np.uint32))
        L = nb.lib()

        def call():
            rc = L.needle_run_batch_ids(eng._h, nb._p(ids_p), nb._p(off_p), args.requests, args.max_new,
                                        nb._p(mask_p), 0, nb._p(out_p), nb._p(lens_p))
            if rc != 0:
                raise nb.NeedleError(nb.last_error())

        call()
        times = []
        for _ in range(args.steps):
            barrier()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            call()
            times.append(time.perf_counter() - t0)
        e2e_s = max_over_ranks(statistics.mean(times))
        h2d = ids.nbytes + off.nbytes + masks.nbytes
        d2h = args.requests * args.max_new * 4 + args.requests * 4
        e2e = {"value": world * tokens_per_step / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": int(h2d),
               "d2h_bytes_per_step": int(d2h), "ms_per_step": 1e3 * e2e_s,
               "tokens_match_device_run": bool(np.array_equal(out_p, out_ids))}

    # ── roofline of the dominant kernel (its launches in the last timed run) ──
    pk, pk_src = peaks()
    avg_s = dom_ms / 1e3 / max(dom_n, 1)
    if CLASS_NAMES[dom] in ("cross_attention", "head_mask_argmax"):
        achieved = dom_by / max(dom_n, 1) / avg_s / 1e9
        peak = pk["hbm_gbs"]
        roof = {"bound": "hbm", "unit": "GB/s", "traffic": None}
    else:
        achieved = dom_fl / max(dom_n, 1) / avg_s / 1e12
        peak = pk["bf16_tflops_sustained"] if "bf16_tflops_sustained" in pk else pk["bf16_tflops"]
        roof = {"bound": "tensor", "unit": "TFLOP/s", "traffic": None}
    roof.update({"kernel": CLASS_NAMES[dom], "achieved": achieved, "peak": peak, "frac": achieved / peak,
                 "peak_source": pk_src, "launches": dom_n, "avg_launch_us": avg_s * 1e6,
                 "algorithmic_per_launch": (dom_by if roof["bound"] == "hbm" else dom_fl) / max(dom_n, 1)})
    if roof["bound"] == "hbm":
        # a read-dominated kernel is bounded by the read stream, which runs
        # faster than the copy the peak is measured on: report that ceiling too
        rd = ctypes.c_double(0.0)
        if nb.lib().needle_hbm_read_gbs(2 << 30, 10, ctypes.byref(rd)) == 0 and rd.value > 0:
            roof.update({"read_peak": rd.value, "frac_of_read_peak": achieved / rd.value,
                         "read_peak_source": "needle_hbm_read_gbs: grid-stride float4 read stream over 2 GiB on "
                                             "this GPU, after the timed region"})
    if dom in DRAM_PER_ALG_BYTE:
        roof["traffic"] = DRAM_PER_ALG_BYTE[dom] * dom_by / max(dom_n, 1)
        roof["traffic_source"] = "ncu dram__bytes_read.sum + dram__bytes_write.sum per algorithmic byte, 512-request capture, scaled"

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, threads, n, t = cpu_sample(args, blob, ids, off, masks, args.cpu_seconds)
        cpu = {"value": v, "unit": "tokens/s", "cores": threads, "kind": "port",
               "sample": f"first {n} of the {args.requests} requests ({t:.1f} s), one request per host thread; "
                         "the reference Rust path restated in C++ (oracle/)"}

    # ── the decode path against the HBM roofline: its algorithmic bytes (the
    # encoder K/V rows read by cross-attention every step, the self-attention
    # K/V cache, the decode projections and the head) over the summed time of
    # those kernel classes in the breakdown run ──
    L_dec = 8
    self_kv = L_dec * args.requests * (args.max_new * (args.max_new + 1) // 2) * 2 * 256 * 4
    dec_cls = ("cross_attention", "self_attention", "decode_matmul", "head_mask_argmax")
    dec_ms = sum(breakdown[c]["ms"] for c in dec_cls)
    dec_bytes = (breakdown["cross_attention"]["bytes"] + self_kv + breakdown["decode_matmul"]["bytes"]
                 + breakdown["head_mask_argmax"]["bytes"])
    dec_gbs = dec_bytes / (dec_ms / 1e3) / 1e9
    decode_path = {"bytes_per_step": dec_bytes, "ms_per_step": dec_ms, "GB/s": dec_gbs,
                   "frac_of_measured_hbm": dec_gbs / pk["hbm_gbs"], "frac_of_8TBs": dec_gbs / 8000.0,
                   "classes": list(dec_cls)}

    ops = None
    if rank == 0 and world == 1 and not args.no_ops:
        ops = op_suite(args, nb, wl, torch, np, pk, eng, blob)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": config_desc(args),
            "e2e": e2e, "gpu_launches": int(launches), "roofline": roof, "cpu_baseline": cpu, "clocks": clk,
            "kernel_breakdown_ms": {k: round(v["ms"], 3) for k, v in breakdown.items()},
            "decode_path": decode_path, "ops": ops,
        }
        print(json.dumps(line), flush=True)
    batch.close()
    eng.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())

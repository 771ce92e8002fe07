"""Benchmark: Q4_K decode step of a Qwen3-8B-shaped block stack (config 2).

One step = one decode token through 36 layers (fused QKV, attention over 128
KV positions, O, fused gate|up, down) and the 151936-row LM head with the
greedy argmax: 4.26 GB of Q4_K weights streamed per token, batch 1.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

value  = algorithmic bytes of all matvecs of the step x ranks / step time
         (GB/s); tokens/s is reported beside it.
e2e    = the same metric through bh_stack_decode_host: the embedding comes
         from pinned host memory and the token is read back every step.
N > 1  = one process per GPU running the row-split (tensor-parallel) step:
         every rank holds 1/N of every matrix's rows and of the heads, the
         vectors each next launch reads whole are completed by peer stores over
         NVLink from the producing launch's epilogue (bh_stack_create_tp; the
         NCCL communicator that connects the ranks comes from the library's
         non-blocking bh_tp_comm_init). value = the whole model's algorithmic
         bytes per step / the slowest rank's step time (strong scaling: the
         same one-sequence step on N GPUs). Replicas (each GPU its own sequence
         and weights, no exchange) are reported beside it.
--impl reference times the reference's own CPU implementation of the step:
the decode graph the reference engine builds (forward.cpp build_block_decode
+ LM head) on the reference's own ggml CPU backend (oracle/_ref, compiled
from the reference tree), all host threads, weights generated and quantized
on the host (ggml_quantize_chunk); it loads nothing of this repository's
product library.
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

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "shannon-prime-burnhard_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

METRIC = "Q4_K matvec achieved HBM GB/s (% of peak) and decode tokens/s at 1/2/4/8 B200"
SEED = 20261201
KV_POS = 127            # the token attends over 128 positions
X_SEED = 777


def peaks() -> tuple[float, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def start_clock_sampler(path: str):
    cmd = ["nvidia-smi",
           "--query-gpu=index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
           "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
           "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
           "--format=csv,noheader,nounits", "-lms", "200"]
    try:
        return subprocess.Popen(cmd, stdout=open(path, "w"), stderr=subprocess.DEVNULL)
    except Exception:
        return None


def stop_clock_sampler(proc, path: str, device: int) -> dict:
    if proc is None:
        return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
    proc.terminate()
    try:
        proc.wait(timeout=5)
    except Exception:
        proc.kill()
    sm, mx, reasons = [], [], set()
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    for line in open(path):
        f = [x.strip() for x in line.split(",")]
        if len(f) < 9 or not f[0].isdigit() or int(f[0]) != device:
            continue
        try:
            sm.append(float(f[1]))
            mx.append(float(f[2]))
        except ValueError:
            continue
        for n, v in zip(names, f[5:9]):
            if v.lower() == "active":
                reasons.add(n)
    return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
            "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


# ---------------------------------------------------------- extra configs
def time_events(fn, reps: int, warm: int = 3) -> float:
    """Average ms of fn() over reps calls, CUDA events on the current stream."""
    import torch

    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    e1.synchronize()
    return e0.elapsed_time(e1) / reps


def bench_lmhead_tp(bh, ctx, world: int, rank: int, reps: int) -> dict:
    """Config 5: the 151936 x 4096 Q4_K LM head, rows split over the ranks,
    all-gather of the fp32 logits (or of the per-rank candidates only) and the
    identical greedy pick on every rank; batch 1 and 4. Eager launches (host
    launch cost included); device time as the max over ranks."""
    import torch

    import sharding

    n, k = 151936, 4096
    lo, hi = sharding.even_shards(n, world)[rank]
    g = torch.Generator(device="cuda").manual_seed(SEED + 5)
    rows = hi - lo
    w_local = ctx.q4k_quantize(torch.randn((rows, k), generator=g, device="cuda") * 0.02)
    head = sharding.TPLMHead(ctx, n, k, rank, world, w_local)
    head.enable_peer_exchange()
    out = {"workload": "LM head 151936 x 4096 (config 5), rows split over the GPUs", "rows_per_gpu": rows}
    wbytes = n * (k // 256) * 144
    for b in (1, 4):
        x = torch.randn((b, k), generator=g, device="cuda")
        for mode, gl in (("gather_logits", True), ("gather_candidates", False)):
            barrier(world)
            ms = max_over_ranks(time_events(lambda: head.forward(x, gather_logits=gl), reps), world)
            out[f"b{b}_{mode}"] = {"ms": round(ms, 4), "weight_GBps_all_gpus": round(wbytes / (ms / 1e3) / 1e9, 1)}
        # the pick exchanged through peer memory by the reducing kernel (no collective call)
        barrier(world)
        ms = max_over_ranks(time_events(lambda: head.forward_peer(x), reps), world)
        out[f"b{b}_peer_exchange"] = {"ms": round(ms, 4), "weight_GBps_all_gpus": round(wbytes / (ms / 1e3) / 1e9, 1)}
    head.close_peer_exchange()
    del w_local, head
    torch.cuda.empty_cache()
    return out


def bench_batch_sweep(bh, ctx, peak: float) -> dict:
    """Config 1 (4096x4096) and config 3 (the FFN matvecs 12288x4096 and
    4096x12288) at batch 1, 2, 4, 8 from fp32 activations (quantized to Q8_K
    in the prologue), standalone launch plan; beside each, the reference's
    own GPU kernel for the same product (ggml-cuda mul_mat_vec_q<Q4_K> with
    its Q8_1 quantizer, built for sm_100a from the reference tree) when
    oracle/_ref holds it. Each timed launch reads a different copy of the
    weights (the copies together exceed the L2 several times); back-to-back
    launches captured in a CUDA graph, CUDA events. GB/s = weight +
    activation + output bytes / time."""
    import torch

    import oracle as om

    ref = None
    if os.path.exists(om.MMVQ_SO):
        try:
            ref = om.RefMMVQ()
        except Exception:
            ref = None
    out = {"workload": "Q4_K matvecs 4096x4096 (config 1), 12288x4096 and 4096x12288 (config 3), batch 1-8",
           "peak_GBps": peak,
           "gpu_reference": "ggml-cuda mul_mat_vec_q<Q4_K> + quantize_q8_1 (vendored ggml, sm_100a)" if ref else None}

    def graph_us(launch, ncopy):
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            for i in range(3):
                launch(i, s)
            s.synchronize()
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=s):
                for i in range(ncopy):
                    launch(i, s)
            gr.replay()
            s.synchronize()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(s)
            for _ in range(5):
                gr.replay()
            e1.record(s)
            e1.synchronize()
        del gr
        return e0.elapsed_time(e1) * 1e3 / (5 * ncopy)

    for n, k in ((4096, 4096), (12288, 4096), (4096, 12288)):
        wbytes = n * (k // 256) * 144
        ncopy = max(8, int(4 * 126e6 // wbytes) + 1)
        g = torch.Generator(device="cuda").manual_seed(SEED + 3)
        w0 = ctx.q4k_quantize(torch.randn((n, k), generator=g, device="cuda") * 0.02)
        ws = [w0] + [w0.clone() for _ in range(ncopy - 1)]
        for b in (1, 2, 4, 8):
            x = torch.randn((b, k), generator=g, device="cuda")
            y = torch.empty((b, n), device="cuda")
            by = wbytes + b * k * 4 + b * n * 4
            us = graph_us(lambda i, s: ctx.matvec_f32(ws[i], n, k, x, y=y, stream=s), ncopy)
            e = {"us": round(us, 2), "GBps": round(by / us / 1e3, 1), "frac_of_peak": round(by / us / 1e3 / peak, 4)}
            # the same sequence with programmatic dependent launch: each matvec
            # streams its (different) weights while the one before finishes
            ctx.tune(bh.TUNE_PDL, 1)
            try:
                pus = graph_us(lambda i, s: ctx.matvec_f32(ws[i], n, k, x, y=y, stream=s), ncopy)
            finally:
                ctx.tune(bh.TUNE_PDL, 0)
            e.update({"pdl_us": round(pus, 2), "pdl_GBps": round(by / pus / 1e3, 1),
                      "pdl_frac_of_peak": round(by / pus / 1e3 / peak, 4)})
            if ref is not None:
                xq = torch.empty(ref.xq_bytes(k, b), dtype=torch.uint8, device="cuda")
                yr = torch.empty((b, n), device="cuda")
                rus = graph_us(lambda i, s: ref.matvec(ws[i].data_ptr(), n, k, x.data_ptr(), b, xq.data_ptr(),
                                                       yr.data_ptr(), s.cuda_stream), ncopy)
                e.update({"ref_us": round(rus, 2), "ref_GBps": round(by / rus / 1e3, 1),
                          "speedup_vs_ref": round(rus / us, 3)})
            out[f"{n}x{k}_b{b}"] = e
        del ws, w0
        torch.cuda.empty_cache()
    return out


def bench_moe(bh, ctx, world: int, rank: int, steps: int) -> dict:
    """Config 4: the 30B-A3B-shaped expert layers (128 experts, 2048 -> 768 ->
    2048, top-8 of seeded router logits, renormalised). One GPU: the 48-layer
    stack (one cooperative launch per layer, CUDA graph), 1 and 8 tokens.
    Several GPUs: one layer expert-parallel (experts split over the ranks,
    NCCL all-reduce of the expert outputs, slot-order combine), eager."""
    import torch

    import sharding

    res = {"workload": "MoE 30B-A3B-shaped expert layers (config 4)"}
    if world == 1:
        for t in (1, 8):
            cfg = bh.default_moe_config(n_tok=t)
            st = bh.MoeStack(ctx, cfg, SEED + 4)
            h = torch.randn((t, cfg.n_embd), device="cuda")
            out = torch.empty_like(h)
            ms = time_events(lambda: st.step(h, out), max(5, steps // 20))
            info = st.info()
            res[f"tokens{t}"] = {"layers": cfg.n_layer, "ms_per_step": round(ms, 4),
                                 "us_per_layer": round(ms * 1e3 / cfg.n_layer, 2),
                                 "expert_bytes_per_step": info["step_bytes"],
                                 "GBps": round(info["step_bytes"] / (ms / 1e3) / 1e9, 1),
                                 "tokens_per_s": round(t * 1e3 / ms, 1)}
            st.close()
            del st
            torch.cuda.empty_cache()
        return res
    E, D, F, k = 128, 2048, 768, 8
    lo, hi = sharding.even_shards(E, world)[rank]
    g = torch.Generator(device="cuda").manual_seed(SEED + 6)
    own = {}
    for name, rows, cols in (("gate", F, D), ("up", F, D), ("down", D, F)):
        own[name] = ctx.q4k_quantize(torch.randn(((hi - lo) * rows, cols), generator=g, device="cuda") * 0.02)
    ep = sharding.EPMoE(ctx, E, D, F, k, rank, world, own["gate"], own["up"], own["down"])
    ep.enable_peer_exchange()
    gi = torch.Generator(device="cuda").manual_seed(SEED + 7)  # the same tokens and logits on every rank
    for t in (1, 8):
        cur = torch.randn((t, D), generator=gi, device="cuda")
        lg = torch.randn((t, E), generator=gi, device="cuda")
        barrier(world)
        ms = max_over_ranks(time_events(lambda: ep.forward(cur, logits=lg), 20), world)
        res[f"tokens{t}_one_layer_expert_parallel"] = {"us": round(ms * 1e3, 2)}
        barrier(world)
        ms = max_over_ranks(time_events(lambda: ep.forward_peer(cur, logits=lg), 20), world)
        res[f"tokens{t}_one_layer_expert_parallel_peer_exchange"] = {"us": round(ms * 1e3, 2)}
    ep.close_peer_exchange()
    return res


# ---------------------------------------------------------------- CPU path
def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_graph_stack(cfg: dict, nthreads: int):
    """The reference's decode step on the host (oracle/ref_stack.py): the
    engine's ggml graph on the reference's ggml CPU backend, host-generated
    weights (4 distinct layers cycled over the 36, plus the LM head)."""
    import ref_stack

    return ref_stack.make_host_stack(cfg, SEED, nthreads, n_distinct=4, kv_pos=KV_POS)


def cpu_legs(nthreads: int, budget_s: float = 3.0) -> dict:
    """BASELINE.md's three CPU legs on config 1 (Q4_K 4096 x 4096, batch 1):
    (a) one ggml_mul_mat graph node on all host threads, (b) the same on one
    thread, (c) the direct ggml_vec_dot_q4_K_q8_K row loop (one thread).
    Each rep reads another of 64 weight copies (604 MB, beyond any host
    cache), so the figures are DRAM-bound. GB/s = weight + activation +
    output bytes of one matvec / time."""
    import numpy as np

    import oracle as om

    n = k = 4096
    L = om.graph_lib()
    w0 = np.empty(n * om.q4k_row_bytes(k), np.uint8)
    tmp = np.empty((n, k), np.float32)
    L.rg_fill_normal(om._ptr(tmp), tmp.size, 0, SEED + 1, 0.0, 0.02, nthreads)
    L.rg_quantize_q4k(om._ptr(tmp), om._ptr(w0), n, k, nthreads)
    copies = np.empty((64, w0.size), np.uint8)
    copies[:] = w0
    x = np.ascontiguousarray(np.random.default_rng(SEED).standard_normal((1, k)), dtype=np.float32)
    y = np.empty((1, n), np.float32)
    by = n * (k // 256) * 144 + (k // 256) * 292 + n * 4
    out = {"workload": "Q4_K 4096 x 4096 matvec, batch 1 (config 1)", "cpu": cpu_model(),
           "isa": "x86 AVX2/FMA/F16C branch of ggml (arch/x86/quants.c)" if L.rg_has_avx2() else "generic",
           "weight_copies": 64}

    def run(fn):
        fn(0)
        t0 = time.perf_counter()
        reps = 0
        while reps < 8 or time.perf_counter() - t0 < budget_s:
            fn(reps % 64)
            reps += 1
            if reps >= 4096:
                break
        sec = (time.perf_counter() - t0) / reps
        return {"us": round(sec * 1e6, 1), "GBps": round(by / sec / 1e9, 2), "reps": reps}

    out["a_graph_all_threads"] = dict(run(lambda i: om.graph_mul_mat(copies[i], n, k, x, nthreads, out=y)),
                                      threads=nthreads)
    out["b_graph_one_thread"] = dict(run(lambda i: om.graph_mul_mat(copies[i], n, k, x, 1, out=y)), threads=1)
    out["c_direct_row_loop"] = dict(run(lambda i: L.rg_vec_dot_rows(om._ptr(copies[i]), n, k, om._ptr(x),
                                                                    om._ptr(y))), threads=1)
    return out


def time_cpu_steps(g, x, pos: int, nthreads: int, steps: int, budget_s: float | None):
    t0 = time.perf_counter()
    n = 0
    while n < steps and (budget_s is None or n == 0 or time.perf_counter() - t0 < budget_s):
        g.decode(x, pos, nthreads, logits=False)
        n += 1
    return (time.perf_counter() - t0) / n, n


def step_bytes_of(cfg: dict) -> int:
    """Algorithmic bytes of one decode step's matvecs (the same count as
    bh_stack_info's): weights, the activations each reads (fp32 input, twice
    for the RMSNorm prologues), and the outputs."""
    qd, kvd = cfg["n_head"] * cfg["head_dim"], cfg["n_head_kv"] * cfg["head_dim"]
    E, F = cfg["n_embd"], cfg["n_ff"]

    def w(r, k):
        return r * (k // 256) * 144

    layer = (w(qd + 2 * kvd, E) + E * 4 + (qd + 2 * kvd) * 4 + w(E, qd) + qd * 4 + E * 4 +
             w(2 * F, E) + E * 4 + F * 4 + w(E, F) + F * 4 + E * 4)
    return cfg["n_layer"] * layer + w(cfg["n_vocab"], E) + E * 4 + cfg["n_vocab"] * 4


def run_reference_arm(args, cfg: dict, workload: dict) -> None:
    """--impl reference: rank 0 times the reference's CPU step; others exit."""
    import numpy as np

    if int(os.environ.get("RANK", "0")) != 0:
        return
    nthreads = len(os.sched_getaffinity(0))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    g = cpu_graph_stack(cfg, nthreads)
    x = np.random.default_rng(X_SEED).standard_normal(cfg["n_embd"]).astype(np.float32)
    for _ in range(args.warmup):
        g.decode(x, KV_POS, nthreads, logits=False)
    sec, n = time_cpu_steps(g, x, KV_POS, nthreads, args.steps, None)
    g.close()
    v = step_bytes_of(cfg) / sec / 1e9
    legs = cpu_legs(nthreads)
    sample = (f"{n} full decode steps ({cfg['n_layer']} layers + {cfg['n_vocab']}-row LM head) of the reference "
              f"engine's ggml graph on the reference's ggml CPU backend, {nthreads} host threads; weights: "
              f"{min(4, cfg['n_layer'])} distinct seeded layers cycled over the {cfg['n_layer']}, quantized by "
              f"ggml_quantize_chunk on the host")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": "GB/s", "n_gpus": world,
        "steps": n, "warmup": args.warmup, "ms_per_step": round(sec * 1e3, 3),
        "tokens_per_s": round(1.0 / sec, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "q4_K x q8_K (int8 dot, fp32 fold)", "data": "synthetic",
        "config": workload,
        "cpu_baseline": {"value": round(v, 3), "unit": "GB/s", "cores": nthreads, "kind": "reference",
                         "sample": sample, "cpu": cpu_model()},
        "cpu_legs": legs,
        "e2e": {"value": round(v, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ---------------------------------------------------------------- main
def run_matvec_only(args) -> None:
    """One standalone Q4_K matvec shape, launched args.steps times back to back
    on one GPU (seeded weights, fp32 activations quantized in the prologue);
    prints the mean device time per launch."""
    import torch

    import burnhard as bh

    n, k, b = (int(v) for v in args.matvec.lower().split("x"))
    ctx = bh.Context(0)
    g = torch.Generator(device="cuda").manual_seed(SEED + 9)
    w = ctx.q4k_quantize(torch.randn((n, k), generator=g, device="cuda") * 0.02)
    x = torch.randn((b, k), generator=g, device="cuda")
    y = torch.empty((b, n), device="cuda")
    for _ in range(args.warmup):
        ctx.matvec_f32(w, n, k, x, y=y)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        ctx.matvec_f32(w, n, k, x, y=y)
    e1.record()
    e1.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / args.steps
    by = n * (k // 256) * 144 + b * k * 4 + b * n * 4
    print(json.dumps({"matvec": [n, k, b], "us": round(us, 2), "GBps": round(by / us / 1e3, 1),
                      "status": ctx.status()}), flush=True)
    ctx.close()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--layers", type=int, default=0, help="override n_layer (testing only)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the config 4 / config 5 measurements")
    ap.add_argument("--matvec", default="", metavar="NxKxB",
                    help="only run one standalone matvec shape (fp32 input, batch B) --steps times and print its "
                         "time (a small case for a profiler)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    # BASELINE config 2 (the values of bh_stack_default_config)
    cfg_d = dict(n_layer=args.layers or 36, n_embd=4096, n_head=32, n_head_kv=8, head_dim=128, n_ff=12288,
                 n_vocab=151936, n_ctx=128, rms_eps=1e-6, rope_theta=1e6)
    world_env = int(os.environ.get("WORLD_SIZE", "1"))
    workload = {"workload": "qwen3-8b-shaped decode block stack (config 2), batch 1",
                **{k: cfg_d[k] for k in ("n_layer", "n_embd", "n_head", "n_head_kv", "head_dim", "n_ff", "n_vocab")},
                "kv_positions": KV_POS + 1, "weights": "random-init N(0,0.02) quantized to Q4_K",
                "l2": "no flush needed: 4.26 GB of weights streamed per step >> 126 MB L2",
                "parallelism": (f"row-split tensor parallel x{world_env} (peer-memory exchange in the epilogues)"
                                if world_env > 1 else "single GPU")}
    if args.matvec:
        run_matvec_only(args)
        return
    if args.impl == "reference":
        run_reference_arm(args, cfg_d, workload)
        return

    world, rank, local = dist_setup()
    import numpy as np
    import torch

    import burnhard as bh

    torch.cuda.set_device(local)
    nthreads = len(os.sched_getaffinity(0))
    cfg = bh.default_stack_config()
    if args.layers:
        cfg.n_layer = args.layers

    ctx = bh.Context(local)
    x_host = np.asarray(__import__("oracle").Oracle().normal((cfg.n_embd,), X_SEED, 0.0, 1.0))
    x_dev = torch.from_numpy(x_host).cuda()
    tok = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.Stream()

    def timed_steps(stk, steps: int, warmup: int) -> float:
        """Device ms per step (CUDA events on the launching stream, the
        slowest rank), after warm-up; every rank runs the same steps."""
        with torch.cuda.stream(stream):
            for _ in range(warmup):
                stk.decode(x_dev, tok, stream)
            stream.synchronize()
            # a broken exchange (a bounded wait that ran out on any rank) ends
            # the run on every rank before the timed region
            if max_over_ranks(float(ctx.status(clear=False) != 0), world) > 0:
                raise RuntimeError("device status set during warm-up (a bounded wait ran out)")
            time.sleep(0.3)
            barrier(world)
            torch.cuda.synchronize()
            ev0 = torch.cuda.Event(enable_timing=True)
            ev1 = torch.cuda.Event(enable_timing=True)
            ev0.record(stream)
            for _ in range(steps):
                stk.decode(x_dev, tok, stream)
            ev1.record(stream)
            ev1.synchronize()
            torch.cuda.synchronize()
            barrier(world)
        return max_over_ranks(ev0.elapsed_time(ev1) / steps, world)

    comm = None
    if world > 1:
        # the headline: the row-split step; the ranks are connected through
        # the library's own non-blocking NCCL communicator
        import torch.distributed as dist

        obj = [bh.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        comm = bh.tp_comm_init(local, obj[0], world, rank, 120000)
        st = bh.Stack(ctx, cfg, SEED, rank=rank, world=world)
        st.tp_connect_comm(comm, 120000)
    else:
        st = bh.Stack(ctx, cfg, SEED)
    st.fill_kv(KV_POS, SEED + 1)
    st.set_pos(KV_POS)
    info = st.info()
    step_bytes, launches = info["step_bytes"], info["launches"]
    if world > 1:
        t = torch.tensor([float(step_bytes)], device="cuda")
        import torch.distributed as dist

        dist.all_reduce(t)
        job_bytes = int(t.item())  # the whole model's bytes of one step, over all ranks
    else:
        job_bytes = step_bytes

    clock_file = os.path.join(tempfile.gettempdir(), f"bh_clocks_{os.getpid()}.csv")
    sampler = start_clock_sampler(clock_file)
    ms = timed_steps(st, args.steps, args.warmup)
    clocks = stop_clock_sampler(sampler, clock_file, local)
    value = job_bytes / (ms / 1e3) / 1e9
    first_tok = int(tok.item())

    # e2e through the host-buffer entry point (pinned input, token read back)
    pinned = torch.from_numpy(x_host).pin_memory()
    for _ in range(3):
        st.decode_host(pinned)
    barrier(world)
    e2e_steps = max(20, args.steps // 4)
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        st.decode_host(pinned)
    e2e_ms = max_over_ranks((time.perf_counter() - t0) / e2e_steps * 1e3, world)
    e2e_value = job_bytes / (e2e_ms / 1e3) / 1e9
    status = ctx.status()

    replicas = None
    if world > 1:
        torch.cuda.synchronize()
        barrier(world)  # every rank done with the peers' exchange regions
        st.close()
        bh.tp_comm_free(comm, 60000)
        # beside it: N replicas of the one-GPU step (no exchange)
        st = bh.Stack(ctx, cfg, SEED)
        st.fill_kv(KV_POS, SEED + 1)
        st.set_pos(KV_POS)
        rms = timed_steps(st, args.steps, args.warmup)
        replicas = {"value": round(st.info()["step_bytes"] * world / (rms / 1e3) / 1e9, 2), "unit": "GB/s",
                    "ms_per_step": round(rms, 4), "tokens_per_s": round(world * 1e3 / rms, 2), "scaling": "weak",
                    "what": f"{world} independent one-GPU decode steps (own weights, own sequence), no exchange"}
        if int(tok.item()) != first_tok:
            replicas["token_mismatch"] = [first_tok, int(tok.item())]

    # dominant kernel: the fused gate|up matvec (52% of the step's bytes)
    op_ms, op_bytes = st.time_op(bh.OP_GATE_UP, reps=3)
    peak, peak_kind = peaks()
    achieved = op_bytes / (op_ms / 1e3) / 1e9
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "gate_up_traffic.json")
    if os.path.exists(tpath):
        try:
            traffic = json.load(open(tpath)).get("dram_bytes_per_launch")
        except Exception:
            traffic = None
    status = ctx.status()

    # the other configurations of the path, reported beside the headline
    extra = {}
    if not args.no_extra:
        try:
            extra["lmhead_row_split"] = bench_lmhead_tp(bh, ctx, world, rank, reps=max(20, args.steps // 10))
        except Exception as e:  # reported, never silently dropped
            extra["lmhead_row_split"] = {"error": repr(e)}
        try:
            extra["moe"] = bench_moe(bh, ctx, world, rank, args.steps)
        except Exception as e:
            extra["moe"] = {"error": repr(e)}
        try:
            extra["batch_sweep"] = bench_batch_sweep(bh, ctx, peaks()[0])
        except Exception as e:
            extra["batch_sweep"] = {"error": repr(e)}

    cpu_baseline = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        # the reference's CPU step (its ggml graph on its ggml CPU backend),
        # bounded to ~12 s of steps, plus the three config-1 legs
        g = cpu_graph_stack(cfg_d, nthreads)
        g.decode(x_host, KV_POS, nthreads, logits=False)  # warm the caches of the CPU path
        sec, n = time_cpu_steps(g, x_host, KV_POS, nthreads, 50, budget_s=12.0)
        g.close()
        cpu_baseline = {"value": round(step_bytes_of(cfg_d) / sec / 1e9, 3), "unit": "GB/s", "cores": nthreads,
                        "kind": "reference", "tokens_per_s": round(1.0 / sec, 3), "cpu": cpu_model(),
                        "sample": f"{n} full decode steps ({cfg_d['n_layer']} layers + LM head) of the reference "
                                  f"engine's ggml graph on the reference's ggml CPU backend in ~12 s, {nthreads} "
                                  f"threads; host-generated weights, {min(4, cfg_d['n_layer'])} distinct layers cycled",
                        "legs": cpu_legs(nthreads)}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "tokens_per_s": round(1e3 / ms, 2),
            "higher_is_better": True, "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
            "dtype": "q4_K x q8_K (int8 dot, fp32 fold)", "data": "synthetic", "config": workload,
            "step_bytes": job_bytes, "frac_of_hbm_peak": round(value / world / peak, 4),
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "ms_per_step": round(e2e_ms, 4),
                    "h2d_bytes_per_step": cfg.n_embd * 4 * world, "d2h_bytes_per_step": 4 * world},
            "token": first_tok,
            "replicas_beside": replicas,
            "roofline": {"bound": "hbm", "kernel": "q4k_matvec (fused gate|up, 24576 x 4096)",
                         "achieved": round(achieved, 1), "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic,
                         "bytes_per_launch": op_bytes, "ms_per_launch": round(op_ms, 5)},
            "cpu_baseline": cpu_baseline,
            "gpu_launches": launches * args.steps * world,
            "configs_beside": extra,
            "clocks": clocks,
            "device_status": status,
        }
        print(json.dumps(line), flush=True)
    st.close()
    ctx.close()
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()

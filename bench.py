#!/usr/bin/env python3
"""pocketinfer decode on B200: BASELINE config 3 (2.6B-class Q4_K_M, b = 1).

A step is one greedy decode token of the synthetic M26 model (40 layers,
d 2304, 36/36 heads x 64, FFN 5760, vocab 73448, Q4_K_M mix with a Q8_0
ffn_down) after its 323-token seeded prompt.  Timed steps cycle over the
BASELINE's decode positions 323..450 (the sequence is rewound every 128
steps), so every step streams the full 1.83 GB of weights plus the KV of
324..451 positions; weights are far larger than L2, so no flush is needed.

  python bench.py [--gpus N --steps K --warmup W]           our CUDA arm
  python bench.py --impl reference [--steps K --warmup W]   CPU restatement of
                                                            the reference path

Multi-GPU (launched by torchrun): b = 1 decode does not shard, so each rank
runs an independent replica; value = all tokens / max-over-ranks device time.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [os.path.join(ROOT, "pocket-workbench-android_b200"), os.path.join(ROOT, "oracle")]

PROMPT_LEN = 323
CYCLE = 128
METRIC = "decode tok/s (2.6B Q4_K_M, b=1)"


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=1024)
    p.add_argument("--warmup", type=int, default=16)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--order", choices=["exact", "fast"], default="exact",
                   help="float order of the decode step (pk_set_order): the reference's exact order, or the fast "
                        "order (Q8 and integer dots exact, float sums regrouped; within 1e-3 per matvec)")
    p.add_argument("--model-dir", default=os.environ.get("PK_MODEL_DIR", tempfile.gettempdir()))
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--cpu-seconds", type=float, default=10.0, help="budget of the bounded CPU baseline sample")
    p.add_argument("--layers", type=int, default=None,
                   help="M26-shaped model with this many layers (the small case for detailed ncu captures)")
    p.add_argument("--vocab", type=int, default=None, help="vocabulary of that model (default M26's)")
    p.add_argument("--tp70", action="store_true",
                   help="tensor-parallel decode of the 70B-shaped stack (BASELINE config 5), one rank per GPU "
                        "(world = the torchrun world size); prints its own JSON line")
    p.add_argument("--tp-layers", type=int, default=None, help="layers of that stack (default 80)")
    p.add_argument("--tp-collective", choices=("peer", "nccl"), default="peer",
                   help="the o / down exchange of --tp70: own peer-memory push, or an NCCL all-reduce")
    p.add_argument("--streams", type=int, default=0,
                   help="independent M26 streams per GPU decoded together (the data-parallel streams case)")
    p.add_argument("--stream-ctx", type=int, default=512, help="KV positions of each stream")
    p.add_argument("--stream-prompt", type=int, default=None,
                   help="prompt tokens prefilled into each stream's cache (default 323)")
    p.add_argument("--kv", choices=("f32", "f16"), default="f32",
                   help="K/V cache entry type of the streams case (pk_set_kv_type)")
    p.add_argument("--stream-pos", type=int, default=None,
                   help="decode the streams at this position (past the prompt: zero-filled cache entries; "
                        "the long-context timing case)")
    p.add_argument("--prefill-only", action="store_true",
                   help="only the prefill leg (warm-up prompt, then the measured 323-token prompt); prints its summary")
    p.add_argument("--config1-only", action="store_true",
                   help="only BASELINE config 1 (one Q4_K 6144x2048 matvec, rotating weight copies); prints its summary")
    p.add_argument("--decode-only", action="store_true",
                   help="only the timed decode (with its traced profile and e2e): no prefill, streams, config-1 "
                        "or CPU legs")
    p.add_argument("--profile-window", action="store_true",
                   help="bracket the timed steps with cudaProfilerStart/Stop (for ncu --profile-from-start off)")
    return p.parse_args()


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            m = json.load(f)
        return float(m["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def dist_info():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 100 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        time.sleep(0.25)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.15)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.t.join(timeout=2)
        return summarize_clocks(self.lines)


def summarize_clocks(lines):
    sm, smax, reasons = [], None, set()
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    for ln in lines:
        f = [x.strip() for x in ln.split(",")]
        if len(f) < 9:
            continue
        try:
            sm.append(float(f[1]))
            smax = float(f[2])
        except ValueError:
            continue
        for n, v in zip(names, f[5:9]):
            if v.lower().startswith("active"):
                reasons.add(n)
    return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
            "samples": len(sm)}


INT8_DENSE_TOPS_NOMINAL = 4500.0  # B200 dense int8 tensor peak (no measured int8 figure on this pool)


def prefill_summary(pre, spec, stream_bytes, hbm):
    """The prefill leg: tok/s through Engine::generate, the int8 ops of the
    layer matvecs per token against the nominal dense int8 peak, and the
    weight stream (every matrix read once per 32-token chunk) against HBM."""
    tokens, s = pre["prefill_tokens"], pre["prefill_ms"] / 1000.0
    ne, ff = spec.n_embd, spec.n_ff
    qdim, kdim = spec.n_head * spec.head_dim, spec.n_head_kv * spec.head_dim
    ops_per_token = 2.0 * spec.n_layer * (ne * qdim + 2 * ne * kdim + qdim * ne + 2 * ne * ff + ff * ne)
    chunks = -(-tokens // 32)
    tops = ops_per_token * tokens / s / 1e12
    gbs = stream_bytes * chunks / s / 1e9
    return {"tokens": tokens, "ms": pre["prefill_ms"], "tok_s": tokens / s, "chunks": chunks,
            "int8_ops_per_token": ops_per_token, "int8_tops": tops, "int8_peak_tops": INT8_DENSE_TOPS_NOMINAL,
            "int8_frac": tops / INT8_DENSE_TOPS_NOMINAL, "int8_peak_kind": "nominal",
            "weight_stream_gbs": gbs, "hbm_frac": gbs / hbm,
            "note": "32-token chunks on six stream lanes in turn; exact reference-order f32 accumulation "
                    "of per-sub-block int8 dots (mma.sync tiles) bounds it, not the tensor pipe or HBM"}


def prefill_tcgen05_leg(pk, path, spec, device, stream_bytes, hbm):
    """The 323-token prefill again with the b > 8 matvecs on the tcgen05 kernel
    (pk_set_matmul_path): same bits, measured beside the default mma.sync tiles."""
    pk.set_matmul_path("tcgen05")
    try:
        eng = pk.Engine(path, n_ctx=512, max_batch=32, device=device)
        eng.generate(synth_prompt(spec, 8, 96), 0, stop_at_eog=False)
        pre = eng.generate(synth_prompt(spec, PROMPT_LEN, PROMPT_LEN), 0, stop_at_eog=False)
        eng.close()
    finally:
        pk.set_matmul_path("mma.sync")
    out = prefill_summary(pre, spec, stream_bytes, hbm)
    out["note"] = ("b > 8 matvecs on tcgen05.mma kind::i8 (one MMA per 32-element block into TMEM, weights staged "
                   "by tensor copies); the same bits as the default mma.sync tiles")
    return out


def prefill_config4(pk, path, spec, device):
    """BASELINE config 4 on the device: a 4096-token prompt prefilled in 32-token
    chunks, and the 323 -> 379 extension, whose second call reuses the 320
    tokens of full chunks it shares with the first (model.rs:1251-1295)."""
    eng = pk.Engine(path, n_ctx=4096 + 64, max_batch=32, device=device)
    warm = synth_prompt(spec, 7, 96)
    eng.generate(warm, 0, stop_at_eog=False)
    long_prompt = synth_prompt(spec, 4096, 4096)
    r = eng.generate(long_prompt, 0, stop_at_eog=False)
    out = {"prefill_4096": {"tokens": r["prefill_tokens"], "ms": r["prefill_ms"],
                            "tok_s": r["prefill_tokens"] / (r["prefill_ms"] / 1000.0)}}
    ext = synth_prompt(spec, 379, 379)
    first = eng.generate(ext[:323], 0, stop_at_eog=False)
    second = eng.generate(ext, 0, stop_at_eog=False)
    out["extension_323_379"] = {"fresh_323_ms": first["prefill_ms"], "cached_tokens": second["prefill_cached_tokens"],
                                "prefill_tokens": second["prefill_tokens"], "ms": second["prefill_ms"]}
    del eng
    return out


def synth_prompt(spec, seed, n):
    from pocketinfer import synth

    return synth.prompt_ids(seed, n, spec.n_vocab)


def cycle_steps(eng, n, state, timed):
    """n decode steps on the device, rewinding to PROMPT_LEN every CYCLE tokens."""
    total_ms, done = 0.0, 0
    while done < n:
        room = PROMPT_LEN + CYCLE - state["pos"]
        if room <= 0:
            eng.set_position(PROMPT_LEN)
            state["pos"] = PROMPT_LEN
            room = CYCLE
        m = min(room, n - done)
        _, ms = eng.decode_steps_device(m, return_ms=True)
        total_ms += ms
        state["pos"] += m
        done += m
    return total_ms


WORKLOAD = "M26 greedy decode b=1 (BASELINE config 3): 323-token prompt, positions 323..450 cycled"


def workload_config(args, world):
    """The line's `config`: the same workload string and model on both arms."""
    from pocketinfer import synth

    full = args.layers is None and args.vocab is None
    return {"workload": WORKLOAD if full else
            f"reduced M26-shaped model {synth.m26_spec(args.layers, args.vocab).name} (profiling case, "
            "not the BASELINE workload)", "model": "synthetic-2.6B-q4km (random blocks)",
            "global_batch": world, "seq_len": PROMPT_LEN + CYCLE,
            "parallelism": f"replicas x{world}" if world > 1 else "single",
            "l2": "no flush: each step streams 1.83 GB of weights (> 126 MB L2)"}


def oracle_decode(path, prompt, warmup, steps, budget_s):
    """The CPU restatement (oracle engine, all host threads) on the bench's own
    workload: the 323-token prompt through Engine::generate's prefill, then
    greedy decode steps at positions 323..450 (cycled), timed until `steps`
    steps or `budget_s` seconds.  Returns (tok/s, steps timed, threads)."""
    import numpy as np

    import pko

    threads = os.cpu_count() or 1
    o = pko.Engine(path, 512, threads)
    o.generate(prompt, 1)  # prefill (32-token chunks), no decode step
    pos = PROMPT_LEN

    def step():
        nonlocal pos
        if pos >= PROMPT_LEN + CYCLE:
            pos = PROMPT_LEN
        tok = int(np.argmax(o.logits()))  # sampler.rs:26-36: first maximum
        o.forward([tok], [pos], True)
        pos += 1

    for _ in range(warmup):
        step()
    t0 = time.perf_counter()
    timed = 0
    while timed < steps:
        step()
        timed += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    o.close()
    return timed / dt, timed, threads


def config1_matvec(pk, synth, device, copies=40, launches=400):
    """one Q4_K 6144 x 2048 matvec (seed 0) against the Q8 of
    x ~ N(0,1), timed over `launches` launches that rotate over `copies`
    distinct weight copies (40 x 7.08 MB = 283 MB > 2 x the 126 MB L2), CUDA
    events on the launching stream.  The launches are captured in one CUDA
    graph and replayed, so the time is the device's: one pk_matmul_packed call
    issued from Python costs more host time than the kernel takes, and the
    host-issued rate is reported beside it.  Bytes per launch: the weights,
    the Q8 activation (q, d, sum) and the f32 output."""
    import torch

    w, x = synth.config1_inputs(0)
    k, rows = 2048, 6144
    wd = torch.from_numpy(w).to(device)
    ws = [wd.clone() for _ in range(copies)]  # Q4_K: the device layout is the GGUF layout
    act = pk.q8_quantize(torch.from_numpy(x).to(device), k, 1)
    out = torch.empty(rows, dtype=torch.float32, device=device)
    st = torch.cuda.Stream(device)
    with torch.cuda.stream(st):
        for i in range(2 * copies):  # warm-up
            pk.matmul_packed(synth.Q4_K, ws[i % copies], k, rows, act, out=out, stream=st.cuda_stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=st):
        for i in range(launches):
            pk.matmul_packed(synth.Q4_K, ws[i % copies], k, rows, act, out=out, stream=st.cuda_stream)
    graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(st):
        e0.record(st)
        graph.replay()
        e1.record(st)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / launches
    h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    h0.record()
    for i in range(launches):
        pk.matmul_packed(synth.Q4_K, ws[i % copies], k, rows, act, out=out)
    h1.record()
    torch.cuda.synchronize()
    us_host = h0.elapsed_time(h1) * 1000.0 / launches
    del graph
    nbytes = w.nbytes + k + 2 * 4 * (k // 32) + 4 * rows
    hbm, kind = peaks()
    return {"shape": "Q4_K 6144x2048, b=1", "us_per_launch": us, "bytes_per_launch": nbytes,
            "achieved_gbs": nbytes / (us * 1e-6) / 1e9, "hbm_frac": nbytes / (us * 1e-6) / 1e9 / hbm,
            "peak_kind": kind, "weight_copies": copies, "launches": launches,
            "us_per_launch_host_issued": us_host,
            "note": "k_mv_b1 (pk_matmul_packed), launches rotating over distinct weight copies, replayed from one "
                    "CUDA graph (us_per_launch_host_issued: the same launches issued one by one from Python)"}


def nccl_allreduce_us(dist, n, iters=200, warmup=20):
    """Device time of one NCCL all-reduce (sum, f32) of the tensor-parallel exchange's
    n floats over the job's ranks (NVLink), CUDA events, max over ranks: the library
    collective the peer-memory exchange is measured against."""
    import torch

    from pocketinfer import replicas

    x = torch.ones(n, dtype=torch.float32, device="cuda")
    for _ in range(warmup):
        dist.all_reduce(x)
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        dist.all_reduce(x)
    e1.record()
    torch.cuda.synchronize()
    return replicas.max_over_ranks(e0.elapsed_time(e1) * 1000.0 / iters, dist, "cuda")


PEER_EXCHANGE = "partial row sums pushed to every rank's peer buffer over NVLink, added in rank order"
NCCL_EXCHANGE = "partial row sums through an NCCL all-reduce on the engine's stream, then added to the residual"


def tp70_leg(world, rank, local, dist, steps=16, warmup=3):
    """BASELINE config 5 (TP half) inside the scaling run: the 70B-shaped stack split
    over this job's world, synthetic weights generated on each device, greedy b = 1
    decode; every rank runs it, the time is the max over ranks.  With more than one
    rank it runs once per exchange (own peer-memory push, NCCL all-reduce) and
    reports the faster as ``value``."""
    peer = tp70_run(world, rank, local, dist, steps, warmup, "peer")
    if world == 1:
        return peer
    try:
        nccl = tp70_run(world, rank, local, dist, steps, warmup, "nccl")
    except Exception as exc:  # noqa: BLE001 -- every rank fails the same way (see TpEngine.connect)
        out = dict(peer)
        out["nccl_error"] = str(exc)[:200]
        return out
    best = nccl if nccl["value"] > peer["value"] else peer
    out = dict(best)
    out["by_collective"] = {"peer": {k: peer[k] for k in ("value", "ms_per_step", "per_rank_hbm_frac")},
                            "nccl": {k: nccl[k] for k in ("value", "ms_per_step", "per_rank_hbm_frac")}}
    return out


def tp70_run(world, rank, local, dist, steps, warmup, collective):
    from pocketinfer import replicas, tp

    model = dict(tp.M70)
    eng = tp.TpEngine(rank, world, device=local, n_ctx=8 + warmup + steps + 16)
    try:
        t0 = time.time()
        err = None
        try:
            eng.load_synthetic(model, seed=70)
        except Exception as exc:  # noqa: BLE001
            err = exc
        load_s = time.time() - t0
        # every rank learns whether all loaded before any of them enters the handle exchange
        if replicas.max_over_ranks(1.0 if err else 0.0, dist, "cuda") > 0.0:
            raise RuntimeError(f"tp70: a rank failed to load ({err})")
        if world > 1:
            eng.connect(collective=collective)
        else:
            eng.connect(exchange=lambda b: [b])
        info = eng.info
        eng.prefill([(7 * i + 3) % model["n_vocab"] for i in range(8)])
        eng.decode(warmup)
        if dist:
            dist.barrier()
        _, ms = eng.decode(steps, return_ms=True)
    finally:
        eng.close()
    max_ms = replicas.max_over_ranks(ms, dist, "cuda")
    ms_step = max_ms / steps
    hbm, kind = peaks()
    gbs = info["stream_bytes"] / (ms_step / 1000.0) / 1e9
    nccl = nccl_allreduce_us(dist, model["n_embd"]) if dist and world > 1 else None
    return {"workload": "BASELINE config 5 TP: 80 L, d 8192, 64/8 heads x 128, FFN 28672, vocab 128256, b=1",
            "nccl_allreduce_us": nccl,
            "nccl_ms_per_token": nccl * info["collectives_per_token"] / 1000.0 if nccl else None,
            "parallelism": f"tp{world}", "value": 1000.0 / ms_step, "unit": "tok/s", "ms_per_step": ms_step,
            "steps": steps, "per_rank_hbm_frac": gbs / hbm, "per_rank_stream_bytes": info["stream_bytes"],
            "peak_kind": kind, "collectives_per_token": info["collectives_per_token"], "load_s": load_s,
            "collective": collective, "exchange": NCCL_EXCHANGE if collective == "nccl" else PEER_EXCHANGE}


def dp_streams_leg(pk, synth, path, spec, world, rank, local, dist, per_gpu=8, ctx=4096, steps=64, warmup=3):
    """BASELINE config 5 (DP half) inside the scaling run: per_gpu x world independent
    greedy M26 streams dealt round-robin to the ranks, each prefilled with its own
    ctx-token prompt (real prompt-filled caches), then batched steps at positions
    ctx.. ; weak scaling, max over ranks."""
    from pocketinfer import replicas

    mine = replicas.assign_streams(per_gpu * world, rank, world)
    n_ctx = ctx + warmup + steps + 4 - (ctx + warmup + steps) % 4
    eng = pk.Engine(path, n_ctx=n_ctx, max_batch=32, device=local)
    try:
        weights = eng.info["stream_bytes"]
        eng.streams_begin(len(mine))
        t0 = time.time()
        for s, sid in enumerate(mine):
            eng.stream_prefill(s, synth.prompt_ids(5000 + sid, ctx, spec.n_vocab))
        prefill_s = time.time() - t0
        eng.streams_decode(warmup)
        if dist:
            dist.barrier()
        _, ms = eng.streams_decode(steps, return_ms=True)
    finally:
        eng.close()
    value, max_ms = replicas.replica_throughput(steps * len(mine), ms, world, dist, "cuda")
    ms_step = max_ms / steps
    hbm, kind = peaks()
    step_bytes = weights + spec.kv_bytes_per_position() * len(mine) * (ctx + warmup + steps / 2)
    gbs = step_bytes / (ms_step / 1000.0) / 1e9
    return {"workload": f"M26, {per_gpu * world} greedy streams ({per_gpu} per GPU), {ctx}-token prompt each, "
                        f"{steps} batched steps", "parallelism": f"dp{world} (streams)", "value": value,
            "unit": "tok/s", "ms_per_step": ms_step, "per_gpu_hbm_frac": gbs / hbm, "per_gpu_bytes_per_step": step_bytes,
            "peak_kind": kind, "prefill_s_per_gpu": prefill_s, "scaling": "weak"}


def cpu_baseline_sample(path, prompt, budget_s):
    """The CPU restatement on this host: decode tok/s on a bounded sample of the
    bench's workload (positions 323.. after the 323-token prompt)."""
    value, timed, threads = oracle_decode(path, prompt, 1, 10 ** 6, budget_s)
    return {"value": value, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"M26 greedy decode, {timed} steps at positions {PROMPT_LEN}..{PROMPT_LEN + timed - 1} after the "
                      f"{PROMPT_LEN}-token prompt ({budget_s:.0f} s budget), C++ restatement of pocketinfer's CPU "
                      f"int8 lanes path, {threads} threads"}


def run_reference(args):
    world, rank, _ = dist_info()
    if rank != 0:
        return
    from pocketinfer import synth

    path = synth.m26_path(args.model_dir, spec=synth.m26_spec(args.layers, args.vocab))
    prompt = synth.prompt_ids(PROMPT_LEN, PROMPT_LEN, synth.m26_spec(args.layers, args.vocab).n_vocab)
    budget = 150.0
    value, timed, threads = oracle_decode(path, prompt, args.warmup, args.steps, budget)
    line = {"metric": METRIC, "value": value, "unit": "tok/s", "impl": "reference", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 / value, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8xint8->int32, f32", "data": "synthetic",
            "config": workload_config(args, 1),
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port",
                             "sample": f"{timed} of {args.steps} decode steps timed (budget {budget:.0f} s), "
                                       "C++ restatement of pocketinfer's CPU path (the Rust crate cannot be "
                                       "built here)"},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_ours(args):
    import torch

    world, rank, local = dist_info()
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    import pocketinfer as pk
    from pocketinfer import replicas, synth

    if rank == 0:
        path = synth.m26_path(args.model_dir, spec=synth.m26_spec(args.layers, args.vocab))
    if dist:
        dist.barrier()
    path = synth.m26_path(args.model_dir, spec=synth.m26_spec(args.layers, args.vocab))
    prompt = synth.prompt_ids(PROMPT_LEN, PROMPT_LEN, synth.m26_spec(args.layers, args.vocab).n_vocab)
    eng = pk.Engine(path, n_ctx=512, max_batch=32, device=local, order=args.order)
    info = eng.info
    # prefill through Engine::generate (32-token chunks); no decode step.  A
    # warm-up prompt of other tokens first (its first token differs, so the
    # measured prompt reuses none of its K/V).
    warm = [(t + 1) % synth.m26_spec(args.layers, args.vocab).n_vocab for t in prompt[:96]]
    eng.generate(warm, 0, stop_at_eog=False)
    pre = eng.generate(prompt, 1, stop_at_eog=False)
    spec = synth.m26_spec(args.layers, args.vocab)
    if args.prefill_only:
        summary = prefill_summary(pre, spec, info["stream_bytes"], peaks()[0])
        summary.update(prefill_config4(pk, path, spec, local))
        if rank == 0:
            print(json.dumps({"prefill": summary}), flush=True)
        if dist:
            dist.destroy_process_group()
        return
    state = {"pos": PROMPT_LEN}
    cycle_steps(eng, args.warmup, state, False)

    gpu_index = local
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        try:
            gpu_index = int(vis.split(",")[local])
        except ValueError:
            pass
    clocks = ClockSampler(gpu_index)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    if args.profile_window:
        torch.cuda.profiler.start()
    total_ms = cycle_steps(eng, args.steps, state, True)
    torch.cuda.synchronize()
    if args.profile_window:
        torch.cuda.profiler.stop()
    clk = clocks.stop()
    if dist:
        dist.barrier()
    value, max_ms = replicas.replica_throughput(args.steps, total_ms, world, dist, "cuda")
    ms_per_step = max_ms / args.steps

    # per-kernel device times of one eager decode step (for the roofline)
    eng.set_position(PROMPT_LEN)
    cycle_steps(eng, CYCLE // 2, {"pos": PROMPT_LEN}, False)
    prof = eng.decode_profile()  # one step at position PROMPT_LEN + CYCLE / 2

    # end to end through Engine::generate: host prompt in, one D2H token read
    # and one H2D token/position write per decode step, host sync per step
    n_e2e = min(args.steps, CYCLE)
    eng.forward(prompt[:1], [0], False)  # public forward: drops the prefix cache
    r = eng.generate(prompt, n_e2e + 1, stop_at_eog=False)
    e2e_value, _ = replicas.replica_throughput(n_e2e, r["gen_ms"], world, dist, "cuda")

    # the partitioned rows of BASELINE config 5, on every rank (same collective steps everywhere)
    tp_row = dp_row = None
    if not args.decode_only and args.layers is None and args.vocab is None:
        eng.close()
        try:
            tp_row = tp70_leg(world, rank, local, dist)
        except Exception as exc:  # noqa: BLE001
            tp_row = {"error": str(exc)[:200]}
        try:
            dp_row = dp_streams_leg(pk, synth, path, spec, world, rank, local, dist)
        except Exception as exc:  # noqa: BLE001
            dp_row = {"error": str(exc)[:200]}

    cpu = None
    c4 = None
    pre_tc = None
    streams = None
    c1 = None
    if rank == 0 and world == 1 and not args.decode_only:
        eng.close()
        try:  # BASELINE config 1, outside the timed region
            c1 = config1_matvec(pk, synth, torch.device("cuda", local))
        except Exception as exc:  # noqa: BLE001
            c1 = {"error": str(exc)[:200]}
        c4 = prefill_config4(pk, path, spec, local)  # BASELINE config 4, outside the timed region
        try:  # the tcgen05 matvec path on the same prefill, outside the timed region
            pre_tc = prefill_tcgen05_leg(pk, path, spec, local, info["stream_bytes"], peaks()[0])
        except Exception as exc:  # noqa: BLE001
            pre_tc = {"error": str(exc)[:200]}
        try:  # the data-parallel streams row, outside the timed region; never fails the line
            streams = streams_summary(pk, synth, path, spec, local)
        except Exception as exc:  # noqa: BLE001
            streams = {"error": str(exc)[:200]}
        if not args.no_cpu_baseline:
            cpu = cpu_baseline_sample(path, prompt, args.cpu_seconds)

    if rank == 0:
        hbm, peak_kind = peaks()
        step_bytes = info["stream_bytes"] + synth.m26_spec(args.layers, args.vocab).kv_bytes_per_position() * (PROMPT_LEN + 1 + CYCLE / 2)
        step_gbs = step_bytes / (ms_per_step / 1000.0) / 1e9
        # the dominant kernel is the persistent decode kernel, one launch per
        # timed step: its average duration is the timed region's per-step time
        # (the per-CTA traced breakdown below explains it, at trace cost)
        achieved = step_gbs
        traffic = None
        if args.layers is None and args.vocab is None:
            try:
                with open(os.path.join(ROOT, "profiles", "k_decode_m26_traffic.json")) as f:
                    traffic = json.load(f)
            except (OSError, ValueError):
                traffic = None
        # persistent kernel: one launch per step, plus argmax + advance once per decode_steps_device call
        calls = -(-args.steps // CYCLE) + 1
        launches = info["decode_kernels"] * args.steps + (2 * calls if info["decode_kernels"] == 1 else 0)
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8xint8->int32, f32", "data": "synthetic",
            "config": dict(workload_config(args, world), order=args.order),
            "prefill_tok_s": pre["prefill_tokens"] / (pre["prefill_ms"] / 1000.0),
            "prefill": dict(prefill_summary(pre, spec, info["stream_bytes"], hbm), **(c4 or {})),
            "prefill_tcgen05": pre_tc,
            "decode_step_hbm": {"bytes_per_step": step_bytes, "achieved_gbs": step_gbs,
                                "frac": step_gbs / hbm, "peak": hbm, "peak_kind": peak_kind},
            "roofline": {"bound": "hbm", "kernel": "k_decode", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                         "frac": achieved / hbm, "peak_kind": f"of {peak_kind}",
                         "algorithmic_bytes_per_launch": step_bytes,
                         "traffic": traffic["traffic_bytes"] if traffic else None,
                         "traffic_source": ("ncu dram__bytes_read.sum + dram__bytes_write.sum of one k_decode launch "
                                            f"at position {traffic['position']} (profiles/k_decode_m26_traffic.md), "
                                            f"{traffic['traffic_over_algorithmic']:.3f} x its algorithmic bytes")
                                           if traffic else None,
                         "per_kernel_traced": prof},
            "e2e": {"value": e2e_value, "unit": "tok/s", "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 4,
                    "path": "pk_generate (C ABI), host prompt, per-token host sync"},
            "gpu_launches": launches,
            "clocks": clk,
            "cpu_baseline": cpu,
            "streams": streams,
            "config1": c1,
            "tp70": tp_row,
            "dp_streams": dp_row,
        }
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def run_tp70(args):
    """BASELINE config 5, tensor-parallel half: the 70B-shaped stack split over
    the torchrun world (1, 2, 4 or 8 GPUs), synthetic weights generated on each
    device, greedy b = 1 decode.  The time is the max over ranks of the CUDA-event
    time of the decode steps; HBM fraction per rank from its shard's bytes."""
    import datetime

    import torch

    world, rank, local = dist_info()
    torch.cuda.set_device(local)
    import torch.distributed as dist

    if world == 1:  # a plain single-process run still gets a (one-rank) group for the handle exchange
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29517")
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=600))
    from pocketinfer import tp

    model = dict(tp.M70)
    if args.tp_layers:
        model["n_layer"] = args.tp_layers
    n_ctx = 8 + max(args.warmup, 3) + args.steps + 16
    eng = tp.TpEngine(rank, world, device=local, n_ctx=n_ctx)
    t0 = time.time()
    eng.load_synthetic(model, seed=70)
    load_s = time.time() - t0
    if world > 1:
        eng.connect(collective=args.tp_collective)
    else:
        eng.connect()
    info = eng.info
    prompt = [(7 * i + 3) % model["n_vocab"] for i in range(8)]
    eng.prefill(prompt)
    eng.decode(max(args.warmup, 3))
    gpu_index = local
    clocks = ClockSampler(gpu_index)
    dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    _, ms = eng.decode(args.steps, return_ms=True)  # args.steps steps, each one token through the model
    clk = clocks.stop()
    t = torch.tensor([ms], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_ms = float(t.item())
    ms_step = max_ms / args.steps
    hbm, peak_kind = peaks()
    gbs = info["stream_bytes"] / (ms_step / 1000.0) / 1e9
    if rank == 0:
        line = {
            "metric": "decode tok/s (70B-shaped Q4_K stack, b=1, tensor-parallel)", "value": 1000.0 / ms_step,
            "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": max(args.warmup, 3),
            "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "int8xint8->int32, f32", "data": "synthetic (weights generated on each device)",
            "config": {"workload": "BASELINE config 5 TP: 80 L, d 8192, 64/8 heads x 128, FFN 28672, vocab 128256"
                       if not args.tp_layers else f"70B-shaped stack cut to {model['n_layer']} layers",
                       "parallelism": f"tp{world}", "prompt": len(prompt),
                       "collectives_per_token": info["collectives_per_token"],
                       "collective": args.tp_collective if world > 1 else "none",
                       "exchange": NCCL_EXCHANGE if args.tp_collective == "nccl" and world > 1 else PEER_EXCHANGE},
            "per_rank": {"stream_bytes": info["stream_bytes"], "achieved_gbs": gbs, "hbm_frac": gbs / hbm,
                         "peak": hbm, "peak_kind": peak_kind, "weight_bytes": info["weight_bytes"],
                         "load_s": load_s},
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    eng.close()
    dist.destroy_process_group()


def streams_summary(pk, synth, path, spec, device, n_streams=8, steps=128, warmup=4):
    """Data-parallel streams on one GPU (outside the timed b = 1 region): n_streams
    independent 323-token prompts, then `steps` batched steps at positions 323..451;
    CUDA-event time of the steps."""
    eng = pk.Engine(path, n_ctx=512, max_batch=32, device=device)  # a multiple of 4: the tiled attention
    try:
        weights = eng.info["stream_bytes"]
        eng.streams_begin(n_streams)
        for s in range(n_streams):
            eng.stream_prefill(s, synth.prompt_ids(1000 + s, PROMPT_LEN, spec.n_vocab))
        eng.streams_decode(warmup)
        eng.streams_set_position(PROMPT_LEN)
        _, ms = eng.streams_decode(steps, return_ms=True)
    finally:
        eng.close()
    ms_step = ms / steps
    step_bytes = weights + spec.kv_bytes_per_position() * n_streams * (PROMPT_LEN + 1 + steps / 2)
    hbm, peak_kind = peaks()
    gbs = step_bytes / (ms_step / 1000.0) / 1e9
    return {"streams": n_streams, "tok_s": n_streams / (ms_step / 1000.0), "ms_per_step": ms_step,
            "bytes_per_step": step_bytes, "achieved_gbs": gbs, "hbm_frac": gbs / hbm, "peak_kind": peak_kind,
            "steps": steps,
            "note": "bench.py --streams 8 for the full line (roofline, clocks, 16K case with --stream-ctx)"}


def run_streams(args):
    """Data-parallel streams: every rank decodes ``--streams`` independent M26
    sequences (its share of streams * world, dealt round-robin), one batched
    step per token of every stream, each stream at its own position over its
    own KV cache.  Weak scaling; the time is the max over ranks of the CUDA-event
    time of the steps."""
    import torch

    world, rank, local = dist_info()
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    import pocketinfer as pk
    from pocketinfer import replicas, synth

    spec = synth.m26_spec(args.layers, args.vocab)
    if rank == 0:
        synth.m26_path(args.model_dir, spec=spec)
    if dist:
        dist.barrier()
    path = synth.m26_path(args.model_dir, spec=spec)
    mine = replicas.assign_streams(args.streams * world, rank, world)
    n_ctx = args.stream_ctx
    plen = args.stream_prompt or PROMPT_LEN
    p0 = args.stream_pos or plen
    if p0 < plen or p0 + CYCLE > n_ctx:
        raise SystemExit(f"need --stream-prompt <= --stream-pos and --stream-pos + {CYCLE} <= --stream-ctx")
    eng = pk.Engine(path, n_ctx=n_ctx, max_batch=max(32, len(mine)), device=local, kv=args.kv)
    info = eng.info
    eng.streams_begin(len(mine))
    t0 = time.time()
    for s, sid in enumerate(mine):  # every stream its own prompt, prefilled into its own cache
        eng.stream_prefill(s, synth.prompt_ids(1000 + sid, plen, spec.n_vocab))
    prefill_s = time.time() - t0

    def cycle(n):
        total, done, pos = 0.0, 0, p0
        while done < n:
            m = min(CYCLE, n - done)
            if pos + m > p0 + CYCLE:
                eng.streams_set_position(p0)
                pos = p0
            _, ms = eng.streams_decode(m, return_ms=True)
            total, done, pos = total + ms, done + m, pos + m
        return total

    eng.streams_set_position(p0)
    cycle(max(args.warmup, 3))
    eng.streams_set_position(p0)
    gpu_index = local
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        try:
            gpu_index = int(vis.split(",")[local])
        except ValueError:
            pass
    clocks = ClockSampler(gpu_index)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    if args.profile_window:
        torch.cuda.profiler.start()
    total_ms = cycle(args.steps)
    torch.cuda.synchronize()
    if args.profile_window:
        torch.cuda.profiler.stop()
    clk = clocks.stop()
    if dist:
        dist.barrier()
    value, max_ms = replicas.replica_throughput(args.steps * len(mine), total_ms, world, dist, "cuda")
    ms_step = max_ms / args.steps
    if rank == 0:
        hbm, peak_kind = peaks()
        mean_pos = p0 + 1 + min(args.steps, CYCLE) / 2
        kv_pos_bytes = spec.kv_bytes_per_position() // (2 if args.kv == "f16" else 1)
        step_bytes = info["stream_bytes"] + len(mine) * kv_pos_bytes * mean_pos
        gbs = step_bytes / (ms_step / 1000.0) / 1e9
        line = {
            "metric": f"decode tok/s (2.6B Q4_K_M, {len(mine)} streams per GPU, batched)", "value": value,
            "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": max(args.warmup, 3),
            "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8xint8->int32, f32", "data": "synthetic",
            "config": {"workload": f"M26, {args.streams * world} independent greedy streams, {len(mine)} per GPU, "
                                   f"{plen}-token prompts, positions {p0}..{p0 + CYCLE} "
                                   f"(rewound every {CYCLE} tokens), n_ctx {n_ctx} per stream, {args.kv} K/V cache"
                                   + ("" if p0 == plen else
                                      f"; cache entries {plen}..{p0 - 1} zero-filled (timing case)"),
                       "model": spec.name, "parallelism": f"dp{world} (streams)", "kv": args.kv,
                       "l2": "weights (1.5 GB) and caches exceed L2"},
            "prefill_s_per_gpu": prefill_s,
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                         "peak_kind": peak_kind, "bytes_per_step": step_bytes},
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    eng.close()
    if dist:
        dist.destroy_process_group()


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.streams:
        run_streams(args)
    elif args.tp70:
        run_tp70(args)
    elif args.config1_only:
        import torch

        import pocketinfer as pk
        from pocketinfer import synth

        print(json.dumps({"config1": config1_matvec(pk, synth, torch.device("cuda", 0))}), flush=True)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

#!/usr/bin/env python3
"""Decode benchmark: Qwen3-8B-shape Q4_K_M-mix synthetic GGUF, batch 1, 512-token
random prompt then greedy decode (ctx up to 512 + warmup + steps).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one decode token through every layer (embedding, 36 x {RMSNorm+QKV,
QK-norm+RoPE+KV append, paged GQA attention, o-proj+residual, RMSNorm+gate/up+SwiGLU,
down+residual}, final norm, LM head, argmax). With N > 1 (torchrun) the model is
tensor-parallel over N GPUs (Megatron split; the o-proj and down partial sums and the
greedy pick over the vocabulary shards go through peer-memory inboxes over NVLink).

Printed JSON (rank 0): value = tok/s timed on the device with CUDA events on the
session stream, weights and KV (f32 pages, the reference's precision) resident in HBM,
inputs larger than L2 (5 GB of weights per step); e2e = the same through
evl_session_step with host buffers (token H2D, logits D2H and the host argmax every
step, same context range); roofline = the dominant kernel (Q4_K dequant-matvec of the
ffn_gate shape 12288x4096) timed live; cpu_baseline = the CPU oracle (a restatement of
the reference's runtime) on a bounded sample. Extra keys: bs32 (32 sequences, 2048-token
prefix each, f16 KV pages, at every N), c1 (Qwen3-0.6B shape, all Q8_0, bs1, N = 1),
c4 (the isolated kernel sweep, N = 1), c5 (Qwen3-32B shape, 8 sequences, N > 1), hybrid
(a Qwen3.5-style gated-delta / gated-query hybrid, bs1, N = 1).
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Qwen3-8B-shape Q4_K decode tok/s (bs1, bs32) and % of HBM roofline"
PROMPT = 512


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 100 ms around the timed regions."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": float(max(mx)), "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup(n):
    if n <= 1:
        return 0, 1, 0
    import torch.distributed as dist
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=600))
    return rank, world, local


def dist_max(x: float, world: int) -> float:
    if world <= 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def cpu_baseline(img, seconds: float = 20.0, max_steps: int = 8):
    """The CPU oracle on this host: one 8B decode step at context PROMPT (synthetic KV
    prefix), repeated until `seconds` of CPU work or `max_steps` steps."""
    from oracle import oracle as orc
    threads = os.cpu_count() or 1
    orc.set_threads(threads)
    m = orc.Model(img)
    s = orc.Session(m)
    s.fill_kv(PROMPT, seed=7)
    s.step(1)  # warm the page cache / thread pool
    n, t0 = 0, time.perf_counter()
    tok = 2
    while n < max_steps:
        lg = s.step(tok)
        tok = orc.argmax(lg)
        n += 1
        if time.perf_counter() - t0 > seconds:
            break
    dt = time.perf_counter() - t0
    return {"value": n / dt, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"{n} decode steps of the 8B-shape model at context {PROMPT + 1}..{PROMPT + n} "
                      f"(synthetic KV prefix), CPU oracle restating src/runtime.rs, {threads} threads"}


def profiled_traffic(name):
    """DRAM bytes (read + write) per launch from the committed ncu summary
    profiles/<name>.md (its `traffic_bytes_per_launch:` line), or None."""
    p = os.path.join(os.path.dirname(os.path.abspath(__file__)), "profiles", name + ".md")
    try:
        with open(p) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_launch:"):
                    return int(line.split(":", 1)[1].strip())
    except OSError:
        pass
    return None


def kernel_roofline(evl_rt, stream, hbm_peak, peak_kind, reps=8):
    """Time the dominant kernel (Q4_K dequant-matvec, ffn_gate shape 12288x4096) with CUDA
    events on its stream, cycling 8 distinct matrices (226 MB > L2)."""
    import torch
    from evelyn_b200 import synth
    rows, cols = 12288, 4096
    rng = np.random.default_rng(1)
    mats = []
    lib = evl_rt.lib()
    w = (rng.standard_normal(rows * cols) * 0.02).astype(np.float32)
    raw = np.frombuffer(synth.encode(synth.GGML_Q4_K, w), dtype=np.uint8)
    for i in range(8):
        h = C.c_void_p()
        raw_i = raw.copy()
        raw_i[16::144] ^= np.uint8(i)  # distinct payloads, same statistics
        evl_rt.check(lib.evl_qmatrix_create(synth.GGML_Q4_K, rows, cols, C.c_void_p(raw_i.ctypes.data), 0,
                                            C.byref(h)))
        mats.append(h)
    x = torch.randn(cols, device="cuda:0")
    y = torch.empty(rows, device="cuda:0")
    ext = torch.cuda.ExternalStream(stream)
    for h in mats:  # warm up
        evl_rt.check(lib.evl_qmatrix_matvec(h, C.c_void_p(x.data_ptr()), C.c_void_p(y.data_ptr()), C.c_void_p(stream)))
    torch.cuda.synchronize()
    # the launches queue up behind a device-side sleep, so the kernels run back to back
    # and the events bracket device time only (not the host's per-call overhead)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(ext):
        torch.cuda._sleep(int(20e-3 * 1.9e9))
    e0.record(ext)
    for _ in range(reps):
        for h in mats:
            evl_rt.check(lib.evl_qmatrix_matvec(h, C.c_void_p(x.data_ptr()), C.c_void_p(y.data_ptr()),
                                                C.c_void_p(stream)))
    e1.record(ext)
    torch.cuda.synchronize()
    evs = [(e0, e1)] * (reps * len(mats))
    ms = e0.elapsed_time(e1) / len(evs)
    alg = rows * cols // 256 * 144 + cols * 4 + rows * 4
    for h in mats:
        lib.evl_qmatrix_free(h)
    gbs = alg / (ms * 1e-3) / 1e9
    return {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm_peak, "unit": "GB/s",
            "frac": round(gbs / hbm_peak, 4), "traffic": profiled_traffic("qmatvec_q4k_12288x4096"),
            "traffic_source": "copied from profiles/qmatvec_q4k_12288x4096.md (one ncu capture of this kernel "
                              "and shape), not measured in this run",
            "peak_source": peak_kind,
            "kernel": "qmatvec_kernel (Q4_K, 12288x4096, ffn_gate shape)", "launch_us": round(ms * 1e3, 2),
            "bytes_per_launch": alg}


def measure_bs1(evl, model, spec, prompt_len, K, W, world):
    """One sequence: `prompt_len` prompt tokens fed step by step, W warm-up steps, then
    K timed device-resident greedy steps (device time on the session stream, max over
    ranks); then the same context range end to end through evl_session_step (token H2D,
    logits D2H and the host argmax every step)."""
    import torch
    max_ctx = prompt_len + 2 * (W + K) + 16
    prompt = np.random.default_rng(0).integers(0, spec.vocab, prompt_len)
    sess = evl.Session(model, max_ctx=max_ctx)
    for t in prompt[:-1]:
        sess.step(int(t), logits=False)
    toks = sess.generate(int(prompt[-1]), W)
    ext = torch.cuda.ExternalStream(sess.stream)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    ctx0 = sess.pos
    e0.record(ext)
    torch.cuda.nvtx.range_push("decode_steps")
    sess.generate(toks[-1], K)
    torch.cuda.nvtx.range_pop()
    e1.record(ext)
    e1.synchronize()
    torch.cuda.synchronize()
    ms = dist_max(e0.elapsed_time(e1), world)
    kernels = sess.kernels_per_step
    del sess
    sess = evl.Session(model, max_ctx=max_ctx)
    for t in prompt[:-1]:
        sess.step(int(t), logits=False)
    tok = int(prompt[-1])
    for _ in range(W):
        tok = evl.argmax(sess.step(tok))
    ext = torch.cuda.ExternalStream(sess.stream)
    barrier(world)
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(ext)
    for _ in range(K):
        tok = evl.argmax(sess.step(tok))
    f1.record(ext)
    f1.synchronize()
    e2e_ms = dist_max(f0.elapsed_time(f1), world)
    del sess
    return {"ms": ms, "e2e_ms": e2e_ms, "ctx0": ctx0, "kernels": kernels}


def step_hbm(spec, kv_elem, ctx0, K, hbm, peak_kind, ms, batch=1, world=1):
    """Weight bytes (every matrix once) + KV bytes read over the timed context range,
    per step, against the measured copy bandwidth; with tensor parallelism the bytes
    are spread over `world` GPUs (reported per GPU)."""
    kv_pos = spec.kv_bytes_per_position(kv_elem)
    step_bytes = spec.weight_bytes_per_token() + batch * kv_pos * (ctx0 + (K + 1) / 2)
    gbs = step_bytes * K / (ms / 1e3) / 1e9 / world
    return {"bytes_per_step": int(step_bytes), "achieved_gbs_per_gpu": round(gbs, 1), "frac": round(gbs / hbm, 4),
            "peak": hbm, "peak_source": peak_kind}


def run_ours(args):
    rank, world, local = dist_setup(args.gpus)
    import torch
    torch.cuda.set_device(local)
    import evelyn_b200 as evl
    from evelyn_b200 import runtime, synth

    spec = synth.qwen3_8b(seed=0)
    t0 = time.perf_counter()
    img = synth.build(spec)
    log(f"[rank {rank}] synthetic GGUF {img.nbytes / 1e9:.2f} GB in {time.perf_counter() - t0:.1f}s")

    def load(image, kv_f32):
        nccl_id = None
        if world > 1:
            import torch.distributed as dist
            obj = [evl.tp_unique_id() if rank == 0 else None]
            dist.broadcast_object_list(obj, src=0)
            nccl_id = obj[0]
        t = time.perf_counter()
        m = evl.Model.load_memory(image, device=local, tp_rank=rank, tp_size=world, nccl_id=nccl_id, kv_f32=kv_f32)
        log(f"[rank {rank}] loaded in {time.perf_counter() - t:.1f}s; {m.weight_bytes / 1e9:.3f} GB/step on this rank")
        return m

    K, W = args.steps, args.warmup
    hbm, peak_kind = peaks()
    # clocks are sampled from the first warm-up on (one timed region alone can be
    # shorter than a sampling period) through every timed loop below
    clk = ClockSampler(local).__enter__()
    # bs1 keeps the KV cache in f32 pages, the reference's precision (src/runtime.rs:
    # 721-722), at which the logits are parity-tested against the oracle
    model = load(img, kv_f32=True)
    r1 = measure_bs1(evl, model, spec, PROMPT, K, W, world)
    roof = None
    if rank == 0:  # on a stream of its own (a session would be a collective under TP)
        roof = kernel_roofline(runtime, torch.cuda.Stream().cuda_stream, hbm, peak_kind)
    del model
    base = cpu_baseline(img) if (rank == 0 and world == 1 and not args.no_cpu_baseline) else None
    bs32 = None
    if args.batch > 1:  # the batched config: f16 KV pages, as the config names them
        model = load(img, kv_f32=False)
        bs32 = run_batch(model, spec, args, hbm, peak_kind, world)
        del model
    c5 = None
    if world > 1 and not args.no_c5:  # Qwen3-32B shape, bs8, tensor-parallel
        c5 = run_c5(evl, synth, args, hbm, peak_kind, rank, world, local)
    c1 = None
    if world == 1 and not args.no_c1:  # Qwen3-0.6B shape, all Q8_0, bs1, 128 + 128
        spec1 = synth.qwen3_0_6b(seed=0)
        img1 = synth.build(spec1)
        m1 = evl.Model.load_memory(img1, device=local, kv_f32=True)
        r = measure_bs1(evl, m1, spec1, 128, 128, W, world)
        c1 = {"value": round(128 / (r["ms"] / 1e3), 2), "unit": "tok/s", "ms_per_step": round(r["ms"] / 128, 4),
              "e2e": {"value": round(128 / (r["e2e_ms"] / 1e3), 2), "unit": "tok/s"},
              "workload": f"Qwen3-0.6B-shape all-Q8_0 decode bs1, 128-token prompt then 128 greedy steps "
                          f"(ctx {r['ctx0']}..{r['ctx0'] + 128}), f32 KV pages",
              "step_hbm": step_hbm(spec1, 4, r["ctx0"], 128, hbm, peak_kind, r["ms"])}
        del m1
    hybrid = None
    if world == 1 and not args.no_hybrid:  # Qwen3.5-style gated-delta / gated-query hybrid, bs1
        hybrid = run_hybrid(evl, synth, args, hbm, peak_kind, local, W)
    c4 = run_c4_summary(args, hbm, peak_kind) if (rank == 0 and world == 1 and not args.no_c4) else None
    clk.__exit__(None, None, None)
    tok_s = K / (r1["ms"] / 1e3)
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(tok_s, 2), "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": round(r1["ms"] / K, 4), "higher_is_better": True,
            "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
            "dtype": "q4_k/q6_k/q8_0 weights, f32 math",
            "data": "synthetic: seeded N(0,0.02) weights quantised to a Q4_K_M-style mix, uniform-random prompt ids",
            "config": {"workload": f"Qwen3-8B-shape decode bs1, {PROMPT}-token prompt then greedy decode "
                                   f"(ctx {r1['ctx0']}..{r1['ctx0'] + K})", "model": "qwen3-8b-shape (36L, d4096, "
                       "32Q/8KV x128, ffn 12288, vocab 151936)", "global_batch": 1, "seq_len": r1["ctx0"] + K,
                       "parallelism": f"tp{world}" if world > 1 else "single GPU",
                       "kv_cache": "paged f32 (the reference's precision), 16-token pages",
                       "l2": "inputs larger than L2 (5.08 GB weights/step)"},
            "step_hbm": step_hbm(spec, 4, r1["ctx0"], K, hbm, peak_kind, r1["ms"], world=world),
            "e2e": {"value": round(K / (r1["e2e_ms"] / 1e3), 2), "unit": "tok/s", "h2d_bytes_per_step": 4,
                    "d2h_bytes_per_step": spec.vocab * 4 + 4 + 4},
            "roofline": roof,
            "gpu_launches": r1["kernels"] * K,
            "kernels_per_step": r1["kernels"],
            "clocks": clk.summary(),
        }
        if base:
            line["cpu_baseline"] = base
        if bs32:
            line["bs32"] = bs32
        if c1:
            line["c1"] = c1
        if c4:
            line["c4"] = c4
        if c5:
            line["c5"] = c5
        if hybrid:
            line["hybrid"] = hybrid
        emit_line(line)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def run_hybrid(evl, synth, args, hbm, peak_kind, local, W, prompt_len=128, K=None, cpu_steps=3):
    """Qwen3.5-style hybrid decoder (synth.qwen35_hybrid_2b), bs1: 128 prompt tokens then
    128 timed greedy steps, device time and end to end, like the headline line. Step
    bytes: the engine's weight bytes, the full-attention layers' f32 KV over the timed
    range, and the gated-delta layers' f32 recurrent state read and written; then the
    oracle on the host cores for a few steps (the same prompt start)."""
    K = K or args.hybrid_steps
    spec = synth.qwen35_hybrid_2b(seed=0)
    img = synth.build(spec)
    m = evl.Model.load_memory(img, device=local, kv_f32=True)
    sc = m.ssm_config
    r = measure_bs1(evl, m, spec, prompt_len, K, W, 1)
    full_layers = spec.layers - sc["delta_layers"]
    kv_pos = 2 * full_layers * spec.kv_heads * spec.head_dim * 4
    vd = spec.ssm_inner // spec.ssm_value_heads
    state = sc["delta_layers"] * spec.ssm_value_heads * spec.ssm_state * vd * 4 * 2
    step_bytes = m.weight_bytes + kv_pos * (r["ctx0"] + (K + 1) / 2) + state
    gbs = step_bytes * K / (r["ms"] / 1e3) / 1e9
    out = {"value": round(K / (r["ms"] / 1e3), 2), "unit": "tok/s", "ms_per_step": round(r["ms"] / K, 4),
           "e2e": {"value": round(K / (r["e2e_ms"] / 1e3), 2), "unit": "tok/s"},
           "workload": f"Qwen3.5-style hybrid decode bs1 ({spec.layers}L: {sc['delta_layers']} gated-delta + "
                       f"{full_layers} gated full-attention, d{spec.dim}, {spec.ssm_value_heads} value heads x "
                       f"{spec.ssm_state}x{vd} state, head_dim {spec.head_dim}), {prompt_len}-token prompt then "
                       f"{K} greedy steps (ctx {r['ctx0']}..{r['ctx0'] + K}), f32 KV pages",
           "kernels_per_step": r["kernels"],
           "step_hbm": {"bytes_per_step": int(step_bytes), "recurrent_state_bytes": state,
                        "achieved_gbs_per_gpu": round(gbs, 1), "frac": round(gbs / hbm, 4), "peak": hbm,
                        "peak_source": peak_kind}}
    del m
    if not args.no_cpu_baseline:
        from oracle import oracle as orc
        orc.set_threads(os.cpu_count() or 1)
        om = orc.Model(img)
        sess = orc.Session(om)
        toks = np.random.default_rng(0).integers(0, spec.vocab, cpu_steps + 1)
        sess.step(int(toks[0]))
        t = time.perf_counter()
        for tk in toks[1:]:
            sess.step(int(tk))
        sec = time.perf_counter() - t
        out["cpu_baseline"] = {"value": round(cpu_steps / sec, 3), "unit": "tok/s", "cores": orc.threads(),
                               "kind": "port", "sample": f"{cpu_steps} oracle steps at ctx 1..{cpu_steps + 1}"}
        del sess, om
    return out


def prefill_batch(batch, B, P, vocab, rng, world):
    """Every sequence's P-token random prefix through evl_batch_prefill (32-position
    chunks on the tensor cores), host-synchronised: the prefill line."""
    prompts = [rng.integers(0, vocab, P) for _ in range(B)]
    barrier(world)
    t = time.perf_counter()
    for i in range(B):
        batch.prefill(i, prompts[i])
    barrier(world)
    sec = dist_max(time.perf_counter() - t, world)
    return {"value": round(B * P / sec, 1), "unit": "tok/s", "tokens": B * P, "seconds": round(sec, 3),
            "note": "evl_batch_prefill per sequence, 32-position chunks, wall clock with a barrier on both sides"}


def run_c5(evl, synth, args, hbm, peak_kind, rank, world, local):
    """Qwen3-32B shape (Q4_K_M-style mix) tensor-parallel over the ranks: 8 sequences,
    each prefilled with an args.c5_prompt-token random prompt, then args.c5_steps timed
    batched greedy steps. Rank 0 builds the synthetic GGUF once and writes it to a
    temporary file that every rank maps; any failure (disk, memory) on any rank gives
    an "unavailable" entry on all of them."""
    import shutil
    import tempfile
    import torch
    import torch.distributed as dist
    spec = synth.qwen3_32b(seed=0)
    obj = [None, None]
    if rank == 0:
        d = None
        try:
            t = time.perf_counter()
            img = synth.build(spec)
            d = tempfile.mkdtemp(prefix="evl_c5_")
            path = os.path.join(d, "qwen3_32b_shape.gguf")
            img.write(path)
            log(f"[rank 0] 32B synthetic GGUF {img.nbytes / 1e9:.2f} GB in {time.perf_counter() - t:.1f}s")
            img.close()
            obj = [path, None]
        except Exception as e:  # noqa: BLE001 - reported in the line
            if d:
                shutil.rmtree(d, ignore_errors=True)
            obj = [None, f"building the 32B image: {type(e).__name__}: {e}"]
    dist.broadcast_object_list(obj, src=0)
    path, err = obj
    if err:
        return {"unavailable": err}
    ids = [evl.tp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(ids, src=0)
    model, err = None, None
    try:
        model = evl.Model.load(path, device=local, tp_rank=rank, tp_size=world, nccl_id=ids[0], kv_f32=False)
    except Exception as e:  # noqa: BLE001
        err = f"rank {rank} loading the 32B image: {type(e).__name__}: {e}"
    errs = [None] * world
    dist.all_gather_object(errs, err)
    if rank == 0:
        shutil.rmtree(os.path.dirname(path), ignore_errors=True)
    errs = [e for e in errs if e]
    if errs:
        del model
        return {"unavailable": errs[0]}
    B, P, K = 8, args.c5_prompt, args.c5_steps
    err, ms = None, 0.0
    try:
        bat = evl.Batch(model, B, max_ctx=P + K + 8)
        rng = np.random.default_rng(5)
        pf = prefill_batch(bat, B, P, spec.vocab, rng, world)
        toks = rng.integers(0, spec.vocab, B)
        for _ in range(3):  # warm-up
            toks = bat.step(toks, logits=False)
        ext = torch.cuda.ExternalStream(bat.stream)
        barrier(world)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(ext)
        for _ in range(K):
            toks = bat.step(toks, logits=False)
        e1.record(ext)
        e1.synchronize()
        ms = e0.elapsed_time(e1)
        del bat
    except Exception as e:  # noqa: BLE001 - reported in the line; every rank learns of it below
        err = f"rank {rank}: {type(e).__name__}: {e}"
    errs = [None] * world
    dist.all_gather_object(errs, err)
    del model
    errs = [e for e in errs if e]
    if errs:
        return {"unavailable": errs[0]}
    ms = dist_max(ms, world)
    ctx0 = P + 3
    return {"value": round(B * K / (ms / 1e3), 1), "unit": "tok/s", "ms_per_step": round(ms / K, 4),
            "global_batch": B, "parallelism": f"tp{world}",
            "workload": f"Qwen3-32B-shape (64L, d5120, 64Q/8KV x128, ffn 25600) Q4_K_M-style mix, {B} sequences, "
                        f"{P}-token random prompt each, then {K} greedy steps (ctx {ctx0}..{ctx0 + K}); f16 KV pages",
            "prefill": pf, "step_hbm": step_hbm(spec, 2, ctx0, K, hbm, peak_kind, ms, batch=B, world=world)}


def run_batch(model, spec, args, hbm, peak_kind, world=1):
    """The batched half of the metric: `args.batch` sequences decoded together after a
    `args.batch_prefix`-token prefix each (evl_batch_prefill); K timed steps through
    evl_batch_step (tokens H2D, argmax D2H, synchronised each step)."""
    import torch
    from evelyn_b200 import runtime as evl_rt
    B, P, K = args.batch, args.batch_prefix, args.batch_steps
    batch = evl_rt.Batch(model, B, max_ctx=P + K + 8)
    rng = np.random.default_rng(1)
    pf = prefill_batch(batch, B, P, spec.vocab, rng, world)
    toks = rng.integers(0, spec.vocab, B)
    for _ in range(3):  # warm-up
        toks = batch.step(toks, logits=False)
    ext = torch.cuda.ExternalStream(batch.stream)
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(ext)
    torch.cuda.nvtx.range_push("batch_steps")  # lets a profiler select the timed steps
    for _ in range(K):
        toks = batch.step(toks, logits=False)
    torch.cuda.nvtx.range_pop()
    e1.record(ext)
    e1.synchronize()
    ms = dist_max(e0.elapsed_time(e1), world)
    ctx0 = P + 3
    del batch
    return {"value": round(B * K / (ms / 1e3), 1), "unit": "tok/s", "ms_per_step": round(ms / K, 4),
            "global_batch": B, "workload": f"{B} sequences, {P}-token prefix each, then {K} greedy steps "
                                           f"(ctx {ctx0}..{ctx0 + K}); products on tcgen05 tensor cores",
            "prefill": pf,
            "e2e_note": "each step through evl_batch_step: token ids H2D, argmax D2H, synchronised",
            "parallelism": f"tp{world}" if world > 1 else "single GPU", "kv_cache": "paged f16, 16-token pages",
            "step_hbm": step_hbm(spec, 2, ctx0, K, hbm, peak_kind, ms, batch=B, world=world)}


def _random_raw(ggml_type: int, rows: int, cols: int, rng) -> np.ndarray:
    """Random GGUF rows with moderate f16 scales (bandwidth does not depend on values)."""
    from evelyn_b200 import synth
    be = 32 if ggml_type == synth.GGML_Q8_0 else 256
    bb = synth.type_bytes(ggml_type, be)
    nb = rows * cols // be
    raw = rng.integers(0, 256, size=(nb, bb), dtype=np.uint8)
    scale = np.full(nb, 0.004, dtype=np.float16).view(np.uint8).reshape(nb, 2)
    if ggml_type == synth.GGML_Q6_K:
        raw[:, 208:210] = scale
    else:
        raw[:, 0:2] = scale
        if ggml_type == synth.GGML_Q4_K:
            raw[:, 2:4] = scale
    return raw.reshape(-1)


def run_sweep(args, emit=None):
    """Isolated kernel sweep: dequant-matvec for 4096x4096, 4096x12288, 12288x4096, 151936x4096
    in Q4_K/Q6_K/Q8_0, and GQA decode attention 32Q/8KV hd128 at KV length 512..32768.
    Each case cycles enough distinct copies to exceed L2 twice; CUDA events on one stream.
    Every case's result goes to `emit` (default: one JSON line on stdout)."""
    if emit is None:
        emit = emit_line
    import torch
    from evelyn_b200 import runtime, synth
    lib = runtime.lib()
    hbm, peak_kind = peaks()
    only = set(args.sweep_only.split(",")) if args.sweep_only else None
    stream = torch.cuda.Stream()
    sp = C.c_void_p(stream.cuda_stream)
    rng = np.random.default_rng(0)
    names = {synth.GGML_Q4_K: "q4k", synth.GGML_Q6_K: "q6k", synth.GGML_Q8_0: "q8_0"}
    for rows, cols in [(4096, 4096), (4096, 12288), (12288, 4096), (151936, 4096)]:
        for t in (synth.GGML_Q4_K, synth.GGML_Q6_K, synth.GGML_Q8_0):
            name = f"{names[t]}_{rows}x{cols}"
            if only and name not in only:
                continue
            raw = _random_raw(t, rows, cols, rng)
            nbytes = raw.size
            copies = max(1, -(-2 * 126 * 2**20 // nbytes))
            mats = []
            for i in range(copies):
                h = C.c_void_p()
                r = raw.copy()
                r[7::97] ^= np.uint8(i)
                runtime.check(lib.evl_qmatrix_create(t, rows, cols, C.c_void_p(r.ctypes.data), 0, C.byref(h)))
                mats.append(h)
            x = torch.randn(cols, device="cuda:0")
            y = torch.empty(rows, device="cuda:0")
            px, py = C.c_void_p(x.data_ptr()), C.c_void_p(y.data_ptr())
            for h in mats:
                runtime.check(lib.evl_qmatrix_matvec(h, px, py, sp))
            reps = max(1, args.reps)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            with torch.cuda.stream(stream):  # launches queue behind a device sleep: back to back
                torch.cuda._sleep(int(20e-3 * 1.9e9))
            e0.record(stream)
            for _ in range(reps):
                for h in mats:
                    runtime.check(lib.evl_qmatrix_matvec(h, px, py, sp))
            e1.record(stream)
            e1.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / (reps * len(mats))
            alg = nbytes + 4 * (rows + cols)
            gbs = alg / (us * 1e-6) / 1e9
            emit({"kernel": "qmatvec", "case": name, "bytes": alg, "us": round(us, 2),
                              "gbs": round(gbs, 1), "frac": round(gbs / hbm, 4), "peak": hbm,
                              "peak_source": peak_kind})
            for h in mats:
                lib.evl_qmatrix_free(h)
            del mats
    # batched products on the tensor cores: 32 vectors per call (evl_qmatrix_matmul: input
    # staging, tcgen05 GEMM, split-K reduce; the call synchronises its stream)
    nvec = 32
    for rows, cols in [(4096, 4096), (4096, 12288), (12288, 4096), (151936, 4096)]:
        for t in (synth.GGML_Q4_K, synth.GGML_Q6_K, synth.GGML_Q8_0):
            name = f"gemm_{names[t]}_{rows}x{cols}_n{nvec}"
            if not only or name not in only:
                continue
            raw = _random_raw(t, rows, cols, rng)
            copies = max(1, -(-2 * 126 * 2**20 // raw.size))
            mats = []
            for i in range(copies):
                h = C.c_void_p()
                r = raw.copy()
                r[7::97] ^= np.uint8(i)
                runtime.check(lib.evl_qmatrix_create(t, rows, cols, C.c_void_p(r.ctypes.data), 0, C.byref(h)))
                mats.append(h)
            x = torch.randn(nvec, cols, device="cuda:0")
            y = torch.empty(nvec, rows, device="cuda:0")
            px, py = C.c_void_p(x.data_ptr()), C.c_void_p(y.data_ptr())
            for h in mats:  # builds each matrix's GEMM-layout copy
                runtime.check(lib.evl_qmatrix_matmul(h, px, nvec, py, sp))
            reps = max(1, args.reps)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            e0.record(stream)
            for _ in range(reps):
                for h in mats:
                    runtime.check(lib.evl_qmatrix_matmul(h, px, nvec, py, sp))
            e1.record(stream)
            e1.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / (reps * len(mats))
            flops = 2.0 * rows * cols * nvec
            emit({"kernel": "qgemm (stage + gemm + reduce, synchronised call)", "case": name,
                              "bytes": raw.size + 4 * nvec * (rows + cols), "us": round(us, 2),
                              "tflops": round(flops / (us * 1e-6) / 1e12, 2),
                              "gbs": round(raw.size / (us * 1e-6) / 1e9, 1)})
            for h in mats:
                lib.evl_qmatrix_free(h)
            del mats
    heads, kvh, hd, ps = 32, 8, 128, 16
    L = 512
    while L <= 32768:
        name = f"attn_{L}"
        if not only or name in only:
            pages = L // ps
            kv_bytes = 2 * pages * kvh * ps * hd * 2
            copies = max(1, -(-2 * 126 * 2**20 // kv_bytes))
            kvs = [(torch.randn(pages, kvh, ps, hd, device="cuda:0").half(),
                    torch.randn(pages, kvh, ps, hd, device="cuda:0").half()) for _ in range(copies)]
            pt = torch.arange(pages, dtype=torch.int32, device="cuda:0")
            q = torch.randn(heads * hd, device="cuda:0")
            out = torch.empty(heads * hd, device="cuda:0")
            wsb = lib.evl_attention_workspace_bytes(L, heads, kvh, hd)
            ws = torch.empty(wsb // 4 + 64, dtype=torch.float32, device="cuda:0")
            wp = (ws.data_ptr() + 255) // 256 * 256

            def call(k, v):
                runtime.check(lib.evl_attention_decode_ws(
                    C.c_void_p(q.data_ptr()), C.c_void_p(k.data_ptr()), C.c_void_p(v.data_ptr()),
                    C.c_void_p(pt.data_ptr()), L, heads, kvh, hd, ps, C.c_void_p(out.data_ptr()), C.c_void_p(wp),
                    wsb, sp))
            for k, v in kvs:
                call(k, v)
            reps = max(1, args.reps)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            with torch.cuda.stream(stream):
                torch.cuda._sleep(int(20e-3 * 1.9e9))
            e0.record(stream)
            for _ in range(reps):
                for k, v in kvs:
                    call(k, v)
            e1.record(stream)
            e1.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / (reps * len(kvs))
            alg = kv_bytes + 2 * heads * hd * 4
            gbs = alg / (us * 1e-6) / 1e9
            emit({"kernel": "attention", "case": name, "bytes": alg, "us": round(us, 2),
                              "gbs": round(gbs, 1), "frac": round(gbs / hbm, 4), "peak": hbm,
                              "peak_source": peak_kind})
            del kvs
        L *= 2


def run_c4_summary(args, hbm, peak_kind):
    """The kernel sweep (every matvec shape x type and the decode attention at KV 512 ..
    32768, 3 timed passes each) as one summary for the bench line."""
    import argparse as _ap
    a = _ap.Namespace(sweep_only="", reps=3)
    res = []
    run_sweep(a, emit=res.append)
    out = {"workload": "isolated kernels: dequant-matvec 4096x4096, 4096x12288, 12288x4096, 151936x4096 in "
                       "Q4_K/Q6_K/Q8_0 (x f32), GQA decode attention 32Q/8KV hd128 over f16 pages at KV "
                       "512..32768; each case cycles distinct copies larger than L2",
           "peak": hbm, "peak_source": peak_kind}
    for d in res:
        out[f"{d['kernel']}:{d['case']}"] = {"us": d["us"], "gbs": d["gbs"], "frac": d.get("frac")}
    return out


def run_reference(args):
    """The reference's CPU runtime (the oracle port: cargo/rustc are not in this image) on the
    host cores, same metric and workload; each step one 8B decode token at ctx >= 512."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from evelyn_b200 import synth
    from oracle import oracle as orc
    spec = synth.qwen3_8b(seed=0)
    img = synth.build(spec)
    threads = os.cpu_count() or 1
    orc.set_threads(threads)
    m = orc.Model(img)
    s = orc.Session(m)
    s.fill_kv(PROMPT, seed=7)
    tok = 1
    budget = 90.0
    for _ in range(min(args.warmup, 1)):
        tok = orc.argmax(s.step(tok))
    n, t0 = 0, time.perf_counter()
    while n < args.steps:
        tok = orc.argmax(s.step(tok))
        n += 1
        if time.perf_counter() - t0 > budget:
            break
    dt = time.perf_counter() - t0
    v = n / dt
    sample = (f"{n} of {args.steps} requested decode steps (capped at {budget:.0f}s) at ctx {PROMPT + 1}.., "
              f"synthetic KV prefix, {threads} threads")
    emit_line({
        "impl": "reference", "metric": METRIC, "value": round(v, 4), "unit": "tok/s", "n_gpus": args.gpus,
        "steps": n, "warmup": min(args.warmup, 1), "ms_per_step": round(dt / n * 1e3, 2), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"Qwen3-8B-shape decode bs1, ctx {PROMPT}+ (CPU, sampled)"},
        "cpu_baseline": {"value": round(v, 4), "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": round(v, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    })


_RESULT_FD = None


def emit_line(d):
    """Writes one JSON result line to the process's original stdout. Everything else the
    process prints (NCCL's version banner, library messages) goes to stderr, so stdout
    carries the result lines only."""
    os.write(_RESULT_FD if _RESULT_FD is not None else 1, (json.dumps(d) + "\n").encode())


def main():
    global _RESULT_FD
    sys.stdout.flush()
    _RESULT_FD = os.dup(1)
    os.dup2(2, 1)
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1024)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--prompt", type=int, default=512, help="prompt tokens fed before decoding")
    ap.add_argument("--sweep", action="store_true", help="isolated kernel sweep (one JSON line per case)")
    ap.add_argument("--sweep-only", default="", help="comma-separated sweep case names")
    ap.add_argument("--batch", type=int, default=32, help="sequences of the batched measurement (0: skip)")
    ap.add_argument("--batch-prefix", type=int, default=2048, help="prefix tokens per sequence before timing")
    ap.add_argument("--batch-steps", type=int, default=64, help="timed batched steps")
    ap.add_argument("--reps", type=int, default=10, help="timed passes per sweep case")
    ap.add_argument("--no-c1", action="store_true", help="skip the Qwen3-0.6B-shape bs1 line")
    ap.add_argument("--no-c4", action="store_true", help="skip the kernel-sweep summary")
    ap.add_argument("--no-hybrid", action="store_true", help="skip the Qwen3.5-style hybrid line")
    ap.add_argument("--hybrid-steps", type=int, default=128, help="timed steps of the hybrid line")
    ap.add_argument("--hybrid-only", action="store_true",
                    help="only the hybrid line, printed as its own JSON object (N = 1)")
    ap.add_argument("--no-c5", action="store_true", help="skip the Qwen3-32B-shape bs8 line (N > 1 only)")
    ap.add_argument("--c5-prompt", type=int, default=4096, help="prompt tokens per sequence of the 32B line")
    ap.add_argument("--c5-steps", type=int, default=64, help="timed batched steps of the 32B line")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    global PROMPT
    PROMPT = max(1, args.prompt)
    if args.sweep:
        run_sweep(args)
    elif args.hybrid_only:
        import torch
        import evelyn_b200 as evl
        from evelyn_b200 import synth
        torch.cuda.set_device(0)
        hbm, peak_kind = peaks()
        emit_line({"hybrid": run_hybrid(evl, synth, args, hbm, peak_kind, 0, args.warmup)})
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

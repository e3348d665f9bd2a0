"""Decode benchmark: batch-1 greedy decode tokens/s and % of the HBM roofline at 4k context.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (benchmark configuration 2 at "4k ctx"): the 36-layer Qwen3-8B-architecture model with seeded random-init
FP8 weights (E4M3, per-output-channel fp32 scales), bf16 embeddings, FP8 per-channel lm_head (151936 rows),
a bf16 KV cache sized for 4096 tokens pre-filled with N(0,1) up to position 4096-K, then K greedy decode
steps under one CUDA graph (ctx 4096-K .. 4095). One step = one token. Every step reads ~8.2 GB (weights +
KV), far more than the 126 MB L2, so no L2 flush is needed between steps.

Timing: W untimed warm-up steps, state reset, then exactly K graph replays between CUDA events on the
replay stream, with a synchronize (and for N>1 a barrier) on both sides; max over ranks. `e2e` repeats the
K steps through the public engine API with, every step, the input token copied from pinned host memory
and the output token read back to pinned host memory (host-synchronous streaming decode).

N > 1: tensor parallelism over the N GPUs (tp.py: Megatron-style shards, vocab-parallel lm_head), one process
per GPU. Default: the fused TP step (one persistent launch per token and rank, the fp32 partials of o_proj
and down exchanged inside the kernel over NVLink); --path ops: the op-by-op engine with NCCL all-reduces.
The same 4k-context workload
(scaling "strong": the job decodes one token stream; value = tokens/s of that stream). The step time is the
max over ranks.

--impl reference: the reference engine's CPU path (its `model.forward` math restated in oracle/, run on the
host cores with all threads), one decoder layer per step at the same context plus the lm_head, reported as
tokens/s of the full 36-layer step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "inferencekit-engines_b200")
for _p in (REPO, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

METRIC = "batch-1 decode tokens/s at 4k ctx (Qwen3-8B FP8, per-channel scales, FP8 lm_head)"
UNIT = "tokens/s"
FALLBACK_HBM_GBS = 6650.0


def peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


class ClockSampler:
    """nvidia-smi clock/throttle samples while the timed region runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.gpu), "-lms", "50"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            time.sleep(0.3)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.out = ""
        if self.proc is not None:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def summary(self):
        rows = [r.split(", ") for r in (self.out or "").strip().splitlines() if r.count(",") >= 8]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no nvidia-smi samples"]}
        sm = [float(r[1]) for r in rows]
        smax = float(rows[0][2])
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for n, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(n)
        under = [s for s in sm if s > 0.5 * smax] or sm
        return {"sm_mhz": statistics.median(under), "sm_max_mhz": smax, "samples": len(sm),
                "power_w_max": max(float(r[3]) for r in rows), "reasons": sorted(reasons)}


def step_bytes(m, ctx_lo, ctx_hi):
    """Algorithmic bytes per token, averaged over the contexts the timed steps see."""
    wb = m.weight_bytes()
    fixed = sum(wb.values())
    kv = m.kv_bytes_per_token((ctx_lo + ctx_hi) / 2.0)
    return fixed + kv, wb


def gate_up_kernel_timing(eng, reps):
    """The dominant kernel (gate_up GEMV, 52% of the step's weight bytes) timed alone with CUDA events on
    the launching stream, cycling through the 36 layers' weights (3.6 GB, no L2 reuse)."""
    m = eng.m
    s = torch.cuda.current_stream()
    for L in m.layers[:4]:
        eng._gemv(2, L.gu, eng.resid, L.ln2, eng.h)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = 0
    e0.record(s)
    for r in range(reps):
        for L in m.layers:
            eng._gemv(2, L.gu, eng.resid, L.ln2, eng.h)
            n += 1
    e1.record(s)
    torch.cuda.synchronize()
    L = m.layers[0]
    H = m.cfg.hidden
    bytes_per_launch = L.gu.packed.numel() + 4 * L.gu.scale.numel() + 2 * H + 2 * H + 2 * (L.gu.N // 2)
    return e0.elapsed_time(e1) / n * 1e-3, bytes_per_launch, n


def load_traffic(name):
    p = os.path.join(REPO, "profiles", name)
    try:
        with open(p) as f:
            return json.load(f)
    except (OSError, ValueError):
        return None


def step_traffic(bytes_tok):
    """DRAM bytes of one full-size decode_step launch, scaled from the ncu capture of the 2-layer profiling
    model (profiles/decode_step_traffic.json: dram__bytes_read.sum + dram__bytes_write.sum of one launch and
    that model's algorithmic bytes); traffic grows with the bytes streamed."""
    t = load_traffic("decode_step_traffic.json")
    if not t:
        return None
    return t["dram_bytes_per_launch"] * bytes_tok / t["algorithmic_bytes_per_launch"]


def time_replays(replay, reset, K: int, W: int) -> float:
    """Seconds for K replays after W untimed ones (reset() before each group), CUDA events on the current stream."""
    reset()
    for _ in range(W):
        replay()
    torch.cuda.synchronize()
    reset()
    torch.cuda.synchronize()
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(K):
        replay()
    e1.record(s)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1e-3


def ref_format_step(K: int, W: int, peak: float):
    """Our fused step in the reference checkpoint's format (block-128 scales, bf16 lm_head; the only format the
    reference's own kernels run), at the bench's 36-layer 4k-context workload: tokens/s and HBM fraction."""
    import model as M
    from generate import Engine
    cfg = M.Config()
    max_seq, start = 4096, 4096 - K
    m = M.Qwen3FP8Decode.synthetic(cfg, max_seq=max_seq, device="cuda", seed=0, scale_mode="block", head_dtype="bf16",
                                   norm_init="ones")
    m.fill_cache_random(start, seed=1234)
    eng = Engine(m, fused=True)
    eng.token.fill_(1)
    eng.state.copy_(torch.tensor([start, 0], dtype=torch.int32))
    eng.capture()

    def reset():
        eng.token.fill_(1)
        eng.state.copy_(torch.tensor([start, 0], dtype=torch.int32, device="cuda"))

    t = time_replays(eng.graph.replay, reset, K, W)
    eng.check()
    bytes_tok, _ = step_bytes(m, start, max_seq - 1)
    out = {"format": "block-128 scales, bf16 lm_head (the reference checkpoint's)", "engine": "fused step",
           "tok_s": K / t, "ms_per_step": t / K * 1e3, "bytes_per_token": bytes_tok,
           "frac": bytes_tok * K / t / 1e9 / peak}
    del eng, m
    torch.cuda.empty_cache()
    return out


def ref_gpu_step(K: int, W: int, peak: float):
    """The reference's own decode kernels (its kernels/decode.cu built for sm_100a, oracle/_ref) driven as its
    engine drives them (Q/generate.py:102-137: one CUDA graph per step, the shipped launch knobs, chunk-64
    attention, lm_head on every SM), at the same 36-layer 4k-context workload in its checkpoint format."""
    import model as M
    from oracle import ref_gpu as R
    if not R.available():
        return {"unavailable": "oracle/_ref/ref_decode.so was not built (no reference checkout where the tree was built)"}
    cfg = M.Config()
    max_seq, start = 4096, 4096 - K
    m = M.Qwen3FP8Decode.synthetic(cfg, max_seq=max_seq, device="cuda", seed=0, scale_mode="block", head_dtype="bf16",
                                   norm_init="ones", keep_rowmajor=True)
    bytes_tok, _ = step_bytes(m, start, max_seq - 1)
    layers = []
    for L in m.layers:
        layers.append(dict(ln1=L.ln1, ln2=L.ln2, q_norm=L.q_norm, k_norm=L.k_norm,
                           qkv=(L.rowmajor["qkv"], L.qkv.scale), o_proj=(L.rowmajor["o_proj"], L.o.scale),
                           gate_up=(L.rowmajor["gate_up"], L.gu.scale), down_proj=(L.rowmajor["down_proj"], L.down.scale)))
        L.qkv = L.o = L.gu = L.down = None
        L.rowmajor = {}
    ref = R.RefEngine(layers, m.embed, m.norm, m.lm_head, m.cos, m.sin, max_seq)
    del layers
    m.k_cache = m.v_cache = None
    torch.cuda.empty_cache()
    g = torch.Generator(device="cuda")
    g.manual_seed(1234)
    for c in (ref.k_cache, ref.v_cache):
        for li in range(c.shape[0]):
            t = c[li, :, :start]
            t.copy_(torch.randn(t.shape, generator=g, device="cuda", dtype=torch.float32))
    ref.token.fill_(1)
    ref.state.copy_(torch.tensor([start, 0], dtype=torch.int32))
    ref.capture()

    def reset():
        ref.token.fill_(1)
        ref.state.copy_(torch.tensor([start, 0], dtype=torch.int32, device="cuda"))
        ref.best.zero_()

    t = time_replays(ref.graph.replay, reset, K, W)
    out = {"kernels": "reference kernels/decode.cu, sm_100a build (oracle/_ref), 183 launches per step in one graph",
           "format": "block-128 scales, bf16 lm_head", "tok_s": K / t, "ms_per_step": t / K * 1e3,
           "bytes_per_token": bytes_tok, "frac": bytes_tok * K / t / 1e9 / peak}
    del ref, m
    torch.cuda.empty_cache()
    return out


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


def _cpu_layer(ctx: int):
    """One synthetic decoder layer (per-channel FP8, unit norms) and a KV cache pre-filled to `ctx`, for the
    CPU restatement of the reference's forward."""
    import model as M
    from oracle import qwen3_ref as O
    H, I = 4096, 12288
    w = {}
    for name, parts in (("qkv", [("q_proj", 4096), ("k_proj", 1024), ("v_proj", 1024)]),
                        ("gate_up", [("gate_proj", I), ("up_proj", I)])):
        qs = [M.synth_linear(0, "cpu." + n, r, H, "channel") for n, r in parts]
        w[name] = (torch.cat([a for a, _ in qs]), torch.cat([b for _, b in qs]).contiguous())
    w["o_proj"] = M.synth_linear(0, "cpu.o", H, H, "channel")
    w["down_proj"] = M.synth_linear(0, "cpu.d", H, I, "channel")
    ones = torch.ones(H, dtype=torch.bfloat16)
    hd1 = torch.ones(128, dtype=torch.bfloat16)
    L = O.LayerW(ones, ones, hd1, hd1, *w["qkv"], *w["o_proj"], *w["gate_up"], *w["down_proj"])
    return L, ones


def cpu_baseline(ctx: int, budget_s: float = 25.0, threads: int | None = None):
    """The reference's CPU path (oracle restatement of Q/model.py forward with the decode kernel's fp32
    attention) on the host cores, as a bounded sample: a few one-layer decode steps at `ctx` (median) and one
    FP8 lm_head call, extrapolated to the 36-layer step (36 x layer + head)."""
    import model as M
    from oracle import qwen3_ref as O
    threads = threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    H = 4096
    L, ones = _cpu_layer(ctx)
    kc = torch.randn(8, ctx + 1, 128).to(torch.bfloat16)
    vc = torch.randn(8, ctx + 1, 128).to(torch.bfloat16)
    cos, sin = M.rope_tables(ctx + 1, 128, 1e6, "cpu")
    h = torch.randn(H).to(torch.bfloat16)
    times = []
    t_start = time.perf_counter()
    for i in range(8):
        t0 = time.perf_counter()
        O.decode_layer(h, L, kc, vc, ctx, cos, sin, 1e-6, attn_impl="f32")
        times.append(time.perf_counter() - t0)
        if i >= 2 and time.perf_counter() - t_start > budget_s * 0.6:
            break
    layer_s = statistics.median(times[1:]) if len(times) > 1 else times[0]
    hw, hs = M.quantize_fp8(M.randn((151936, H), 0, "cpu.head", std=0.02), "channel")
    O.lm_head_logits(h, ones, hw[:1024], hs[:1024], 1e-6)
    t0 = time.perf_counter()
    O.lm_head_logits(h, ones, hw, hs, 1e-6)
    head_s = time.perf_counter() - t0
    step_s = 36 * layer_s + head_s
    return {"value": 1.0 / step_s, "unit": UNIT, "cores": threads, "cpu_model": cpu_model(), "kind": "port",
            "extrapolated": True, "layers_timed": len(times) - 1 if len(times) > 1 else 1, "head_calls_timed": 1,
            "sample": f"{len(times)} one-layer decode steps at ctx {ctx} (first untimed; median {layer_s * 1e3:.1f} "
                      f"ms) + one FP8 lm_head call ({head_s * 1e3:.0f} ms), extrapolated to 36 layers + head",
            "layer_ms": layer_s * 1e3, "head_ms": head_s * 1e3}


def run_reference(args):
    """The reference's CPU implementation of the decode step (its model.forward math, restated in oracle/)
    on all host cores: whole 36-layer tokens (embedding row, 36 layers, final norm, FP8 lm_head, greedy
    argmax), timed as they run. To keep set-up bounded the 36 layers share one synthetic layer's weights
    (each layer keeps its own KV cache); the arithmetic per token is the full step's. Steps past a time
    budget are not run: `steps` is the number actually timed and `steps_requested` the asked-for K."""
    ws, rank, _ = dist_env()
    if rank != 0:
        return
    import model as M
    from oracle import qwen3_ref as O
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    ctx = 4096 - args.steps
    H, n_layers = 4096, 36
    L, ones = _cpu_layer(ctx)
    g = torch.Generator().manual_seed(1234)
    kcs = [torch.randn(8, 4096, 128, generator=g).to(torch.bfloat16) for _ in range(n_layers)]
    vcs = [torch.randn(8, 4096, 128, generator=g).to(torch.bfloat16) for _ in range(n_layers)]
    cos, sin = M.rope_tables(4096, 128, 1e6, "cpu")
    embed = M.randn((151936, H), 0, "cpu.embed", std=0.02).to(torch.bfloat16)
    hw, hs = M.quantize_fp8(M.randn((151936, H), 0, "cpu.head", std=0.02), "channel")
    layers = [L] * n_layers

    def token_step(tok, pos):
        nxt, _ = O.decode_step(tok, pos, embed, layers, kcs, vcs, cos, sin, ones, hw, hs, 1e-6, attn_impl="f32")
        return nxt

    tok, pos = 1, ctx
    warm = min(args.warmup, 2)
    for _ in range(warm):
        tok = token_step(tok, pos)
    budget_s = float(os.environ.get("QK_REFERENCE_BUDGET_S", "90"))
    tok, pos, done = 1, ctx, 0
    t0 = time.perf_counter()
    while done < args.steps:
        tok = token_step(tok, pos)
        pos += 1
        done += 1
        if time.perf_counter() - t0 > budget_s:
            break
    t = time.perf_counter() - t0
    value = done / t
    base = {"value": value, "unit": UNIT, "cores": threads, "cpu_model": cpu_model(), "kind": "port",
            "extrapolated": False,
            "sample": f"{done} whole decode tokens (36 layers sharing one synthetic layer's weights, own KV caches "
                      f"from ctx {ctx}, FP8 lm_head, greedy argmax) after {warm} untimed"}
    out = {"metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
           "steps": done, "steps_requested": args.steps, "warmup": warm, "ms_per_step": t / done * 1e3,
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
           "dtype": "fp8-e4m3 x fp8 -> fp32 (bf16 activations)",
           "data": "synthetic (seeded random-init weights, N(0,1) KV)",
           "config": {"workload": f"reference CPU path: Qwen3-8B-shape decode step at ctx {ctx}", "global_batch": 1,
                      "seq_len": 4096, "parallelism": "cpu"},
           "cpu_baseline": base,
           "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if torch.cuda.is_available() and not args.no_ref_gpu:
        # the reference's GPU kernels on this box (not the arm's value: the reference arm is its CPU path)
        try:
            out["ref_gpu"] = ref_gpu_step(min(args.steps, 64), args.warmup, peaks()[0])
        except Exception as e:   # report, do not fail the CPU arm
            out["ref_gpu"] = {"unavailable": f"{type(e).__name__}: {e}"[:300]}
    print(json.dumps(out), flush=True)


def run_ours(args):
    import model as M
    from generate import Engine
    ws, rank, local = dist_env()
    if ws > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    dev = f"cuda:{local}" if ws > 1 else "cuda:0"
    torch.cuda.set_device(dev)
    K, W = args.steps, args.warmup
    max_seq = 4096
    start = max_seq - K
    assert start > 0, "--steps must be < 4096"
    cfg = M.Config()
    if ws > 1:
        import tp as TP
        m = TP.synthetic_shard(cfg, ws, rank, max_seq=max_seq, device=dev, seed=args.seed, scale_mode=args.scale,
                               head_dtype=args.head, norm_init="ones")
        m.fill_cache_random(start, seed=1234 + rank)
        fused = args.path == "fused"
        eng = TP.FusedTPEngine(m) if fused else TP.TPEngine(m, attn_chunk=args.chunk)
    else:
        m = M.Qwen3FP8Decode.synthetic(cfg, max_seq=max_seq, device=dev, seed=args.seed, scale_mode=args.scale,
                                       head_dtype=args.head, norm_init="ones")
        m.fill_cache_random(start, seed=1234 + rank)
        fused = args.path == "fused"
        eng = Engine(m, pdl=not args.no_pdl, attn_chunk=args.chunk, fused=fused)
    eng.token.fill_(1)
    eng.state.copy_(torch.tensor([start, 0], dtype=torch.int32))
    eng.capture()

    def reset():
        eng.token.fill_(1)
        eng.state.copy_(torch.tensor([start, 0], dtype=torch.int32, device=dev))
        eng.best.zero_()

    def barrier():
        if ws > 1:
            import torch.distributed as dist
            dist.barrier()

    stream = torch.cuda.current_stream()
    # warm-up
    reset()
    eng.step(W)
    torch.cuda.synchronize()
    reset()
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local if ws > 1 else 0) as clk:
        torch.cuda.synchronize()
        barrier()
        e0.record(stream)
        for _ in range(K):
            eng.graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
    t = e0.elapsed_time(e1) * 1e-3
    tokens = eng.out_tokens[:K].tolist()
    err = eng.k.device_error()
    if err:   # a timed-out wait makes every later wait give up at once: the timing would be of broken steps
        raise RuntimeError(f"decode steps failed on the device (error word {err:#x}); no valid measurement")

    # e2e through the public API: pinned h2d of the step's input token, graph replay, d2h of its output
    reset()
    torch.cuda.synchronize()
    h_in = torch.empty(1, dtype=torch.int32, pin_memory=True)
    h_out = torch.empty(1, dtype=torch.int32, pin_memory=True)
    h_in[0] = 1
    barrier()
    t0 = time.perf_counter()
    for _ in range(K):
        eng.token.copy_(h_in, non_blocking=True)
        eng.graph.replay()
        h_out.copy_(eng.token, non_blocking=True)
        stream.synchronize()
        h_in[0] = h_out[0]
    t_e2e = time.perf_counter() - t0
    barrier()

    peak, peak_src = peaks()
    bytes_tok, wb = step_bytes(m, start, max_seq - 1)
    if fused or ws > 1:
        # fused: the step kernel is the whole step (TP: the rank's, on its shard's bytes)
        k_s, k_bytes, k_n = t / K, bytes_tok, K
    else:
        k_s, k_bytes, k_n = gate_up_kernel_timing(eng, reps=2)   # dominant kernel alone

    if ws > 1:
        import torch.distributed as dist
        tt = torch.tensor([t, t_e2e], dtype=torch.float64, device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t, t_e2e = float(tt[0]), float(tt[1])
    value = K / t
    if rank == 0:
        achieved = k_bytes / k_s / 1e9
        if ws > 1 and fused:
            kname = (f"decode_step_kernel<TP={ws}>: one rank's whole token on 1/{ws} of the weights, KV and "
                     f"lm_head, partials exchanged in-kernel over NVLink")
            traffic = None
        elif ws > 1:
            kname = (f"one TP rank's step ({6 + 6 * len(m.layers)} kernels on 1/{ws} of the weights, KV and "
                     f"lm_head, {2 * len(m.layers) + 1} NCCL all-reduces)")
            traffic = None
        elif fused:
            kname = "decode_step_kernel (the whole token: 36 layers + lm_head, one persistent launch)"
            traffic = step_traffic(bytes_tok)
        else:
            kname = "fp8 gate_up GEMV (SwiGLU epilogue)"
            tr = load_traffic("gate_up_gemv_traffic.json")
            traffic = tr.get("bytes_per_launch") if tr else None
        out = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": K, "warmup": W,
            "ms_per_step": t / K * 1e3, "higher_is_better": True, "scaling": "strong" if ws > 1 else "weak",
            "vs_baseline": None,
            "dtype": "fp8-e4m3 x fp8 -> fp32 (bf16 activations, bf16 KV)", "data": "synthetic (seeded random-init "
            "weights, N(0,1) KV cache, no checkpoint)",
            "config": {"workload": f"Qwen3-8B FP8 decode, 36 layers, per-channel FP8 + FP8 lm_head, KV 4096 "
                                   f"pre-filled to {start}, {K} greedy steps (ctx {start}..{max_seq - 1}), CUDA graph",
                       "global_batch": 1, "seq_len": max_seq, "parallelism": f"tp{ws}",
                       "scale_mode": args.scale, "head": args.head, "attn_chunk": args.chunk, "pdl": not args.no_pdl,
                       "path": ("fused-tp" if fused else "ops+nccl") if ws > 1 else args.path,
                       "l2": "inputs larger than L2 (8.2 GB read per step), no flush"},
            "e2e": {"value": K / t_e2e, "unit": UNIT, "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4},
            # ops path: embed, per layer qkv + attention (partials, merge) + o + gate_up + down, lm_head, finalize
            # (TP also residual_add and two argmax-key flips); NCCL kernels are not counted
            "gpu_launches": K * (1 if fused else (3 + 6 * len(m.layers) + (3 if ws > 1 else 0))),
            "roofline": {"bound": "hbm", "kernel": kname, "achieved": achieved, "peak": peak,
                         "peak_source": f"{peak_src} hbm_gbs (burst copy)", "unit": "GB/s", "frac": achieved / peak,
                         "traffic": traffic, "bytes_per_launch_algorithmic": k_bytes, "launch_us": k_s * 1e6,
                         "launches_timed": k_n},
            "step_roofline": {"bytes_per_token": bytes_tok, "achieved_gbs": bytes_tok * K / t / 1e9,
                              "frac": bytes_tok * K / t / 1e9 / peak, "roofline_tok_s": peak * 1e9 / bytes_tok,
                              "breakdown": dict(wb, kv=int(bytes_tok - sum(wb.values())))},
            "clocks": clk.summary(),
            "device_error": err,
            "tokens_head": tokens[:8],
        }
        if not args.no_cpu_baseline and ws == 1:
            out["cpu_baseline"] = cpu_baseline(start)
        if ws == 1 and fused and not args.no_ref_format:
            del eng, m
            torch.cuda.empty_cache()
            out["ref_format"] = ref_format_step(K, W, peak)
        print(json.dumps(out), flush=True)
    if ws > 1:
        import torch.distributed as dist
        eng.release()
        dist.barrier()
        dist.destroy_process_group()


def run_profile_kernel(args):
    """A few launches of one kernel on one layer's worth of synthetic inputs (for ncu captures)."""
    import model as M
    from kernels import ops
    k = ops()
    k.set_pdl(False)
    dev = "cuda"
    shapes = {"qkv": (0, 6144, 4096), "o_proj": (1, 4096, 4096), "gate_up": (2, 24576, 4096),
              "down": (3, 4096, 12288), "lm_head": (4, 151936, 4096)}
    if args.profile_kernel == "decode_step":
        from generate import Engine
        cfg = M.Config(layers=args.layers, vocab=16384)
        m = M.Qwen3FP8Decode.synthetic(cfg, max_seq=4096, device=dev, seed=0, scale_mode="channel", head_dtype="fp8")
        m.fill_cache_random(3840)
        eng = Engine(m, fused=True)
        eng.token.fill_(1)
        eng.state.copy_(torch.tensor([3840, 0], dtype=torch.int32))
        for _ in range(args.launches):
            eng.decode_step()
        torch.cuda.synchronize()
        pos0 = 3840
        alg, _ = step_bytes(m, pos0, pos0 + args.launches - 1)
        print(f"profiled decode_step ({args.layers} layers, vocab 16384) x{args.launches}; algorithmic bytes per "
              f"launch {alg:.0f}")
        return
    if args.profile_kernel == "gemm_rows":   # the tcgen05 batched linear, gate_up shape, 64 rows (or --rows)
        rows = int(args.rows) if args.rows else 64
        w, s = M.synth_linear(0, "prof.gemm", 24576, 4096, "channel", device=dev)
        x = torch.randn(rows, 4096, device=dev).to(torch.bfloat16)
        out = torch.empty(rows, 24576, dtype=torch.bfloat16, device=dev)
        for _ in range(args.launches):
            k.fp8_gemm_rows(x, w, s, out)
        torch.cuda.synchronize()
        print(f"profiled gemm_rows x{args.launches}")
        return
    if args.profile_kernel == "attention_fp8kv":   # 8 sequences at 32k over an FP8 cache (512-key splits)
        batch, max_seq = 8, 32769
        kb = torch.randn(batch, 8, max_seq, 128, device=dev).to(torch.bfloat16)
        k8, ks = M.quantize_kv_rows(kb)
        v8, vs = M.quantize_kv_rows(kb.flip(2))
        del kb
        qkv = torch.randn(batch, 6144, device=dev).to(torch.bfloat16)
        nw = torch.ones(128, dtype=torch.bfloat16, device=dev)
        cos, sin = M.rope_tables(max_seq, 128, 1e6, dev)
        ms = (max_seq + 63) // 64
        o_part = torch.zeros(batch, 32, ms, 128, device=dev)
        ml = torch.zeros(batch, 32, ms, 2, device=dev)
        out = torch.empty(batch, 4096, dtype=torch.bfloat16, device=dev)
        state = torch.tensor([[max_seq - 1, 0]] * batch, dtype=torch.int32, device=dev).view(-1)
        for _ in range(args.launches):
            k.attention_fp8kv(qkv, nw, nw, cos, sin, state, k8.view(torch.uint8), ks, v8.view(torch.uint8), vs, o_part,
                              ml, out, 128 ** -0.5, 1e-6, batch=batch)
        torch.cuda.synchronize()
        print(f"profiled attention_fp8kv x{args.launches}")
        return
    if args.profile_kernel == "prefill_attention":   # the last 128-row chunk of a 2,048-token prompt
        n_kv, max_seq, M_, p0 = 8, 2048, 128, 1920
        kc = torch.randn(n_kv, max_seq, 128, device=dev).to(torch.bfloat16)
        vc = torch.randn(n_kv, max_seq, 128, device=dev).to(torch.bfloat16)
        q = torch.randn(M_, 32, 128, device=dev).to(torch.bfloat16)
        out = torch.empty(M_, 4096, dtype=torch.bfloat16, device=dev)
        for _ in range(args.launches):
            k.prefill_attention(q, p0, kc, vc, 128 ** -0.5, out)
        torch.cuda.synchronize()
        print(f"profiled prefill_attention x{args.launches}")
        return
    if args.profile_kernel == "attention":
        max_seq = 4096
        kc = torch.randn(8, max_seq, 128, device=dev).to(torch.bfloat16)
        vc = torch.randn(8, max_seq, 128, device=dev).to(torch.bfloat16)
        qkv = torch.randn(6144, device=dev).to(torch.bfloat16)
        nw = torch.ones(128, dtype=torch.bfloat16, device=dev)
        cos, sin = M.rope_tables(max_seq, 128, 1e6, dev)
        ms = max_seq // 32
        o_part = torch.zeros(32, ms, 128, device=dev)
        ml = torch.zeros(32, ms, 2, device=dev)
        cnt = torch.zeros(8, dtype=torch.int32, device=dev)
        out = torch.empty(4096, dtype=torch.bfloat16, device=dev)
        state = torch.tensor([max_seq - 1, 0], dtype=torch.int32, device=dev)
        for _ in range(args.launches):
            k.attention(qkv, nw, nw, cos, sin, state, kc, vc, o_part, ml, cnt, out, 128 ** -0.5, 1e-6, 0, args.chunk)
    else:
        kind, N, K = shapes[args.profile_kernel]
        w, s = M.synth_linear(0, "prof", N, K, "channel", device=dev)
        p = M.pack_fp8(w, pairs=(kind == 2))
        x = (torch.randn(K, device=dev) * 0.5).to(torch.bfloat16)
        nw = torch.ones(K, dtype=torch.bfloat16, device=dev)
        if kind == 4:
            logits = torch.empty(N, dtype=torch.bfloat16, device=dev)
            best = torch.zeros(1, dtype=torch.int64, device=dev)
            for _ in range(args.launches):
                k.lm_head_argmax(p, x, nw, logits, best, 1e-6, 0, w_scale=s)
        else:
            out = torch.zeros(N // 2 if kind == 2 else N, dtype=torch.bfloat16, device=dev)
            for _ in range(args.launches):
                k.fp8_gemv(kind, p, s, x, nw if kind in (0, 2) else None, out, N, 1e-6)
    torch.cuda.synchronize()
    print(f"profiled {args.profile_kernel} x{args.launches}")


PHASES = ("qkv", "attn", "o_proj", "gate_up", "down")


def timeline_summary(tl, n_layers: int, clock_ghz: float = 1.965) -> dict:
    """Per-phase breakdown of one fused-step launch from its timeline (int64 [CTAs, 5*layers+1, 32], words as in
    csrc/step.cuh: 0 consumers start the phase, 1 prologue done (attention: arrival counted and, on the CTA
    that completed a KV head, its merge done), 2 the whole CTA done (stamped inside the grid barrier), 3
    producer's first load of the phase, 4-6 cumulative clock64 cycles (consumer warp 0 waiting for ring
    stages, folding units; producer waiting for free slots), 7 consumer warp 0 leaves the stage loop
    (attention: partials done), 8 cumulative cycles warp 0 waited for the slowest warp to release a stage it
    folds, 9-15 warps 1-7 leave the stage loop, 16-18 warp 0's cycles computing slice pairs, taking and
    counting them, and the pairs it took; attention: 9-12 K/V landed, setup, scores, softmax done; merge: 13-15
    entered, KV head counter complete, split weights ready). Times in us: medians over CTAs, then over layers 1..n-1 (layer 0 includes the
    launch ramp). `barrier` is the time from a CTA's end of the phase to its start of the next one; `tail` from
    warp 0 leaving the stage loop to the whole CTA being done; `ring_wait` the consumer's stage waits inside
    the phase; `producer_wait` the producer's waits for free slots while issuing the phase. For every grid
    barrier: how long after the median CTA the last one arrived, and how long after that the first CTA left."""
    import numpy as np
    t = tl.cpu().numpy().astype(np.int64)
    G, P = t.shape[0], t.shape[1]
    us = lambda a: a / 1e3                 # noqa: E731  (globaltimer: ns)
    cyc = lambda a: a / (clock_ghz * 1e3)  # noqa: E731  (clock64 cycles -> us)
    cw = np.diff(np.concatenate([np.zeros((G, 1), np.int64), t[:, :, 4]], axis=1), axis=1)   # per phase
    pw = np.diff(np.concatenate([t[:, :, 6], t[:, -1:, 6]], axis=1), axis=1)                 # phase -> next phase
    names = {0: "qkv", 2: "o_proj", 3: "gate_up", 4: "down"}
    per = {k: [] for k in ("qkv", "attn", "o_proj", "gate_up", "down")}
    layer_us, bar_stats, lags = [], [], {}
    for l in (range(1, n_layers) if n_layers > 1 else range(n_layers)):
        b = 5 * l
        for j, name in names.items():
            ph = t[:, b + j]
            exits = np.concatenate([ph[:, 7:8], ph[:, 9:16]], axis=1)      # loop exit of warps 0..7
            rw = np.diff(np.concatenate([np.zeros((G, 1), np.int64), t[:, :, 8]], axis=1), axis=1)
            per[name].append(dict(prologue=us(ph[:, 1] - ph[:, 0]), stage_loop=us(ph[:, 7] - ph[:, 1]),
                                  tail=us(ph[:, 2] - ph[:, 7]), barrier=us(t[:, b + j + 1, 0] - ph[:, 2]),
                                  ring_wait=cyc(cw[:, b + j]), producer_wait=cyc(pw[:, b + j]),
                                  warp_exit_spread=us(exits.max(1) - exits.min(1)),
                                  last_warp_to_done=us(ph[:, 2] - exits.max(1)),
                                  fold=cyc(np.diff(np.concatenate([np.zeros((G, 1), np.int64), t[:, :, 5]], axis=1),
                                                   axis=1)[:, b + j]),
                                  slowest_warp_wait=cyc(rw[:, b + j]),
                                  warp0_compute=cyc(ph[:, 16]), warp0_take_and_count=cyc(ph[:, 17]),
                                  warp0_pairs=ph[:, 18].astype(np.float64)))
            lags.setdefault(name, []).append(us(exits - exits.min(1, keepdims=True)))
        a = t[:, b + 1]
        merged = us(a[:, 1] - a[:, 7])
        mg = a[:128]   # the merging CTAs
        per["attn"].append(dict(partials=us(a[:, 7] - a[:, 0]), arrive=merged,
                                merge_on_merging_ctas=np.sort(merged)[-4:], tail=us(a[:, 2] - a[:, 1]),
                                barrier=us(t[:, b + 2, 0] - a[:, 2]), producer_wait=cyc(pw[:, b + 1]),
                                kv_landed=us(a[:, 9] - a[:, 0]), setup=us(a[:, 10] - a[:, 9]),
                                scores=us(a[:, 11] - a[:, 10]), softmax=us(a[:, 12] - a[:, 11]),
                                pv_and_store=us(a[:, 7] - a[:, 12]), merge_counter_wait=us(mg[:, 14] - mg[:, 13]),
                                merge_weights=us(mg[:, 15] - mg[:, 14]), merge_sum=us(mg[:, 1] - mg[:, 15]),
                                merge_entry_after_release=us(mg[:, 14] - a[:, 0].min())))
        layer_us.append(np.median(us(t[:, b + 5, 0] - t[:, b, 0])))
        for end_ph in (b, b + 1, b + 2, b + 3, b + 4):
            arrive, leave = t[:, end_ph, 2], t[:, end_ph + 1, 0]
            bar_stats.append((us(arrive.max() - np.median(arrive)), us(leave.min() - arrive.max())))
    out = {"ctas": G, "layers": n_layers, "layer_us": float(np.median(layer_us))}
    bs = np.array(bar_stats).reshape(-1, 5, 2)
    out["barriers"] = {n: {"last_arrival_after_median_us": round(float(np.median(bs[:, i, 0])), 3),
                           "release_after_last_arrival_us": round(float(np.median(bs[:, i, 1])), 3)}
                       for i, n in enumerate(["qkv->attn", "attn->o", "o->gu", "gu->down", "down->qkv"])}
    for k, v in per.items():
        out[k] = {f: round(float(np.median([np.median(d[f]) for d in v])), 3) for f in v[0]}
    # per consumer warp: how long after the CTA's first warp it left the stage loop (median over CTAs, layers)
    out["warp_exit_lag_us"] = {k: [round(float(np.median(np.stack(v)[:, :, w])), 3) for w in range(8)]
                               for k, v in lags.items()}
    h = t[:, 5 * n_layers]
    out["head"] = {"prologue": float(np.median(us(h[:, 1] - h[:, 0]))),
                   "stage_loop": float(np.median(us(h[:, 7] - h[:, 1]))),
                   "tail": float(np.median(us(h[:, 2] - h[:, 7])))}
    out["launch_us"] = float(us(h[:, 2].max() - t[:, 0, 0].min()))
    lead = [np.median(us(t[:, p, 0] - t[:, p, 3])) for p in range(5, 5 * n_layers)]
    out["producer_lead_us"] = float(np.median(lead))
    return out


def run_timeline(args):
    """Fused step with its timeline on: warm-up launches, then one launch whose per-phase stamps are summarised
    (the 36-layer model at the bench's 4k context unless --layers is given)."""
    import model as M
    from generate import Engine
    cfg = M.Config(layers=args.layers if args.layers != 2 else 36)
    max_seq = 4096
    start = max_seq - 64
    m = M.Qwen3FP8Decode.synthetic(cfg, max_seq=max_seq, device="cuda", seed=0, scale_mode="channel", head_dtype="fp8",
                                   norm_init="ones")
    m.fill_cache_random(start, seed=1234)
    eng = Engine(m, fused=True)
    n = len(m.layers)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    eng.step_timeline = torch.zeros(sms, 5 * n + 1, 32, dtype=torch.int64, device="cuda")
    eng.token.fill_(1)
    eng.state.copy_(torch.tensor([start, 0], dtype=torch.int32))
    for _ in range(args.launches):
        eng.decode_step()
    torch.cuda.synchronize()
    eng.check()
    summ = timeline_summary(eng.step_timeline, n)
    summ["ctx"] = start + args.launches - 1
    if args.timeline_out:   # the raw stamps [CTA][phase][word], for per-CTA analysis
        torch.save(eng.step_timeline.cpu(), args.timeline_out)
    print(json.dumps({"timeline": summ}), flush=True)


def run_gemv_sweep(args):
    """Benchmark configuration 3: the FP8 linear of each decode GEMV shape K -> N in {4096->6144, 4096->4096,
    4096->24576, 12288->4096, 4096->151936} for rows in {1, 4, 16, 64}, x ~ N(0,1) bf16, per-channel scales.
    rows 1: the batch-1 GEMV (qk_fp8_gemv, the decode step's kernel; kind 5 = W8A8 dot to fp32); every row
    count also through the tcgen05 batched linear (qk_fp8_gemm_rows: activation quantization + the tensor-core
    GEMM). Per point: time per call (one replay of a CUDA graph of K calls after W eager ones; enough weight
    copies are cycled that the weights come from HBM), algorithmic bytes N*K + scales + rows*K*2 + output, and
    GB/s against the measured HBM peak. One JSON line per point."""
    from kernels import ops
    import model as M
    k = ops()
    peak, _ = peaks()
    K_calls, W = max(args.steps, 8), max(args.warmup, 3)
    shapes = ((4096, 6144), (4096, 4096), (4096, 24576), (12288, 4096), (4096, 151936))
    if args.shapes:
        shapes = [tuple(int(v) for v in sh.split("x")) for sh in args.shapes.split(",")]
    for (Kd, N) in shapes:
        copies = max(1, -(-256 * 2 ** 20 // (N * Kd)))
        ws = [M.synth_linear(c, f"sweep.{N}.{Kd}", N, Kd, "channel", device="cuda") for c in range(copies)]
        packed = [M.pack_fp8(w) for w, _ in ws]
        for rows in ([int(r) for r in args.rows.split(",")] if args.rows else (1, 4, 16, 64)):
            x = torch.randn(rows, Kd, device="cuda").to(torch.bfloat16)
            impls = [("tcgen05", None)] if rows > 1 else [("gemv", None), ("tcgen05", None)]
            for impl, _ in impls:
                if impl == "gemv":
                    out = torch.empty(N, dtype=torch.float32, device="cuda")

                    def call(i):
                        w, s = ws[i % copies]
                        k.fp8_gemv(5, packed[i % copies], s, x[0], None, out, N, 1e-6)
                    out_bytes = N * 4
                else:
                    out = torch.empty(rows, N, dtype=torch.bfloat16, device="cuda")

                    def call(i):
                        w, s = ws[i % copies]
                        k.fp8_gemm_rows(x, w, s, out)
                    out_bytes = rows * N * 2
                for i in range(W):
                    call(i)
                torch.cuda.synchronize()
                graph = torch.cuda.CUDAGraph()
                side = torch.cuda.Stream()
                side.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(side):
                    with torch.cuda.graph(graph, stream=side):
                        for i in range(K_calls):
                            call(i)
                torch.cuda.current_stream().wait_stream(side)
                graph.replay()
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                graph.replay()
                e1.record()
                torch.cuda.synchronize()
                us = e0.elapsed_time(e1) / K_calls * 1e3
                nbytes = N * Kd + N * 4 + rows * Kd * 2 + out_bytes
                gbs = nbytes / (us * 1e-6) / 1e9
                print(json.dumps({"sweep": "gemv", "K": Kd, "N": N, "rows": rows, "impl": impl, "us_per_call": us,
                                  "bytes": nbytes, "gbs": gbs, "frac_of_peak": gbs / peak,
                                  "flops": 2 * rows * N * Kd}), flush=True)
                del graph
        del ws, packed
        torch.cuda.empty_cache()
    assert k.device_error() == 0


def run_attention_sweep(args):
    """Benchmark configuration 4 through the drop-in attention op (the two kernels of qk_attention: partials, merge):
    contexts L in {1k, 4k, 8k, 16k, 32k}, batch 1 (length L) and batch 8 (lengths ~ U[L/2, L], seeded), KV
    N(0,1) bf16, the new token at position len. Per point: time per call (CUDA events around one replay of a
    graph of K calls, after W eager ones; the caches of as many independent layers as keep the working set
    above the 126 MB L2, cycled), the KV bytes
    it must read (K and V of len + 1 keys, 8 heads, plus the appended row), and GB/s against the measured HBM
    peak. One JSON line per point."""
    from kernels import ops
    import model as M
    k = ops()
    peak, _ = peaks()
    K, W = max(args.steps, 8), max(args.warmup, 3)
    out = []
    for L in (1024, 4096, 8192, 16384, 32768):
        for batch in (1, 8):
            if batch == 1:
                lengths = [L]
            else:
                g = torch.Generator().manual_seed(L)
                lengths = [int(x) for x in torch.randint(L // 2, L + 1, (batch,), generator=g)]
            max_seq = L + 1
            fp8 = args.kv == "fp8"
            row_bytes = 128 + 4 if fp8 else 128 * 2       # an FP8 row carries its fp32 scale
            kv_bytes = sum((p + 1) * 8 * row_bytes * 2 for p in lengths)
            per_layer = 2 * batch * 8 * max_seq * row_bytes
            n_layers = max(1, -(-256 * 2 ** 20 // per_layer))           # > 2 x L2 of caches, cycled
            g = torch.Generator(device="cuda").manual_seed(L + batch)
            caches = []
            for _ in range(n_layers):
                kc = torch.randn(batch, 8, max_seq, 128, generator=g, device="cuda").to(torch.bfloat16)
                vc = torch.randn(batch, 8, max_seq, 128, generator=g, device="cuda").to(torch.bfloat16)
                if fp8:
                    (k8, ks), (v8, vs) = M.quantize_kv_rows(kc), M.quantize_kv_rows(vc)
                    caches.append((k8.view(torch.uint8), ks, v8.view(torch.uint8), vs))
                else:
                    caches.append((kc, vc))
            qkv = (torch.randn(batch, 6144, generator=g, device="cuda") * 2).to(torch.bfloat16)
            qn = torch.ones(128, dtype=torch.bfloat16, device="cuda")
            cos, sin = M.rope_tables(max_seq, 128, 1e6, "cuda")
            max_splits = (max_seq + 63) // 64
            o_part = torch.zeros(batch, 32, max_splits, 128, device="cuda")
            ml_part = torch.zeros(batch, 32, max_splits, 2, device="cuda")
            counters = torch.zeros(batch, 8, dtype=torch.int32, device="cuda")
            state = torch.tensor([[p, 0] for p in lengths], dtype=torch.int32, device="cuda").view(-1)
            att = torch.empty(batch, 4096, dtype=torch.bfloat16, device="cuda")

            def call(i):
                if fp8:
                    k8, ks, v8, vs = caches[i % n_layers]
                    k.attention_fp8kv(qkv, qn, qn, cos, sin, state, k8, ks, v8, vs, o_part, ml_part, att,
                                      128 ** -0.5, 1e-6, batch=batch)
                    return
                kc, vc = caches[i % n_layers]
                k.attention(qkv, qn, qn, cos, sin, state, kc, vc, o_part, ml_part, counters, att, 128 ** -0.5,
                            1e-6, 0, 64, batch=batch)

            for i in range(W):
                call(i)
            torch.cuda.synchronize()
            # the timed calls replay from one CUDA graph (as the engine runs them), so host launch cost is out
            graph = torch.cuda.CUDAGraph()
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                with torch.cuda.graph(graph, stream=side):
                    for i in range(K):
                        call(i)
            torch.cuda.current_stream().wait_stream(side)
            graph.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            graph.replay()
            e1.record()
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) / K * 1e3
            del graph
            gbs = kv_bytes / (us * 1e-6) / 1e9
            rec = {"sweep": "attention", "kv": args.kv, "ctx": L, "batch": batch, "lengths": lengths, "us_per_call": us,
                   "kv_bytes": kv_bytes, "gbs": gbs, "frac_of_peak": gbs / peak, "layers_cycled": n_layers}
            print(json.dumps(rec), flush=True)
            out.append(rec)
            del caches
            torch.cuda.empty_cache()
    assert k.device_error() == 0
    return out


def run_prefill(args):
    """Prompt processing on the benchmarked model (36 layers, per-channel FP8 scales, FP8 head): a P-token
    synthetic prompt through Engine.prefill_chunked (the batched forward, 128 positions per pass: the tcgen05
    FP8 linear plus the row-wise prefill kernels) against the same prompt fed position by position through the
    fused decode step (Engine.prefill). Prints one JSON line: prompt tokens/s of each path, the chunked path's
    algorithmic weight stream (every layer's weights once per chunk, the head once) in GB/s and as a fraction
    of the measured HBM peak, and whether both paths pick the same first token. The weights (7.5 GB per pass
    over the layers) are far larger than L2, so no flush is needed between passes."""
    import model as M
    from generate import Engine
    peak, peak_kind = peaks()
    P, chunk = args.prompt, args.prefill_chunk
    K, W = max(1, min(args.steps, 8)), max(args.warmup, 3)
    cfg = M.Config()
    m = M.Qwen3FP8Decode.synthetic(cfg, max_seq=4096, device="cuda", seed=args.seed, scale_mode=args.scale,
                                   head_dtype=args.head, norm_init="ones")
    eng = Engine(m, fused=True)
    ids = torch.randint(0, cfg.vocab, (P,), generator=torch.Generator().manual_seed(7)).tolist()
    eng.prefill_weights()
    for _ in range(W):
        eng.prefill_chunked(ids, chunk)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        torch.cuda.synchronize()
        e0.record()
        for _ in range(K):
            tok_c = eng.prefill_chunked(ids, chunk)
        e1.record()
        torch.cuda.synchronize()
    t_chunked = e0.elapsed_time(e1) * 1e-3 / K
    tok_c = int(tok_c)
    logits_c = eng.logits.float().clone()
    eng.check()

    # the decode-path prefill: one warm call (captures the step graph), then one timed
    eng.prefill(ids)
    torch.cuda.synchronize()
    e0.record()
    tok_d = eng.prefill(ids)
    e1.record()
    torch.cuda.synchronize()
    t_decode = e0.elapsed_time(e1) * 1e-3
    tok_d = int(tok_d)
    logits_d = eng.logits.float()
    eng.check()
    # the two paths compute the same function with different fp32 summation orders (and so, now and then, a
    # different e4m3 rounding): how far apart their last-position logits are, and the decode path's top-2 gap
    top2 = logits_d.topk(2).values
    agreement = {"same_first_token": tok_c == tok_d,
                 "logits_rel_l2": float((logits_c - logits_d).norm() / logits_d.norm()),
                 "logits_max_abs_diff": float((logits_c - logits_d).abs().max()),
                 "decode_top2_gap": float(top2[0] - top2[1])}

    layer_bytes = sum(lin.N * lin.K + lin.scale.numel() * 4 for L in m.layers for lin in (L.qkv, L.o, L.gu, L.down))
    head_bytes = cfg.vocab * cfg.hidden + (cfg.vocab * 4 if args.head == "fp8" else cfg.vocab * cfg.hidden)
    chunks = -(-P // chunk)
    nbytes = chunks * layer_bytes + head_bytes
    gbs = nbytes / t_chunked / 1e9
    rec = {"metric": "prefill_tokens_per_s", "value": P / t_chunked, "unit": "tok/s", "higher_is_better": True,
           "prompt": P, "chunk": chunk, "ms_per_prompt": t_chunked * 1e3, "steps": K, "warmup": W,
           "decode_path": {"value": P / t_decode, "unit": "tok/s", "ms_per_prompt": t_decode * 1e3},
           "speedup_vs_decode_path": t_decode / t_chunked, "paths_agreement": agreement,
           "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                        "algorithmic_bytes": nbytes, "peak_kind": peak_kind},
           "dtype": "fp8 weights, bf16 activations", "data": "synthetic",
           "config": {"workload": f"Qwen3-8B FP8 prompt of {P} tokens (36 layers, {args.scale} scales, "
                                  f"{args.head} head), chunks of {chunk}", "l2": "weights > L2, no flush"},
           "clocks": clk.summary()}
    print(json.dumps(rec), flush=True)
    return rec


def run_batch(args):
    """The batch-16, 32k-context case of the tensor-parallel configuration, on one GPU: the 36-layer model
    (per-channel FP8, FP8 head), `--batch` sequences with their caches pre-filled with N(0,1) rows up to
    `--ctx` (bf16 or, with --kv fp8, the FP8 cache), then K greedy steps of generate.BatchEngine from seeded
    random tokens, CUDA graph replays timed with CUDA events. Prints one JSON line: tokens/s over all sequences,
    and the step's algorithmic bytes (every weight once, each sequence's KV rows up to its position, the
    appended rows) against the measured HBM peak. The KV cache alone is ~78 GB (bf16), far above L2."""
    import model as M
    from generate import BatchEngine
    peak, peak_kind = peaks()
    B, ctx, K, W = args.batch, args.ctx, args.steps, max(args.warmup, 3)
    cfg = M.Config()
    m = M.Qwen3FP8Decode.synthetic(cfg, max_seq=ctx + K + W + 8, device="cuda", seed=args.seed,
                                   scale_mode=args.scale, head_dtype="fp8", norm_init="ones", batch=B)
    if args.kv == "fp8":
        m.set_kv_dtype("fp8")
    m.fill_cache_random(ctx, seed=1234)
    eng = BatchEngine(m)
    g = torch.Generator().manual_seed(args.seed)
    toks = torch.randint(0, cfg.vocab, (B,), generator=g, dtype=torch.int32)
    start = torch.tensor([[ctx, 0]] * B, dtype=torch.int32)
    eng.token.copy_(toks)
    eng.state.copy_(start)
    eng.capture()
    eng.step(W)
    torch.cuda.synchronize()
    eng.token.copy_(toks)
    eng.state.copy_(start)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        torch.cuda.synchronize()
        e0.record()
        eng.step(K)
        e1.record()
        torch.cuda.synchronize()
    t = e0.elapsed_time(e1) * 1e-3
    eng.check()
    wb = m.weight_bytes()
    weights = sum(v for v in wb.values())
    row = (128 + 4) if args.kv == "fp8" else 256
    kv_per_step = sum(B * 2 * cfg.layers * cfg.n_kv_heads * (ctx + i + 1) * row for i in range(K)) / K
    step_bytes = weights + kv_per_step
    gbs = step_bytes / (t / K) / 1e9
    rec = {"metric": "batched decode tokens/s", "value": B * K / t, "unit": "tokens/s", "batch": B, "ctx": ctx,
           "kv": args.kv, "steps": K, "warmup": W, "ms_per_step": t / K * 1e3, "higher_is_better": True,
           "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                        "bytes_per_step": step_bytes, "weight_bytes": weights, "kv_bytes": kv_per_step,
                        "peak_kind": peak_kind},
           "tokens_head": eng.out_tokens[:2, :4].tolist(), "dtype": "fp8 weights, bf16 activations",
           "data": "synthetic", "config": {"workload": f"Qwen3-8B FP8, batch {B}, context {ctx}, {args.kv} KV, "
                                                       "1 GPU (the batch-16 case of the TP configuration)",
                                           "l2": "weights and KV far above L2, no flush"},
           "clocks": clk.summary()}
    print(json.dumps(rec), flush=True)
    return rec


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--profile-kernel", choices=["qkv", "o_proj", "gate_up", "down", "lm_head", "attention", "decode_step",
                                                 "gemm_rows", "attention_fp8kv", "prefill_attention"],
                    help="launch one kernel --launches times on synthetic inputs and exit (for ncu)")
    ap.add_argument("--launches", type=int, default=3)
    ap.add_argument("--layers", type=int, default=2, help="decoder layers of the --profile-kernel decode_step model")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--scale", default="channel", choices=["channel", "block"])
    ap.add_argument("--head", default="fp8", choices=["fp8", "bf16"])
    ap.add_argument("--chunk", type=int, default=64)
    ap.add_argument("--no-pdl", action="store_true")
    ap.add_argument("--path", default="fused", choices=["fused", "ops"],
                    help="fused: one persistent kernel per token; ops: the reference's 183 per-op launches")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-ref-format", action="store_true",
                    help="skip the extra measurement of the fused step in the reference checkpoint's format")
    ap.add_argument("--no-ref-gpu", action="store_true",
                    help="reference arm: skip timing the reference's own decode kernels on the GPU")
    ap.add_argument("--sweep", choices=["attention", "gemv"],
                    help="attention: benchmark configuration 4 (contexts x batches); gemv: configuration 3 (shapes x rows)")
    ap.add_argument("--kv", default="bf16", choices=["bf16", "fp8"],
                    help="--sweep attention: the KV cache format (fp8: e4m3 rows + fp32 row scales)")
    ap.add_argument("--shapes", default="", help="--sweep gemv: comma-separated KxN shapes instead of the five")
    ap.add_argument("--rows", default="", help="--sweep gemv: comma-separated row counts instead of 1,4,16,64")
    ap.add_argument("--timeline-out", default="", help="--timeline: also save the raw stamps (torch.save) here")
    ap.add_argument("--batch", type=int, default=0,
                    help="batched decode (generate.BatchEngine) of this many sequences at --ctx, one GPU")
    ap.add_argument("--ctx", type=int, default=32768, help="--batch: the context the caches are filled to")
    ap.add_argument("--prefill", action="store_true",
                    help="prompt processing: chunked prefill against the decode-path prefill (--prompt tokens)")
    ap.add_argument("--prompt", type=int, default=512, help="--prefill: prompt length")
    ap.add_argument("--prefill-chunk", type=int, default=128, help="--prefill: positions per batched pass (1..128)")
    ap.add_argument("--timeline", action="store_true",
                    help="one fused-step launch with per-phase timeline stamps, summarised (36 layers unless --layers)")
    args = ap.parse_args()
    if args.timeline:
        return run_timeline(args)
    if args.prefill:
        return run_prefill(args)
    if args.batch:
        return run_batch(args)
    if args.sweep == "attention":
        return run_attention_sweep(args)
    if args.sweep == "gemv":
        return run_gemv_sweep(args)
    if args.profile_kernel:
        return run_profile_kernel(args)
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

"""Benchmark: batch-1 greedy decode tokens/s on B200, BASELINE's north-star configuration.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config NAME]
                  [--prompt P] [--layers L] [--replicas] [--repeats R] [--no-extras]

Defaults: N = 1 runs config 2 (`llama3-8b-q8`: Llama-3.1-8B shape, every linear Q8_0, KV cache
prefilled with 4000 positions, decode at max-ctx 4096) — the largest single-GPU configuration and
the one the north star's >= 70 % roofline target is stated on. N > 1 (one process per GPU under
torchrun) runs config 3 (`qwen3-14b`) tensor parallel over the N ranks: ONE sequence split across
the GPUs (strong scaling; value = that sequence's tokens/s); `--replicas` instead runs N independent
copies of the config (weak scaling, no data-path collective).

A step is one decode token (batch 1). Inputs are synthetic: a seeded random-init GGUF with the
config's exact shapes and weight distributions (no checkpoints exist offline); the prompt is
uniform-random token ids, prefilled through fence_prefill (batched on the tensor cores where the
model allows it, else token by token; untimed for the decode value). The timed region is K device-resident
decode steps (one step-kernel launch each, CUDA events on the engine's stream), bracketed by a
barrier and synchronisations; it is repeated R times at the same positions (R chosen so the timed
regions span >= 1.5 s for the clock samples) and the median repeat, max over ranks, is reported.

The line carries, besides the contract keys: `roofline` (the step kernel: algorithmic bytes per
launch = every weight byte once + the embedding row + the K/V rows read, against the measured HBM
copy bandwidth), `e2e` (the same decode through fence_forward + fence_sample_greedy from the host),
`cpu_baseline` (the reference's own scalar Q6_K dequant-dot GEMV, tests/test_gemv_q6k.cu:117-128,
on config 0 on the host cores, 1 thread and all threads), `cpu_port_decode` (the CPU restatement of
the token loop at the same positions), `prefill` (the prompt through fence_prefill: batched
tensor-core GEMMs), and with N = 1 the extra keys `gemv_config0` (the drop-in Q6_K GEMV on config
0), `config1` (Qwen3-4B shape, with the reference's own CUDA forward on this B200 beside it),
`config3_tp1` (config 3 on one GPU: the base of the N > 1 strong-scaling runs) and `config4`
(Mixtral-8x7B shape, sparse MoE, on one GPU).

--impl reference times the reference's algorithm for the path on the host cores: the CPU
restatement of the token loop (oracle/fence_oracle.c; the reference has no CPU forward of its own,
only the per-GEMV host oracle reported in cpu_baseline), all threads, same config and positions,
a bounded number of tokens; only rank 0 runs it. It writes its model file with oracle/libsynth.so
and never loads the product library.
"""
import argparse
import json
import math
import os
import platform
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
from __graft_entry__ import _load_pkg  # noqa: E402

PROMPT_LEN = {"qwen3-4b": 128, "llama3-8b-q8": 4000, "qwen3-14b": 512, "mixtral-8x7b": 256}
MODEL_GB = {"qwen3-4b": 3.5, "llama3-8b-q8": 8.6, "qwen3-14b": 12.5, "mixtral-8x7b": 39.0}  # file sizes
PEAKS_PATH = os.path.join(ROOT, "MEASURED_PEAKS.json")
TRAFFIC_PATH = os.path.join(ROOT, "profiles", "traffic.json")
FALLBACK_HBM_GBS = 6650.0
CONFIG0_BYTES = 4096 * 16 * 210 + 4096 * 2 + 4096 * 4  # W + fp16 x + fp32 y = 13,787,136
MIN_TIMED_S = 1.5


def hbm_peak():
    try:
        v = json.load(open(PEAKS_PATH))["hbm_gbs"]
        return float(v), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def traffic_record(name):
    """A machine-readable ncu figure (profiles/traffic.json) for a kernel / workload, or None."""
    try:
        return json.load(open(TRAFFIC_PATH)).get(name)
    except (OSError, ValueError):
        return None


def step_algorithmic_bytes(cfg, positions):
    """Bytes one decode token must move (the roofline numerator): every weight streamed once
    (layer linears + the tied LM head, weight_bytes), the token's embedding row, and the K and V
    rows of the context read by attention (fp16), averaged over the timed positions."""
    kv_dim = cfg.n_kv_heads * cfg.head_dim // max(1, cfg.tp_size)
    embed_row = cfg.embed_dim // 32 * 34
    kv = sum(2 * cfg.n_layers * (p + 1) * kv_dim * 2 for p in positions) / max(1, len(positions))
    return int(cfg.weight_bytes + embed_row + kv)


class ClockSampler:
    """nvidia-smi clock/throttle samples every 200 ms while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.25)
        return self

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            out, _ = self.proc.communicate(timeout=10)
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in self.lines:
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons), "samples": len(sm)}


def cpu_model_name():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return platform.processor() or "unknown"


def synth_model(fb, config, tmp, layers=0):
    path = os.path.join(tmp, f"{config}.gguf")
    if layers > 0:
        fb.synth_write(path, config, seed=2024, n_layers=layers)
    else:
        fb.synth_write(path, config, seed=2024)
    return path


def shm_dir(need_bytes):
    try:
        st = os.statvfs("/dev/shm")
        return "/dev/shm" if st.f_bavail * st.f_frsize > need_bytes else None
    except OSError:
        return None


# ------------------------------------------------------------------ GPU decode measurement
def measure_decode(fb, torch, model, prompt_len, steps, warmup, repeats, dist=None, tp=False, seed=7,
                   e2e_steps=None, clocks_index=None):
    """Prefill through fence_prefill (untimed for the decode value; its own rate is reported), W
    warm-up steps, then R timed regions of K device-resident decode steps at the same positions;
    e2e through fence_forward +
    fence_sample_greedy from the host. Returns a dict (times max over ranks)."""
    cfg = model.config
    rng = np.random.default_rng(seed)
    prompt = [int(t) for t in rng.integers(0, cfg.vocab_size, prompt_len)]
    # prefill through the public API (batched tensor-core GEMMs where the model allows it; untimed
    # for the decode value, its own rate reported as `prefill`)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    d = model.prefill(prompt)
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t0
    first = model.sample_greedy(d)
    pos = prompt_len
    warm_ids = model.decode_greedy(first, pos, warmup)
    pos += warmup
    tok = warm_ids[-1]
    torch.cuda.synchronize()
    # repeats: enough timed regions to span MIN_TIMED_S (the same count on every rank)
    if repeats <= 0:
        probe = model.time_decode(tok, pos, steps)
        repeats = int(min(60, max(3, math.ceil(MIN_TIMED_S * 1e3 / max(probe, 1e-3)))))
    if dist:
        t = torch.tensor([repeats], device="cuda", dtype=torch.int64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        repeats = int(t.item())
    times = []
    clk = ClockSampler(clocks_index) if clocks_index is not None else None
    if clk:
        clk.__enter__()
    try:
        for _ in range(repeats):
            if dist:
                dist.barrier()
            torch.cuda.synchronize()
            ms = model.time_decode(tok, pos, steps)  # CUDA events; raises on a device wait error
            torch.cuda.synchronize()
            times.append(ms)
    finally:
        if clk:
            clk.__exit__()
    if dist:
        t = torch.tensor(times, device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        times = [float(x) for x in t.tolist()]
        dist.barrier()
    ms = statistics.median(times)
    positions = range(pos, pos + steps)
    pos += steps
    # e2e through the reference-facing API: forward(token, pos) from the host (16-byte state H2D from
    # pinned memory, 16-byte state D2H) + sample_greedy every step
    e2e_steps = e2e_steps or min(steps, 64)
    nxt = tok
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        dl = model.forward(nxt, pos + i)
        nxt = model.sample_greedy(dl)
    e2e_s = time.perf_counter() - t0
    if dist:
        t = torch.tensor([e2e_s], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    return {"ms": ms, "times": times, "repeats": repeats, "positions": positions, "e2e_tok_s": e2e_steps / e2e_s,
            "prefill_tok_s": prompt_len / prefill_s, "prefill_s": prefill_s,
            "e2e_steps": e2e_steps, "step_bytes": step_algorithmic_bytes(cfg, positions),
            "clocks": clk.summary() if clk else None}


def measure_gemv_roofline(fb, torch, copies=32, launches=256, pdl=True):
    """Config-0 Q6_K GEMV (4096x4096) through the drop-in C-ABI, rotating over `copies` weight
    copies (> L2) so every launch streams from HBM: one launch per copy captured in a CUDA graph,
    the graph replayed back to back; CUDA events on the replay stream. With pdl=True the launches
    use FENCE_LAUNCH_PDL (weights are never written), so each GEMV starts streaming while the
    previous one drains, as inside the decode step."""
    fb.lib().fence_set_launch_flags(fb.FENCE_LAUNCH_PDL if pdl else 0)
    M = K = 4096
    nblk = M * K // 256
    W = np.frombuffer(fb.synth_blocks(fb.GGML_Q6_K, nblk, seed=0), np.uint8)
    dW = torch.empty((copies, W.size), dtype=torch.uint8, device="cuda")
    dW[:] = torch.from_numpy(W.copy()).cuda()
    x = np.random.default_rng(0).standard_normal(K).astype(np.float32).astype(np.float16).view(np.int16)
    dx = torch.from_numpy(x.copy()).cuda()
    dy = torch.empty(M, dtype=torch.float32, device="cuda")
    L = fb.lib()
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        for i in range(copies):  # warm-up (and the kernel's shared-memory attribute) outside capture
            fb.check(L.fence_gemv_q6k(dW[i].data_ptr(), dx.data_ptr(), dy.data_ptr(), M, K, st.cuda_stream))
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        for i in range(copies):
            fb.check(L.fence_gemv_q6k(dW[i].data_ptr(), dx.data_ptr(), dy.data_ptr(), M, K,
                                      torch.cuda.current_stream().cuda_stream))
    reps = max(1, launches // copies)
    with torch.cuda.stream(st):
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(reps):
            g.replay()
        e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / (reps * copies)
    fb.lib().fence_set_launch_flags(0)
    del g, dW
    return ms


# ------------------------------------------------------------------ CPU legs (checker libraries)
def cpu_reference_gemv():
    """The reference's own scalar Q6_K dequant-dot GEMV (cpu_gemv_q6k, tests/test_gemv_q6k.cu:117-128,
    compiled unmodified into oracle/_ref/libref_cpu.so) on config 0 (4096 x 4096, seeded blocks,
    x N(0,1) rounded to fp16): 1 thread as shipped, and all host threads as a row split of the
    unchanged per-row loop (one call per row range, threads released from the GIL by ctypes).
    Median of 5 runs each, in GB/s of CONFIG0_BYTES. None when the library was not built."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc  # CPU-baseline leg only
    ref = orc.ref_cpu()
    if ref is None:
        return None
    M = K = 4096
    rng = np.random.default_rng(0)
    # seeded Q6_K blocks with the config-0 distribution, generated here (no product library): ql/qh
    # uniform bytes, int8 scales uniform in [-127, 127], d = fp16(1.5e-5)
    blk = np.empty((M * K // 256, 210), np.uint8)
    blk[:, :192] = rng.integers(0, 256, (blk.shape[0], 192), dtype=np.uint8)
    blk[:, 192:208] = rng.integers(-127, 128, (blk.shape[0], 16)).astype(np.int8).view(np.uint8)
    blk[:, 208:210] = np.frombuffer(np.float16(1.5e-5).tobytes(), np.uint8)
    W = np.ascontiguousarray(blk)
    x = rng.standard_normal(K).astype(np.float32).astype(np.float16).view(np.uint16).copy()
    y = np.empty(M, np.float64)
    row_bytes = K // 256 * 210

    def run(threads):
        if threads == 1:
            t0 = time.perf_counter()
            ref.ref_cpu_gemv_q6k(W.ctypes.data, x.ctypes.data, y.ctypes.data, M, K)
            return time.perf_counter() - t0
        bounds = [M * i // threads for i in range(threads + 1)]

        def part(i):
            r0, r1 = bounds[i], bounds[i + 1]
            ref.ref_cpu_gemv_q6k(W.ctypes.data + r0 * row_bytes, x.ctypes.data, y.ctypes.data + 8 * r0, r1 - r0, K)
        ths = [threading.Thread(target=part, args=(i,)) for i in range(threads)]
        t0 = time.perf_counter()
        for t in ths:
            t.start()
        for t in ths:
            t.join()
        return time.perf_counter() - t0

    threads = os.cpu_count() or 1
    run(1)  # warm-up
    t1 = statistics.median(run(1) for _ in range(5))
    run(threads)
    tn = statistics.median(run(threads) for _ in range(5))
    return {"gbs_1_thread": CONFIG0_BYTES / t1 / 1e9, "gbs_all_threads": CONFIG0_BYTES / tn / 1e9,
            "s_1_thread": t1, "s_all_threads": tn, "threads": threads, "cpu": cpu_model_name()}


def cpu_port_decode(path, start_pos, budget_s, max_tokens, threads, seed=7):
    """The CPU restatement of the token loop (oracle/fence_oracle.c, fp64 accumulation) decoding
    at positions start_pos.. of a cache pre-filled with seeded K/V rows (the prefill's stand-in),
    one warm-up token, then tokens until the budget is spent (at least one). Returns (n, seconds)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc  # CPU legs only
    m = orc.OracleModel(path, max_ctx=max(4096, start_pos + max_tokens + 2), kv_bf16=False, threads=threads)
    m.fill_kv(start_pos, seed)
    rng = np.random.default_rng(seed)
    V = m.vocab_size
    m.forward(int(rng.integers(0, V)), start_pos)  # warm-up (page cache)
    n, t0 = 0, time.perf_counter()
    while n < max_tokens:
        m.forward(int(rng.integers(0, V)), start_pos + 1 + n)
        n += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    m.close()
    return n, dt


def run_reference_arm(args, rank, world):
    """--impl reference: the reference's algorithm for the path on the host cores (rank 0 only)."""
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import importlib.util
    import oracle as orc  # reference arm only
    # the binding module for its config table and struct layout only: the product library is not loaded
    spec = importlib.util.spec_from_file_location(
        "fence_b200_cfg", os.path.join(ROOT, "-damn-low-level-fence-inference-version-1_b200", "__init__.py"))
    cfgmod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(cfgmod)
    threads = os.cpu_count() or 1
    start = args.prompt + args.warmup
    with tempfile.TemporaryDirectory(dir=args.tmp) as tmp:
        path = os.path.join(tmp, f"{args.config}.gguf")
        fields = dict(cfgmod.CONFIGS[args.config])
        fields["seed"] = 2024
        orc.synth_write(path, cfgmod.SynthSpec, fields, threads)
        budget = min(120.0, 3.0 * max(args.steps, 1))
        n, dt = cpu_port_decode(path, start, budget, args.steps, threads)
    value = n / dt
    sample = (f"{n} of {args.steps} decode tokens of {args.config} at positions {start + 1}..{start + n} "
              f"(K/V of positions 0..{start} pre-filled with seeded rows in place of the {args.prompt}-token prefill), "
              f"oracle/fence_oracle.c on {threads} threads, bounded to {budget:.0f} s")
    line = {
        "impl": "reference", "metric": "decode_tokens_per_s", "value": round(value, 4), "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": n, "warmup": 1, "ms_per_step": round(1e3 * dt / n, 3),
        "higher_is_better": True, "scaling": "strong" if args.tp else "weak", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic (seeded random-init GGUF, config shapes)",
        "config": {"workload": f"{args.config} batch-1 greedy decode (CPU restatement of the reference's token loop)",
                   "model": args.config, "prefill_positions": start},
        "cpu_baseline": {"value": round(value, 4), "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ extras (N = 1, rank 0)
def extra_config1(fb, torch, args, kv):
    """Config 1 (Qwen3-4B shape, Q6_K): this engine's decode and, beside it, the reference's own
    CUDA forward (src/model/qwen3.cu rebuilt unmodified for sm_100a, oracle/_ref/ref_model) on the
    same model file, prompt length and B200."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc  # reference-on-B200 comparator only
    out = {}
    with tempfile.TemporaryDirectory(dir=args.tmp) as tmp:
        path = synth_model(fb, "qwen3-4b", tmp)
        m = fb.Model(path, max_ctx=4096, kv_dtype=kv)
        r = measure_decode(fb, torch, m, 128, 128, 4, 0)
        cfg = m.config
        m.close()
        peak, _ = hbm_peak()
        gbs = r["step_bytes"] / (r["ms"] / 128 * 1e-3) / 1e9
        out = {"workload": "qwen3-4b batch-1 greedy decode, 128 prompt tokens, 128 timed steps",
               "tok_s": round(128 / (r["ms"] / 1e3), 2), "e2e_tok_s": round(r["e2e_tok_s"], 2),
               "roofline_frac": round(gbs / peak, 4), "achieved_gbs": round(gbs, 1)}
        if os.path.exists(orc.REF_MODEL):
            prompt = ",".join(str(int(t)) for t in np.random.default_rng(7).integers(0, cfg.vocab_size, 128))
            try:
                p = subprocess.run([orc.REF_MODEL, path, os.path.join(tmp, "ref.bin"), "--tokens", prompt,
                                    "--steps", "65", "--no-logits"], capture_output=True, text=True, timeout=600)
                rec = json.loads(p.stdout.strip().splitlines()[-1])
                out["reference_b200_tok_s"] = round(rec["ref_decode_tok_s"], 2)
                out["reference_b200_prefill_tok_s"] = round(rec["ref_prefill_tok_s"], 2)
                out["reference_b200"] = ("the reference's unmodified CUDA forward (src/model/qwen3.cu, -O3 "
                                         "--use_fast_math, sm_100a) via oracle/_ref/ref_model: 128-token prefill, "
                                         "64 greedy steps, host-timed forward + sample_greedy")
            except Exception as e:  # the comparator is optional
                out["reference_b200_error"] = str(e)[:200]
    return out


def extra_config3_tp1(fb, torch, args, kv):
    """Config 3 (Qwen3-14B shape) on one GPU: the single-GPU base of the tensor-parallel runs."""
    with tempfile.TemporaryDirectory(dir=args.tmp) as tmp:
        path = synth_model(fb, "qwen3-14b", tmp)
        m = fb.Model(path, max_ctx=4096, kv_dtype=kv)
        r = measure_decode(fb, torch, m, 512, 64, 4, 0)
        m.close()
    peak, _ = hbm_peak()
    gbs = r["step_bytes"] / (r["ms"] / 64 * 1e-3) / 1e9
    return {"workload": "qwen3-14b batch-1 greedy decode on 1 GPU, 512 prompt tokens, 64 timed steps",
            "tok_s": round(64 / (r["ms"] / 1e3), 2), "roofline_frac": round(gbs / peak, 4)}


def extra_config4(fb, torch, args, kv):
    """Config 4 (Mixtral-8x7B shape, sparse MoE top-2 of 8 experts) on one GPU: decode through the
    step kernel with routing on the device; the roofline counts the routed experts' bytes only."""
    gb = MODEL_GB["mixtral-8x7b"] * 1e9
    tmp_dir = shm_dir(gb + 20e9) or args.tmp
    with tempfile.TemporaryDirectory(dir=tmp_dir) as tmp:
        path = synth_model(fb, "mixtral-8x7b", tmp)
        m = fb.Model(path, max_ctx=4096, kv_dtype=kv)
        r = measure_decode(fb, torch, m, PROMPT_LEN["mixtral-8x7b"], 64, 4, 0)
        m.close()
    peak, _ = hbm_peak()
    gbs = r["step_bytes"] / (r["ms"] / 64 * 1e-3) / 1e9
    return {"workload": "mixtral-8x7b batch-1 greedy decode on 1 GPU (top-2 of 8 experts), 256 prompt tokens, "
                        "64 timed steps", "tok_s": round(64 / (r["ms"] / 1e3), 2), "roofline_frac": round(gbs / peak, 4),
            "active_bytes_per_token": r["step_bytes"]}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default=None, help="default: llama3-8b-q8 at one rank, qwen3-14b (TP) at N > 1")
    ap.add_argument("--prompt", type=int, default=None, help="prefill tokens (default: the config's own)")
    ap.add_argument("--layers", type=int, default=0, help="cut the model to this many layers (ncu captures)")
    ap.add_argument("--ep", action="store_true",
                    help="sparse MoE (mixtral-8x7b) with N > 1: whole experts per rank instead of a slice of each")
    ap.add_argument("--replicas", action="store_true",
                    help="with N > 1: N independent replicas (weak scaling) instead of one tensor-parallel model")
    ap.add_argument("--repeats", type=int, default=0, help="timed regions (0: enough for >= 1.5 s)")
    ap.add_argument("--kv", default="f16", choices=["f16", "bf16"])
    ap.add_argument("--tmp", default=None, help="directory for the synthetic GGUF (default: /dev/shm if roomy)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="skip the extra keys (config 0 / 1 / 3-TP1)")
    ap.add_argument("--mode", default="decode", choices=["decode", "gemv", "prefill"],
                    help="gemv: only the config-0 Q6_K GEMV roofline measurement (small; used for ncu captures); "
                         "prefill: only the batched prefill of --prompt tokens of --config")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    args.tp = world > 1 and not args.replicas
    if args.config is None:
        args.config = "qwen3-14b" if args.tp else "llama3-8b-q8"
    if args.prompt is None:
        args.prompt = PROMPT_LEN.get(args.config, 128)
    if args.tmp is None:
        gb = MODEL_GB.get(args.config, 20.0) * 1e9
        args.tmp = shm_dir(gb * (1 if args.tp else world) + 20e9)

    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return

    import torch
    torch.cuda.set_device(local)
    if args.mode == "gemv":
        fb = _load_pkg()
        peak, peak_kind = hbm_peak()
        ms = measure_gemv_roofline(fb, torch, copies=16, launches=max(args.steps, 1), pdl=False)
        ms_pdl = measure_gemv_roofline(fb, torch, copies=16, launches=max(args.steps, 1), pdl=True)
        print(json.dumps({"metric": "gemv_q6k_config0_GBps", "value": round(CONFIG0_BYTES / (ms * 1e-3) / 1e9, 1),
                          "unit": "GB/s", "us_per_launch": round(ms * 1e3, 3), "kernel": "gemv_q6k_reg_kernel",
                          "us_per_launch_pdl": round(ms_pdl * 1e3, 3), "kernel_pdl": "gemv_stream_kernel",
                          "peak": peak, "peak_kind": peak_kind}))
        return
    if args.mode == "prefill":
        fb = _load_pkg()
        with tempfile.TemporaryDirectory(dir=args.tmp) as tmp:
            path = synth_model(fb, args.config, tmp, args.layers)
            m = fb.Model(path, max_ctx=max(4096, args.prompt + 8))
            c = m.config
            rng = np.random.default_rng(7)
            m.prefill([int(t) for t in rng.integers(0, c.vocab_size, 64)])  # scratch allocation, warm-up
            toks = [int(t) for t in rng.integers(0, c.vocab_size, args.prompt)]
            times = []
            for _ in range(max(1, args.steps)):
                torch.cuda.synchronize()
                t0 = time.perf_counter()
                m.prefill(toks)
                torch.cuda.synchronize()
                times.append(time.perf_counter() - t0)
            m.close()
        qd, kvd = c.n_heads * c.head_dim, c.n_kv_heads * c.head_dim
        params = c.n_layers * (c.embed_dim * (qd + 2 * kvd) + qd * c.embed_dim + 3 * c.embed_dim * c.ff_dim)
        s_med = statistics.median(times)
        print(json.dumps({"metric": "prefill_tokens_per_s", "value": round(args.prompt / s_med, 1), "unit": "tokens/s",
                          "config": args.config, "layers": c.n_layers, "tokens": args.prompt, "s": round(s_med, 4),
                          "linear_tflop": round(2 * params * (args.prompt - 1) / 1e12, 2),
                          "linear_tflops_if_all_time": round(2 * params * (args.prompt - 1) / s_med / 1e12, 1)}))
        return
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))

    fb = _load_pkg()
    kv = fb.FENCE_KV_F16 if args.kv == "f16" else fb.FENCE_KV_BF16
    tp = args.tp
    max_ctx = max(4096, args.prompt + args.warmup + args.steps + 64 + 8)
    with tempfile.TemporaryDirectory(dir=args.tmp) as tmp:
        if tp:
            # one model file for all ranks: rank 0 writes it, the others read it (same host)
            gloo = dist.new_group(backend="gloo")
            box = [tmp]
            dist.broadcast_object_list(box, src=0, group=gloo)
            path = os.path.join(box[0], f"{args.config}.gguf")
            if rank == 0:
                synth_model(fb, args.config, box[0], args.layers)
            dist.barrier(group=gloo)
            model = fb.Model(path, max_ctx=max_ctx, kv_dtype=kv, device=local, tp_rank=rank, tp_size=world,
                             moe_ep=args.ep)
            import fence_b200.tp as fbtp
            fbtp.connect(model, gloo)
            dist.barrier(group=gloo)  # every rank has read the file before rank 0 removes it
        else:
            # every rank writes its own copy (same seed -> identical bytes); ranks stay independent
            path = synth_model(fb, args.config, tmp, args.layers)
            model = fb.Model(path, max_ctx=max_ctx, kv_dtype=kv, device=local)
        cfg = model.config
        r = measure_decode(fb, torch, model, args.prompt, args.steps, args.warmup, args.repeats, dist=dist, tp=tp,
                           seed=7 if tp else 7 + rank, clocks_index=local)
        model.close()
        derr = fb.lib().fence_device_error()
        if derr != 0:
            print(json.dumps({"error": f"device error word {derr} after the timed regions"}), flush=True)
            sys.exit(1)
        ms = r["ms"]
        tok_s = args.steps / (ms / 1e3)
        value = tok_s if tp else tok_s * world  # one sequence over all ranks / one per replica
        e2e_val = r["e2e_tok_s"] * (1 if tp else world)
        # CPU legs on the same model file, rank 0 of a single-rank run only
        cpu_port = None
        if rank == 0 and world == 1 and not args.no_cpu_baseline and not args.layers:
            threads = os.cpu_count() or 1
            start = args.prompt + args.warmup
            n, dt = cpu_port_decode(path, start, 15.0, 32, threads)
            cpu_port = {"value": round(n / dt, 4), "unit": "tokens/s", "cores": threads, "kind": "port",
                        "sample": f"{n} decode tokens of {args.config} at positions {start + 1}..{start + n} "
                                  f"(K/V of positions 0..{start} pre-filled with seeded rows), "
                                  f"oracle/fence_oracle.c (fp64) on {threads} threads, ~15 s"}

    peak, peak_kind = hbm_peak()
    step_bytes = r["step_bytes"]
    step_us = ms / args.steps * 1e3
    step_gbs = step_bytes / (step_us * 1e-6) / 1e9
    trec = traffic_record(f"step_kernel_{args.config.replace('-', '_')}")
    step_traffic = int(trec["ratio"] * step_bytes) if trec and "ratio" in trec else None
    line = {
        "metric": "decode_tokens_per_s", "value": round(value, 3), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5),
        "higher_is_better": True, "scaling": "strong" if tp else "weak", "vs_baseline": None, "dtype": "int8xint16",
        "data": "synthetic (seeded random-init GGUF, config shapes)",
        "config": {"workload": f"{args.config} batch-1 greedy decode, {args.prompt} prompt tokens, positions "
                               f"{r['positions'][0]}..{r['positions'][-1]}"
                               + (f" ({args.layers}-layer cut for profiling, not the config)" if args.layers else ""),
                   "model": args.config, "kv_cache": args.kv, "global_batch": 1 if tp else world,
                   "seq_len": r["positions"][-1] + 1,
                   "parallelism": (f"ep{world}" if args.ep else f"tp{world}") if tp
                   else (f"replicas{world}" if world > 1 else "single"),
                   "repeats": r["repeats"], "timing": "median of the repeats of K steps, max over ranks",
                   "l2": "weights larger than L2 (no flush needed)"},
        "roofline": {"bound": "hbm", "kernel": "step_kernel (one launch = one whole token step)",
                     "achieved": round(step_gbs, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(step_gbs / peak, 4), "peak_kind": peak_kind,
                     "traffic": step_traffic, "us_per_launch": round(step_us, 2),
                     "algorithmic_bytes_per_launch": step_bytes,
                     "traffic_source": (trec or {}).get("summary")},
        "e2e": {"value": round(e2e_val, 3), "unit": "tokens/s", "h2d_bytes_per_step": 16, "d2h_bytes_per_step": 16,
                "steps": r["e2e_steps"]},
        "prefill": {"tok_s": round(r["prefill_tok_s"], 1), "tokens": args.prompt, "s": round(r["prefill_s"], 4),
                    "path": ("batched tcgen05 GEMMs (fence_prefill)" if not tp and not getattr(cfg, "n_experts", 0)
                             else "token by token through the decode step (fence_prefill)"),
                    "timing": "host wall clock around fence_prefill incl. the last token's decode step"},
        "gpu_launches": args.steps,
        "gpu_launches_note": "one step-kernel launch per decode step; the K-step region is repeated `repeats` times",
        "clocks": r["clocks"],
        "cpu_baseline": None,
        "cpu_port_decode": cpu_port,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        g = cpu_reference_gemv()
        if g:
            line["cpu_baseline"] = {
                "value": round(g["gbs_all_threads"] * 1e9 / step_bytes, 5), "unit": "tokens/s", "cores": g["threads"],
                "kind": "reference",
                "sample": (f"the reference's scalar Q6_K dequant-dot GEMV cpu_gemv_q6k (tests/test_gemv_q6k.cu:117-128, "
                           f"oracle/_ref/libref_cpu.so) on config 0, median of 5: {g['gbs_all_threads']:.3f} GB/s on "
                           f"{g['threads']} threads (row split), {g['gbs_1_thread']:.3f} GB/s on 1 thread; value = that "
                           f"weight-streaming rate over this config's {step_bytes / 1e9:.3f} GB per token"),
                "gbs_all_threads": round(g["gbs_all_threads"], 4), "gbs_1_thread": round(g["gbs_1_thread"], 4),
                "cpu": g["cpu"]}
    if rank == 0 and world == 1 and not args.no_extras and not args.layers:
        # the drop-in's default launch (stream-ordered, as the reference's) is the headline; the
        # opt-in programmatic-dependent-launch chain beside it
        gemv_ms = measure_gemv_roofline(fb, torch, pdl=False)
        gemv_ms_pdl = measure_gemv_roofline(fb, torch, pdl=True)
        achieved = CONFIG0_BYTES / (gemv_ms * 1e-3) / 1e9
        grec = traffic_record("gemv_q6k_config0") or {}
        line["gemv_config0"] = {
            "kernel": "drop-in gemv_q6k 4096x4096 (config 0), back-to-back launches in a CUDA graph: "
                      "gemv_q6k_reg_kernel (stream-ordered launch); gemv_stream_kernel under PDL",
            "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
            "traffic": grec.get("bytes_per_launch"), "us_per_launch": round(gemv_ms * 1e3, 3),
            "us_per_launch_pdl": round(gemv_ms_pdl * 1e3, 3), "algorithmic_bytes_per_launch": CONFIG0_BYTES}
        line["config1"] = extra_config1(fb, torch, args, kv)
        line["config3_tp1"] = extra_config3_tp1(fb, torch, args, kv)
        line["config4"] = extra_config4(fb, torch, args, kv)
        derr = fb.lib().fence_device_error()
        if derr != 0:
            print(json.dumps({"error": f"device error word {derr} after the extra measurements"}), flush=True)
            sys.exit(1)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

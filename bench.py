"""Decode throughput of the B200 token loop on the TinyLlama-1.1B Q4_K workload.

Workload (one replica per GPU): the TinyLlama-1.1B architecture (22 layers,
hidden 2048, FFN 5632, 32 query / 4 KV heads, vocab 32000) with seeded
synthetic Q4_K weights, batch 1, a 128-token uniform-random prompt, greedy
decoding. A step is one decode token (forward of one token over the 22 layers +
LM head + on-device argmax). The weights (582 MB) exceed the 126 MB L2, so no
L2 flush is needed between steps.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  torchrun --nproc-per-node N bench.py --gpus N --tp [--layers L] [--prompt P]
      (the Llama-2-70B shape, tensor-parallel over N GPUs; not the headline line)
  [torchrun ...] bench.py --serve [--sequences S] [--prompt P] [--sampled]
      (batched serving: S sequences of a P-token prompt + --steps decode tokens,
      split evenly over the ranks, fp16 KV; not the headline line)
  python bench.py --microbench REPS
      (Q4_K GEMV/GEMM through wcb_gemv_dev at 5 weight shapes x M = 1, 16, 512;
      one JSON line each; not the headline line)

N > 1 runs under torchrun as N independent data-parallel replicas (no
collective on the data path); value is the total tokens/s over all ranks with
the time taken as the max over ranks.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "wasm-chord_b200")
for _p in (REPO, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402

MODEL_DIR = os.environ.get("WCB_MODEL_DIR", "/tmp/wcb_models")
PROMPT_LEN = 128
METRIC = "decode tok/s (TinyLlama-1.1B Q4_K, batch 1)"
# --model llama7b: the Llama-2-7B shape with the Q4_K_M mix, 512-token prompt (not the headline)
MODELS = {"tinyllama": ("TinyLlama-1.1B Q4_K", "tinyllama-1.1b-arch", 128),
          "llama7b": ("Llama-2-7B Q4_K_M", "llama-2-7b-arch", 512)}

# DRAM bytes (read + write) of one decode_step_kernel launch from an ncu capture
# (dram__bytes_read.sum + dram__bytes_write.sum of the 5th decode step of
# `bench.py --steps 16 --warmup 3 --no-cpu-baseline`) and the KV position of the captured step; the f32 KV rows read grow with the
# position, so the figure is moved to the bench's mean position by the KV bytes
# in between.
NCU_STEP_TRAFFIC = {"tinyllama-1.1b-arch": (588723712 + 3977472, 133)}


def peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def weight_bytes(cfg, path):
    """Bytes of the 2-D weights one decode token streams (Q4_K 144/256, Q6_K 210/256 B per value)."""
    from gguf import GGUFReader
    total = 0
    for t in GGUFReader(path).tensors:
        if t.name.endswith("norm.weight") or t.name == "token_embd.weight":
            continue
        total += int(t.n_bytes)
    return total


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.proc = None
        self.path = tempfile.mktemp(prefix="wcb_clocks_", suffix=".csv")

    def __enter__(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", str(self.device), "-lms", "200"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self):
        if self.proc is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def model_file(preset="tinyllama"):
    """Path of the synthetic GGUF for ``preset``, written first if missing. The
    generator runs in a child process, so the timing process never loads the
    generator's native library (the reference arm loads nothing of this package)."""
    path = os.path.join(MODEL_DIR, f"wcb_{preset}.gguf")
    if not os.path.exists(path):
        code = ("import sys; sys.path.insert(0, %r); from wcb import synth; "
                "synth.cached_model(%r, %r)" % (PKG, preset, MODEL_DIR))
        subprocess.run([sys.executable, "-c", code], check=True)
    return path


def ensure_model(rank, world, dist, preset="tinyllama"):
    path = os.path.join(MODEL_DIR, f"wcb_{preset}.gguf")
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if local == 0:
        model_file(preset)
    if world > 1:
        dist.barrier()
    return path


def time_gemv(torch, wcb, stream_ptr, n, k, m, reps_per_copy=8, seed=99):
    """Times wcb_gemv_dev (y[m][n] = x[m][k] W[n][k]^T, W Q4_K) on the stream it is
    launched on, rotating over enough weight copies that each launch reads its
    weights from HBM, not from the 126 MB L2. Returns (bytes, flops, us per launch)."""
    from wcb import synth
    blocks = synth.quantize_q4_k_fast(synth.normal(seed, 1, n * k, 0.0, 0.02))
    nbytes = blocks.nbytes
    copies = max(4, int(2 * 126e6 // nbytes) + 1)
    dev = torch.from_numpy(blocks.reshape(-1)).cuda()
    ws = [dev.clone() for _ in range(copies)]
    del dev
    x = torch.from_numpy(synth.normal(seed - 1, 1, m * k, 0.0, 1.0)).cuda()
    y = torch.empty(m * n, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()  # the copies above ran on torch's stream, the launches below on stream_ptr
    s = torch.cuda.ExternalStream(stream_ptr)
    reps = reps_per_copy * copies
    with torch.cuda.stream(s):
        for i in range(min(2, reps_per_copy) * copies):
            wcb.gemv_dev(ws[i % copies].data_ptr(), wcb.DTYPE_Q4_K, n, k, x.data_ptr(), m, y.data_ptr(), stream_ptr)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for i in range(reps):
            wcb.gemv_dev(ws[i % copies].data_ptr(), wcb.DTYPE_Q4_K, n, k, x.data_ptr(), m, y.data_ptr(), stream_ptr)
        e1.record(s)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) / reps * 1e3
    return nbytes + 4 * m * k + 4 * m * n, 2 * m * n * k, us, copies


def gemv_roofline(torch, wcb, stream_ptr, cfg, peak, reps_per_copy=8):
    """Times the dominant kernel of the decode step — the fused Q4_K dequant-GEMV
    at the FFN gate+up shape [2*F, H], M = 1 — on the stream it is launched on."""
    n, k = 2 * cfg.intermediate_size, cfg.hidden_size
    algo, _, us, copies = time_gemv(torch, wcb, stream_ptr, n, k, 1, reps_per_copy)
    gbs = algo / (us * 1e-6) / 1e9
    return {"kernel": "gemv_kernel<1,PRO_NONE,EPI_STORE> (Q4_K)", "shape_nk": [n, k], "m": 1,
            "bytes_per_launch": algo, "us_per_launch": us, "achieved": gbs, "copies_rotated": copies}


# the Q4_K GEMV / GEMM microbenchmark: weight shapes [N, K] at M activation rows
MICRO_SHAPES = ((2048, 2048), (5632, 2048), (4096, 4096), (11008, 4096), (32000, 4096))
MICRO_M = (1, 16, 512)


def run_microbench(reps_per_copy):
    """One JSON line per (shape, M) through wcb_gemv_dev: M < 16 runs the dp4a
    GEMV, M >= 16 the tcgen05 tensor-core GEMM. M <= 16 is bound by the weight
    bytes (HBM roofline), M = 512 by the tensor cores (arithmetic intensity
    2*512 / 0.5625 = 1820 flop per weight byte)."""
    import torch
    import wcb
    hbm, kind = peaks()
    tf = None
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        tf = float(json.load(open(p))["bf16_tflops"])
    tf = tf or 1590.0
    st = torch.cuda.Stream()  # a created stream: the library and the events order on the same handle
    sp = st.cuda_stream
    for n, k in MICRO_SHAPES:
        for m in MICRO_M:
            algo, flops, us, copies = time_gemv(torch, wcb, sp, n, k, m, reps_per_copy)
            gbs = algo / (us * 1e-6) / 1e9
            tfs = flops / (us * 1e-6) / 1e12
            tensor = m >= 256
            frac = (tfs / tf) if tensor else (gbs / hbm)
            print(json.dumps({
                "metric": "Q4_K GEMV/GEMM microbenchmark", "shape_nk": [n, k], "m": m,
                "kernel": "gemm_tc_kernel (tcgen05)" if m >= 16 else "gemv_kernel (dp4a)",
                "us_per_launch": round(us, 3), "bytes_per_launch": algo, "flops_per_launch": flops,
                "roofline": {"bound": "tensor" if tensor else "hbm",
                             "achieved": tfs if tensor else gbs, "peak": tf if tensor else hbm,
                             "unit": "TFLOP/s" if tensor else "GB/s",
                             "frac": frac, "peak_kind": kind},
                "valid": frac < 1.5,  # far above the measured peak: the timed launches did not do the work
                "gbs": round(gbs, 1), "tflops": round(tfs, 2), "copies_rotated": copies,
                "l2": "weight copies rotated so each launch reads its weights from HBM"}), flush=True)


def cpu_baseline(path, budget_s=20.0, prompt_len=8):
    """The oracle (the reference CPU path restated in C++) on this host, with the
    reference's threading: projections on one thread, the LM head on all cores."""
    import oracle
    cores = os.cpu_count() or 1
    oracle.set_threads(cores, cores)
    o = oracle.OracleModel(path)
    from wcb import synth
    prompt = synth.random_prompt(prompt_len, o.vocab, seed=1).tolist()
    logits = o.forward(prompt, 0)
    oracle.set_threads(cores, 1)
    oracle.set_faithful(True)
    tok = int(len(logits) - 1 - np.argmax(logits[::-1]))
    n = 0
    t0 = time.perf_counter()
    while True:
        logits = o.forward([tok], o.kv_len())
        tok = int(len(logits) - 1 - np.argmax(logits[::-1]))
        n += 1
        if time.perf_counter() - t0 > budget_s or n >= 64:
            break
    dt = time.perf_counter() - t0
    o.close()
    return {"value": n / dt, "unit": "tok/s", "cores": cores, "kind": "port",
            "sample": f"{n} greedy decode tokens after an {prompt_len}-token prompt on the same TinyLlama Q4_K "
                      f"model (weights dequantised to f32 at load as the reference does; projections on 1 thread, "
                      f"LM head on {cores} threads)"}


def run_reference(args, rank, world):
    """--impl reference: the reference CPU path (the oracle port; the Rust
    reference cannot be built without a Rust toolchain) on this host."""
    if rank != 0:
        return
    path = model_file("tinyllama")
    import oracle
    cores = os.cpu_count() or 1
    oracle.set_threads(cores, cores)
    o = oracle.OracleModel(path)
    # the prompt of our arm (wcb.synth.random_prompt), drawn here with numpy alone
    prompt = np.random.default_rng(1).integers(3, o.vocab, size=PROMPT_LEN, dtype=np.int64).tolist()
    logits = o.forward(prompt, 0)  # untimed prefill
    oracle.set_threads(cores, 1)  # the reference's threading for the timed decode steps
    oracle.set_faithful(True)  # and its one-row-at-a-time matmul loop
    tok = int(len(logits) - 1 - np.argmax(logits[::-1]))
    for _ in range(args.warmup):  # about 0.6 s a step on 16 host cores
        logits = o.forward([tok], o.kv_len())
        tok = int(len(logits) - 1 - np.argmax(logits[::-1]))
    n = 0
    t0 = time.perf_counter()
    while n < args.steps:
        logits = o.forward([tok], o.kv_len())
        tok = int(len(logits) - 1 - np.argmax(logits[::-1]))
        n += 1
        if time.perf_counter() - t0 > 90.0:
            break
    dt = time.perf_counter() - t0
    v = n / dt
    line = {"metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": world, "steps": n, "warmup": args.warmup,
            "ms_per_step": dt * 1e3 / n, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (seeded N(0,0.02) weights, Q4_K dequantised to f32 at load)",
            "config": {"workload": "TinyLlama-1.1B Q4_K greedy decode after a 128-token prompt, batch 1",
                       "prompt_len": PROMPT_LEN, "global_batch": 1, "parallelism": "cpu"},
            "impl": "reference",
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": cores, "kind": "port",
                             "sample": f"{n} decode tokens from position {PROMPT_LEN + 1 + args.warmup}; projections on 1 thread "
                                       f"and the LM head on {cores} threads, as in the reference"},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_ours(args, rank, world, dist):
    import torch
    import wcb
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    global PROMPT_LEN, METRIC
    label, arch, PROMPT_LEN = MODELS[args.model]
    METRIC = f"decode tok/s ({label}, batch 1)"
    path = ensure_model(rank, world, dist, args.model)
    m = wcb.Model.load_from_gguf(path, device=local, stream_weights=args.stream_weights)
    if args.stream_weights:
        METRIC = f"decode tok/s ({label}, batch 1, layer weights streamed from pinned host memory)"
    # --sampled: the reference's default GenerationConfig (config.rs:74-78), drawn on the device
    samp = dict(temperature=0.7, top_p=0.9, top_k=40, repetition_penalty=1.1, seed=1) if args.sampled else \
        dict(temperature=0.0, repetition_penalty=1.0)
    if args.sampled:
        METRIC = f"decode tok/s ({label}, batch 1, sampled: temperature 0.7, top-p 0.9, top-k 40, penalty 1.1)"
    cfg = m.config
    sp = m.stream()
    s = torch.cuda.ExternalStream(sp)
    prompt = __import__("wcb.synth", fromlist=["x"]).random_prompt(PROMPT_LEN, cfg.vocab_size, seed=1)
    K, W = args.steps, args.warmup
    if PROMPT_LEN + W + K + 1 > cfg.max_seq_len:
        raise SystemExit(f"steps + warmup exceed the context ({cfg.max_seq_len})")
    gc = wcb.GenerationConfig(max_tokens=W + K + 1, eos_id=None, **samp)
    stream = m.infer(prompt.tolist(), gc)
    stream.next_tokens(1 + W)  # first token + W warm-up decode steps
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        torch.cuda.nvtx.range_push("timed")
        e0.record(s)
        toks = stream.next_tokens(K)
        e1.record(s)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
    if world > 1:
        dist.barrier()
    assert len(toks) == K, (len(toks), K)
    ms = e0.elapsed_time(e1)
    t = torch.tensor([ms], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    value = world * K / (ms_max * 1e-3)

    peak, peak_kind = peaks()
    wbytes = weight_bytes(cfg, path)
    avg_pos = PROMPT_LEN + 1 + W + (K - 1) / 2.0
    kv_bytes = 2 * cfg.num_layers * cfg.num_kv_heads * cfg.head_dim * avg_pos * 4
    step_bytes = wbytes + kv_bytes
    step_gbs = step_bytes / (ms_max / K * 1e-3) / 1e9

    # end to end through the public generate() call with host buffers
    gc2 = wcb.GenerationConfig(max_tokens=K + 1, eos_id=None, **samp)
    m.generate_tokens(prompt.tolist(), gc2)  # warm
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(s)
    out = m.generate_tokens(prompt.tolist(), gc2)
    f1.record(s)
    torch.cuda.synchronize()
    e2e_ms = f0.elapsed_time(f1)
    et = torch.tensor([e2e_ms], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(et, op=dist.ReduceOp.MAX)
    e2e_ms = float(et.item())
    e2e = {"value": world * len(out) / (e2e_ms * 1e-3), "unit": "tok/s",
           "h2d_bytes_per_step": PROMPT_LEN * 4 / len(out), "d2h_bytes_per_step": 4 + 64 / len(out),
           "call": "wcb_generate_tokens: %d-token prompt from host memory -> %d generated ids to host memory, "
                   "prefill included" % (PROMPT_LEN, len(out))}

    roof = gemv_roofline(torch, wcb, sp, cfg, peak) if rank == 0 else None
    if args.stream_weights:
        # the bound is the host-to-device copy of every layer's weights per token: against a
        # plain pinned-memory copy of 256 MB timed here
        from gguf import GGUFReader
        head = sum(int(t.n_bytes) for t in GGUFReader(path).tensors if t.name == "output.weight")
        layer_bytes = wbytes - head
        src = torch.empty(256 << 20, dtype=torch.uint8).pin_memory()
        dst = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
        for _ in range(3):  # warm-up: first-touch of the pinned pages and the device buffer
            dst.copy_(src, non_blocking=True)
        torch.cuda.synchronize()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record()
        for _ in range(8):
            dst.copy_(src, non_blocking=True)
        c1.record()
        torch.cuda.synchronize()
        h2d_peak = 8 * (256 << 20) / (c0.elapsed_time(c1) * 1e-3) / 1e9
        h2d = layer_bytes / (ms_max / K * 1e-3) / 1e9
        roof = None
        roofline_stream = {"bound": "h2d", "achieved": h2d, "peak": h2d_peak, "unit": "GB/s", "frac": h2d / h2d_peak,
                           "traffic": None, "peak_kind": "measured here: pinned 256 MB host-to-device copy",
                           "kernel": "layer-weight copies on the copy stream (cudaMemcpyAsync)",
                           "bytes_per_step": layer_bytes}
    if args.stream_weights:
        roofline = roofline_stream
    elif m.launches_per_step() == 1 or (args.sampled and m.launches_per_step() == 2):
        # one persistent kernel per decode step (+ the sampler kernel of a sampled
        # config): its bytes are the step's weights + KV reads
        traffic = None
        if arch in NCU_STEP_TRAFFIC:
            cap_bytes, cap_pos = NCU_STEP_TRAFFIC[arch]
            kv_row = 2 * cfg.num_layers * cfg.num_kv_heads * cfg.head_dim * 4
            traffic = cap_bytes + kv_row * (avg_pos - cap_pos)
        roofline = {"bound": "hbm", "achieved": step_gbs, "peak": peak, "unit": "GB/s", "frac": step_gbs / peak,
                    "traffic": traffic, "peak_kind": peak_kind, "kernel": "decode_step_kernel (persistent decode step)",
                    "us_per_launch": ms_max / K * 1e3, "bytes_per_launch": step_bytes,
                    "traffic_note": None if traffic is None else
                    "ncu DRAM read+write bytes of one launch at KV position %d, moved to the mean position %.1f by "
                    "the f32 KV row bytes in between" % (NCU_STEP_TRAFFIC[arch][1], avg_pos)}
    elif roof is not None:
        roofline = {"bound": "hbm", "achieved": roof["achieved"], "peak": peak, "unit": "GB/s",
                    "frac": roof["achieved"] / peak, "traffic": None, "peak_kind": peak_kind,
                    "kernel": roof["kernel"], "us_per_launch": roof["us_per_launch"],
                    "bytes_per_launch": roof["bytes_per_launch"]}
    else:
        roofline = None
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(path)
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": ms_max / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32 activations, Q4_K weights (int8 dp4a on exact 24-bit activation limbs)",
            "data": f"synthetic (seeded N(0,0.02) weights quantised to {label.split()[-1]}; "
                    f"{PROMPT_LEN} uniform-random prompt ids)",
            "config": {"workload": f"{label} greedy decode after a {PROMPT_LEN}-token prompt, batch 1 per GPU",
                       "model": arch, "prompt_len": PROMPT_LEN, "global_batch": world,
                       "seq_len": PROMPT_LEN + 1 + W + K, "parallelism": f"dp{world} (independent replicas)",
                       "l2": f"weights {wbytes / 1e6:.0f} MB > 126 MB L2, no flush", "kv_cache": "f32",
                       "cuda_graph": m.launches_per_step() > 1},
            "roofline": roofline,
            "step_roofline": {"bytes_per_step": step_bytes, "weight_bytes": wbytes, "achieved_gbs": step_gbs,
                              "frac": step_gbs / peak, "peak_kind": peak_kind},
            "gemv_roofline": None if roof is None else {
                "achieved": roof["achieved"], "frac": roof["achieved"] / peak, "unit": "GB/s",
                "kernel": roof["kernel"], "shape_nk": roof["shape_nk"],
                "us_per_launch": roof["us_per_launch"], "bytes_per_launch": roof["bytes_per_launch"]},
            "e2e": e2e,
            "gpu_launches": m.launches_per_step() * K,
            "clocks": clk.summary(),
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    stream.close()
    m.close()


def run_tp(args, rank, world, dist):
    """The Llama-2-70B shape (hidden 8192, FFN 28672, 64 / 8 heads, vocab 32000, Q4_K),
    tensor-parallel over the `world` ranks of this torchrun: one sequence, greedy
    decode after a `--prompt`-token prompt; value = the group's tokens/s."""
    import torch
    import wcb
    from wcb import synth
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    layers = args.layers
    path = [synth.cached_model("llama70b", MODEL_DIR, num_layers=layers, layer_period=2)
            if local == 0 else None]
    if world > 1:
        dist.barrier()
        dist.broadcast_object_list(path, src=0)
    path = path[0]
    tp_id = [wcb.tp_unique_id() if rank == 0 else None]
    if world > 1:
        dist.broadcast_object_list(tp_id, src=0)
    m = wcb.Model.load_from_gguf(path, device=local, tp_rank=rank, tp_size=world, tp_id=tp_id[0],
                                 max_seq=args.prompt + args.warmup + args.steps + 8,
                                 use_persistent=not args.tp_per_op)
    exchange = "nccl"
    if world > 1 and not args.tp_nccl:  # decode steps: partial sums by peer stores over NVLink
        handles = [None] * world
        dist.all_gather_object(handles, m.tp_ipc_handle())
        m.tp_connect(handles)
        exchange = "peer stores"
    cfg = m.config
    s = torch.cuda.ExternalStream(m.stream())
    prompt = synth.random_prompt(args.prompt, cfg.vocab_size, seed=1)
    K, W = args.steps, args.warmup
    gc = wcb.GenerationConfig(max_tokens=W + K + 1, temperature=0.0, repetition_penalty=1.0, eos_id=None)
    stream = m.infer(prompt.tolist(), gc)
    stream.next_tokens(1 + W)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        e0.record(s)
        toks = stream.next_tokens(K)
        e1.record(s)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    assert len(toks) == K, (len(toks), K)
    t = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    peak, peak_kind = peaks()
    wbytes = weight_bytes(cfg, path) / world  # each rank streams its shard
    per_rank_gbs = wbytes / (ms / K * 1e-3) / 1e9
    if rank == 0:
        print(json.dumps({
            "metric": "decode tok/s (Llama-2-70B shape Q4_K, batch 1, tensor parallel)", "value": K / (ms * 1e-3),
            "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": ms / K,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32 activations, Q4_K weights", "data": "synthetic (seeded N(0,0.02) weights quantised to Q4_K)",
            "config": {"workload": f"Llama-2-70B shape, {layers} of its 80 layers, greedy decode after a "
                                   f"{args.prompt}-token prompt", "layers": layers, "prompt_len": args.prompt,
                       "weights": "two distinct layers' synthetic weights, repeated (every layer's bytes are read)",
                       "persistent_step": m.launches_per_step() == 1,
                       "parallelism": f"tp{world} (partial sums of attn-out and ffn-down all-reduced by {exchange}; "
                                      "prefill: NCCL)",
                       "l2": "weights > 126 MB L2, no flush"},
            "roofline": {"bound": "hbm", "achieved": per_rank_gbs, "peak": peak, "unit": "GB/s",
                         "frac": per_rank_gbs / peak, "traffic": None, "peak_kind": peak_kind,
                         "kernel": "whole decode step per rank (shard weights / ms per token)",
                         "bytes_per_launch": wbytes},
            "gpu_launches": m.launches_per_step() * K,
            "clocks": clk.summary(),
        }), flush=True)
    stream.close()
    m.close()


def run_tp_batch(args, rank, world, dist):
    """The Llama-2-70B shape tensor-parallel over the ranks with `--tp-batch` sequences
    decoded together (the batched tensor-core step, partial sums all-reduced by NCCL):
    greedy decode after `--prompt`-token prompts. Decode time = wcb_generate_batch with
    max_tokens steps + 1 minus the same call with max_tokens 1, maxed over the ranks."""
    import torch
    import wcb
    from wcb import synth
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    layers, B, P, K, W = args.layers, args.tp_batch, args.prompt, args.steps, args.warmup
    path = [synth.cached_model("llama70b", MODEL_DIR, num_layers=layers, layer_period=2)
            if local == 0 else None]
    if world > 1:
        dist.barrier()
        dist.broadcast_object_list(path, src=0)
    path = path[0]
    tp_id = [wcb.tp_unique_id() if rank == 0 else None]
    if world > 1:
        dist.broadcast_object_list(tp_id, src=0)
    m = wcb.Model.load_from_gguf(path, device=local, tp_rank=rank, tp_size=world, tp_id=tp_id[0],
                                 max_seq=P + K + 8, max_batch=B)
    cfg = m.config
    s = torch.cuda.ExternalStream(m.stream())
    prompts = [synth.random_prompt(P, cfg.vocab_size, seed=1 + i).tolist() for i in range(B)]

    def timed(max_tokens):
        gc = wcb.GenerationConfig(max_tokens=max_tokens, temperature=0.0, repetition_penalty=1.0, eos_id=None)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0.record(s)
        out = m.generate_batch(prompts, gc)
        e1.record(s)
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device="cuda")
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item()), out

    timed(W + 1)
    t_pre, _ = timed(1)
    with ClockSampler(local) as clk:
        t_full, out = timed(K + 1)
    assert all(len(o) == K + 1 for o in out)
    slots, launches = m.batch_info()
    dec_ms = t_full - t_pre
    peak, peak_kind = peaks()
    wbytes = weight_bytes(cfg, path) / world
    per_rank_gbs = wbytes / (dec_ms / K * 1e-3) / 1e9
    if rank == 0:
        print(json.dumps({
            "metric": f"decode tok/s (Llama-2-70B shape Q4_K, batch {B}, tensor parallel)",
            "value": B * K / (dec_ms * 1e-3), "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": dec_ms / K, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32 activations (fp16 hi+lo tensor-core operands), Q4_K weights",
            "data": "synthetic (seeded N(0,0.02) weights quantised to Q4_K)",
            "config": {"workload": f"Llama-2-70B shape, {layers} of its 80 layers, {B} sequences x {P}-token "
                                   f"prompts, greedy", "layers": layers, "prompt_len": P, "batch": B,
                       "parallelism": f"tp{world} (batched step; partial sums all-reduced by NCCL)",
                       "l2": "weights > 126 MB L2, no flush"},
            "roofline": {"bound": "hbm", "achieved": per_rank_gbs, "peak": peak, "unit": "GB/s",
                         "frac": per_rank_gbs / peak, "traffic": None, "peak_kind": peak_kind,
                         "kernel": "whole batched decode step per rank (shard weights / ms per step)",
                         "bytes_per_launch": wbytes},
            "prefill": {"value": B * P / (t_pre * 1e-3), "unit": "tok/s", "ms": t_pre},
            "gpu_launches": launches * K, "launches_per_step": launches,
            "clocks": clk.summary(),
        }), flush=True)
    m.close()


def run_serve(args, rank, world, dist):
    """Batched serving on the TinyLlama shape: `sequences` prompts of `prompt`
    uniform-random ids split evenly over the ranks (independent replicas), each
    decoding `steps` greedy tokens, fp16 KV cache. Each rank serves its share with
    one wcb_generate_batch call (prefill per sequence, then batched decode steps on
    the tensor cores). Decode time = that call minus the same call with
    max_tokens 1 (prefill + first token only), both timed with CUDA events on the
    model's stream and maxed over the ranks."""
    import torch
    import wcb
    from wcb import synth
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    path = ensure_model(rank, world, dist, "tinyllama")
    S, P, K, W = args.sequences, args.prompt, args.steps, args.warmup
    if S % world:
        raise SystemExit("--sequences must split evenly over the ranks")
    B = S // world
    max_seq = P + K + 8
    m = wcb.Model.load_from_gguf(path, device=local, kv_dtype=wcb.KV_F16, max_batch=B, max_seq=max_seq)
    cfg = m.config
    sp = m.stream()
    s = torch.cuda.ExternalStream(sp)
    prompts = [synth.random_prompt(P, cfg.vocab_size, seed=1000 + rank * B + i).tolist() for i in range(B)]
    # --sampled: the reference's default GenerationConfig (config.rs:74-78), drawn on the device
    samp = dict(temperature=0.7, top_p=0.9, top_k=40, repetition_penalty=1.1, seed=1) if args.sampled else \
        dict(temperature=0.0, repetition_penalty=1.0)

    def timed(max_tokens):
        gc = wcb.GenerationConfig(max_tokens=max_tokens, eos_id=None, **samp)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0.record(s)
        out = m.generate_batch(prompts, gc)
        e1.record(s)
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device="cuda")
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item()), out

    timed(W + 1)  # warm-up: prefill path, graph capture, W batched steps
    t_pre, _ = timed(1)
    with ClockSampler(local) as clk:
        t_full, out = timed(K + 1)
    assert all(len(o) == K + 1 for o in out), [len(o) for o in out]
    slots, launches = m.batch_info()
    dec_ms = t_full - t_pre
    value = world * B * K / (dec_ms * 1e-3)
    peak, peak_kind = peaks()
    wbytes = weight_bytes(cfg, path)
    avg_pos = P + 1 + (K - 1) / 2.0
    kv_bytes = B * 2 * cfg.num_layers * cfg.num_kv_heads * cfg.head_dim * avg_pos * 2
    step_ms = dec_ms / K
    step_gbs = (wbytes + kv_bytes) / (step_ms * 1e-3) / 1e9
    if rank == 0:
        print(json.dumps({
            "metric": "batched decode tok/s (TinyLlama-1.1B Q4_K, %d sequences x %d-token prompt, fp16 KV%s)"
                      % (S, P, ", sampled: temperature 0.7, top-p 0.9, top-k 40, penalty 1.1" if args.sampled else ""),
            "value": value, "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": step_ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32 activations (fp16 hi+lo tensor-core operands), Q4_K weights, fp16 KV",
            "data": "synthetic (seeded N(0,0.02) weights quantised to Q4_K; uniform-random prompt ids)",
            "config": {"workload": f"{S} sequences x ({P}-token prompt + {K} {'sampled' if args.sampled else 'greedy'} "
                                   f"tokens), split over {world} GPU(s)",
                       "model": "tinyllama-1.1b-arch", "sequences_per_gpu": B, "prompt_len": P,
                       "parallelism": f"dp{world} (independent replicas)", "kv_cache": "f16",
                       "l2": "weights 582 MB + KV > 126 MB L2, no flush"},
            "roofline": {"bound": "hbm", "achieved": step_gbs, "peak": peak, "unit": "GB/s", "frac": step_gbs / peak,
                         "traffic": None, "peak_kind": peak_kind,
                         "kernel": "batched decode step (tensor-core GEMMs + attention, one graph)",
                         "bytes_per_step": wbytes + kv_bytes, "weight_bytes": wbytes, "kv_bytes": kv_bytes},
            "prefill": {"value": world * B * P / (t_pre * 1e-3), "unit": "tok/s", "ms": t_pre},
            "e2e": {"value": world * B * (K + 1) / (t_full * 1e-3), "unit": "tok/s",
                    "h2d_bytes_per_step": B * P * 4 / (K + 1), "d2h_bytes_per_step": B * 4,
                    "call": "wcb_generate_batch: prompts from host memory -> generated ids to host memory, "
                            "prefill included"},
            "gpu_launches": launches * K, "batch_slots": slots, "launches_per_step": launches,
            "clocks": clk.summary(),
        }), flush=True)
    m.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--gemv-only", type=int, default=0, metavar="REPS",
                    help="only time the dominant GEMV (REPS launches per weight copy) and print its line")
    ap.add_argument("--microbench", type=int, default=0, metavar="REPS",
                    help="Q4_K GEMV/GEMM sweep over 5 weight shapes x M in (1, 16, 512), REPS launches per weight copy")
    ap.add_argument("--model", choices=sorted(MODELS), default="tinyllama",
                    help="the decoder shape of the decode line (the headline is tinyllama)")
    ap.add_argument("--tp", action="store_true",
                    help="the Llama-2-70B shape, tensor-parallel over the torchrun ranks, instead of the headline")
    ap.add_argument("--layers", type=int, default=80, help="--tp: layers of the 70B shape to build")
    ap.add_argument("--prompt", type=int, default=1024, help="--tp: prompt tokens before the timed decode")
    ap.add_argument("--tp-nccl", action="store_true", help="--tp: all-reduce decode steps with NCCL too")
    ap.add_argument("--tp-per-op", action="store_true",
                    help="--tp: decode steps on the per-op kernels (CUDA graph) instead of the single-launch step")
    ap.add_argument("--tp-batch", type=int, default=1, help="--tp: sequences decoded together (batched step)")
    ap.add_argument("--stream-weights", action="store_true",
                    help="decode line with the layer weights streamed from pinned host memory (not the headline)")
    ap.add_argument("--sampled", action="store_true",
                    help="decode with the reference's default sampling config instead of greedy")
    ap.add_argument("--serve", action="store_true",
                    help="batched serving of --sequences prompts of --prompt tokens (default 2048) over the ranks")
    ap.add_argument("--sequences", type=int, default=32, help="--serve: sequences over all ranks")
    args = ap.parse_args()
    if args.serve and "--prompt" not in sys.argv:
        args.prompt = 2048
    if args.gemv_only:
        import torch
        import wcb
        from wcb import synth
        cfg = synth.PRESETS["tinyllama"]
        st = torch.cuda.Stream()
        stream_ptr = st.cuda_stream
        r = gemv_roofline(torch, wcb, stream_ptr, cfg, peaks()[0], reps_per_copy=args.gemv_only)
        print(json.dumps(r), flush=True)
        return
    if args.microbench:
        run_microbench(args.microbench)
        return
    if args.warmup < 3:
        args.warmup = 3
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    dist = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
    try:
        if args.tp and args.tp_batch > 1:
            run_tp_batch(args, rank, world, dist)
        elif args.tp:
            run_tp(args, rank, world, dist)
        elif args.serve:
            run_serve(args, rank, world, dist)
        else:
            run_ours(args, rank, world, dist)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()

"""Decode benchmark: Llama-2-7B-shaped int8 model, batch 1, on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one decode token (the hot path: TransformerEngine::forward_single_token
of the reference) at batch 1.  Workload: random-init int8 weights (seed 0)
generated on the device, a 512-token random prompt processed first (untimed),
then W warm-up and K timed greedy decode steps with an fp16 KV cache.  The
7.4 GB of weights read per step are 59x the 126 MB L2, so no flush is needed.

value   tokens/s of all ranks (each rank decodes its own sequence; one JSON line
        from rank 0), device-timed with CUDA events on the engine's stream,
        max over ranks.
e2e     the same metric through the reference-facing API with host buffers:
        bt_engine_forward_token with the token id copied host->device and the
        32000 fp32 logits copied device->host every step.
roofline  algorithmic HBM bytes per step (weights + norms + embedding row + KV
        read/write) / step time, against the measured copy bandwidth; plus the
        dominant kernel (gate/up GEMV) timed per launch with events.
cpu_baseline  the reference's own CPU engine (oracle/_ref/libbtref.so; falls
        back to the C restatement) timed for a few 7B decode tokens on rank 0.

--impl reference times the reference CPU implementation of the same step
(rank 0 only) and prints the same JSON line with "impl": "reference".
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tokens/s and % HBM roofline at 1/2/4/8 B200 (7B int8, batch 1)"
PEAKS_FILE = os.path.join(ROOT, "MEASURED_PEAKS.json")
FALLBACK_HBM = 6650.0


def hbm_peak():
    try:
        with open(PEAKS_FILE) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.out = os.path.join("/tmp", f"bt_clocks_{os.getpid()}.csv")

    def start(self):
        """Starts sampling every 50 ms and returns once the first sample is written (nvidia-smi
        takes a while to come up), so samples cover the whole timed region that follows."""
        try:
            self.f = open(self.out, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=self.f, stderr=subprocess.DEVNULL)
            t0 = time.time()
            while time.time() - t0 < 5.0 and self.proc.poll() is None:
                if os.path.getsize(self.out) > 0:
                    break
                time.sleep(0.02)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.06)  # one more sample at the end of the region
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.out) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx = max(mx, float(parts[2]))
                except ValueError:
                    continue
                for n, v in zip(names, parts[5:9]):
                    if v.lower().startswith("active"):
                        reasons.add(n)
        os.unlink(self.out)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# ---------------------------------------------------------------- step-kernel timeline

PHASE_KINDS = ("qkv", "attention", "oproj", "gateup", "down")


def trace_summary(tr: np.ndarray, n_layers: int) -> dict:
    """Per-phase latency breakdown of one step from bt_engine_read_trace ([P][G][8] ns).

    For each phase kind, medians over the middle layers (microseconds):
      dur      end of the previous phase -> end of this one (last CTA's release)
      wait     end of the previous phase -> median CTA passing its counter wait
      digits   counter wait -> input digits in shared memory (median CTA)
      first    digits -> first row tile's sums at the finisher (median CTA)
      tail     median CTA's end -> last CTA's end (imbalance and merge polls)
      lead     producer's first copy of the phase -> the phase's end (how far ahead the weights stream)
    """
    t = tr.astype(np.float64)
    P = t.shape[0]
    t[t == 0] = np.nan
    end = np.nanmax(t[:, :, 3], axis=1)
    start = np.nanmedian(t[:, :, 0], axis=1)
    out = {k: {"dur": [], "wait": [], "digits": [], "first": [], "tail": [], "lead": []} for k in PHASE_KINDS}
    out["head"] = {"dur": [], "wait": [], "digits": [], "first": [], "tail": [], "lead": []}
    for p in range(1, P):
        kind = "head" if p == P - 1 else PHASE_KINDS[p % 5]
        layer = p // 5
        if kind != "head" and not (1 <= layer < n_layers - 1):
            continue
        d = out[kind]
        d["dur"].append(end[p] - end[p - 1])
        d["wait"].append(start[p] - end[p - 1])
        d["digits"].append(np.nanmedian(t[p, :, 1] - t[p, :, 0]))
        d["first"].append(np.nanmedian(t[p, :, 2] - t[p, :, 1]))
        d["tail"].append(end[p] - np.nanmedian(t[p, :, 3]))
        d["lead"].append(end[p] - np.nanmin(t[p, :, 4]))
    res = {}
    for k, d in out.items():
        res[k] = {m: (round(float(np.nanmedian(v)) / 1000.0, 2) if len(v) and np.isfinite(np.nanmedian(v)) else None)
                  for m, v in d.items()}
    res["step_us"] = round(float((np.nanmax(t[:, :, 3]) - np.nanmin(t[:, :, 0])) / 1000.0), 1)
    return res


# ---------------------------------------------------------------- diagnostics: GEMV microbenchmark, tiny model

def c1_gemv(torch, bt, dev, log):
    """The dequant-GEMV microbenchmark: W 4096 x 4096 int8 (uniform [-127, 127]) with fp32
    scales per 32-block (U(0.001, 0.02)), x [B, 4096] fp32 N(0, 1), y = x W^T, B in {1, 4, 16}.
    16 copies of W (302 MB, over twice L2) are cycled so every launch streams W from HBM.
    HBM bytes per launch: W (int8 + scales) + x + y."""
    import ctypes
    M = K = 4096
    copies = 16
    peak, _ = hbm_peak()
    g = torch.Generator(device=f"cuda:{dev}").manual_seed(0)
    qs = torch.randint(-127, 128, (M, K), dtype=torch.int8, device=f"cuda:{dev}", generator=g)
    sc = torch.rand((M, K // 32), device=f"cuda:{dev}", generator=g) * 0.019 + 0.001
    blocks = torch.empty((M * K // 32, 36), dtype=torch.uint8, device=f"cuda:{dev}")
    blocks[:, :4] = sc.reshape(-1, 1).view(torch.uint8).reshape(-1, 4)
    blocks[:, 4:] = qs.reshape(-1, 32).view(torch.uint8)
    units = bt.pack_q8_units(blocks, M, K)
    ub = units.numel()
    units_all = units.repeat(copies)
    split = torch.cat([qs.view(torch.uint8).reshape(-1), sc.reshape(-1).view(torch.uint8)])
    sb = split.numel()
    split_all = split.repeat(copies)
    out = []
    lib = bt.load()
    for B in (1, 4, 16):
        x = torch.randn((B, K), device=f"cuda:{dev}", generator=g)
        y = torch.empty((B, M), device=f"cuda:{dev}")
        w_bytes = M * K + M * (K // 32) * 4
        nbytes = w_bytes + 4 * B * K + 4 * B * M
        for kind, name, w, stride in ((0, "tcgen05 GEMV (tile layout)", units_all, ub),
                                      (1, "tcgen05 GEMM (tile layout, token image)", units_all, ub),
                                      (2, "CUDA-core GEMV (split layout)", split_all, sb)):
            if kind == 0 and B != 1:
                continue
            us = ctypes.c_float()
            bt.native.check(lib.bt_cuda_gemv_bench(kind, w.data_ptr(), x.data_ptr(), y.data_ptr(), M, K, B, copies,
                                                   stride, 200, None, ctypes.byref(us)))
            gbs = nbytes / (us.value * 1e-6) / 1e9
            out.append({"B": B, "kernel": name, "us": round(us.value, 2), "GBps": round(gbs, 1),
                        "frac_of_measured_hbm": round(gbs / peak, 3), "bytes": nbytes})
    log("[ours] C1 GEMV: " + json.dumps(out))
    return out


def c0_tiny(torch, bt, dev, log):
    """The tiny Llama-style config (D288 F768 L6 H6 V32000): 16-token prompt (prefilled), then
    128 greedy decode steps at batch 1 with an fp32 KV cache, device-timed."""
    from blocktensor_b200 import synthetic
    cfg = synthetic.config("tiny", 256)
    eng = bt.TransformerEngine(cfg, device=dev)
    eng.generate(seed=0, sigma=0.02)
    kv = bt.KVCache(eng, 256, bt.BT_KV_FP32)
    prompt = synthetic.tokens(0, 16, cfg.vocab_size)
    eng.prefill(kv, prompt)
    eng.steps(kv, 1)
    torch.cuda.synchronize()
    stream = torch.cuda.ExternalStream(eng.stream_handle, device=torch.device("cuda", dev))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = 128
    e0.record(stream)
    eng.steps(kv, n, stream=eng.stream_handle)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    nbytes = sum(synthetic.step_bytes(cfg, 17 + i + 1, 4) for i in range(n)) / n
    peak, _ = hbm_peak()
    gbs = nbytes / (ms / n * 1e-3) / 1e9
    kv.close()
    eng.close()
    res = {"tokens_per_s": round(n / (ms / 1000.0), 1), "us_per_token": round(ms / n * 1000.0, 1),
           "bytes_per_token": int(nbytes), "GBps": round(gbs, 1), "frac_of_measured_hbm": round(gbs / peak, 4)}
    log("[ours] C0 tiny decode: " + json.dumps(res))
    return res


# ---------------------------------------------------------------- CPU reference

def cpu_reference_tokens_per_s(n_tokens: int, warmup: int, budget_s: float, log=print, pos0: int = 0):
    """Time the reference CPU engine on the 7B-shaped model (seed 0), decoding from position
    pos0: each step attends over pos + 1 cached positions, as the GPU arm's steps after a
    pos0-token prompt do.  The prompt itself is not run (on one host thread it would take
    hours): the earlier cache rows stay as allocated, which changes no amount of work."""
    from oracle import oracle as O
    from blocktensor_b200 import synthetic
    shape = synthetic.SHAPES["llama2-7b"]
    max_seq = pos0 + warmup + n_tokens + 2
    ocfg = O.make_config(*shape, max_seq)
    t0 = time.time()
    m = O.Model(ocfg, seed=0)
    log(f"[cpu] 7B weights generated on the host in {time.time() - t0:.1f} s")
    kind = "reference" if O.ref_available() else "port"
    if kind == "reference":
        eng = O.RefEngine(O.RefLib(), m, kv_max_seq=max_seq)
        step = lambda t, p: eng.forward(t, p)
    else:
        kv = O.KV(ocfg, max_seq)
        step = lambda t, p: O.forward_token(m, kv, t, p, nthreads=1)
    prompt = synthetic.tokens(0, 1, shape[0])
    tok, pos = int(prompt[0]), pos0
    for _ in range(warmup):
        tok = int(np.argmax(step(tok, pos)))
        pos += 1
    done, t0 = 0, time.perf_counter()
    while done < n_tokens:
        tok = int(np.argmax(step(tok, pos)))
        pos += 1
        done += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    return done / dt, kind, done, pos


def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    n = max(1, min(args.steps, 3))
    w = min(args.warmup, 1)
    tps, kind, done, pos = cpu_reference_tokens_per_s(n, w, budget_s=90.0, log=lambda *a: print(*a, file=sys.stderr),
                                                      pos0=args.prompt)
    sample = (f"{done} decode tokens of the 7B-shaped int8 model after {w} warm-up token(s), contexts {pos - done + 1}-{pos} "
              f"(the GPU arm's contexts after its {args.prompt}-token prompt)")
    line = {
        "impl": "reference", "metric": METRIC, "value": tps, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": done, "warmup": w, "ms_per_step": 1000.0 / tps, "higher_is_better": True,
        # the same one sequence as our arm (tensor parallel when N > 1, unless --replicas)
        "scaling": "strong" if (args.gpus > 1 and not args.replicas) else "weak",
        "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": "llama2-7b-shaped int8 decode, batch 1 (reference CPU backend, one host thread)",
                   "model": "llama2-7b", "global_batch": 1, "parallelism": "reference CPU",
                   "vocab": 32000, "dim": 4096, "hidden": 11008, "layers": 32, "heads": 32, "head_dim": 128},
        "cpu_baseline": {"value": tps, "unit": "tokens/s", "cores": 1, "kind": kind, "sample": sample},
        "e2e": {"value": tps, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- CUDA arm

def run_ours(args):
    import torch
    import blocktensor_b200 as bt
    from blocktensor_b200 import synthetic

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
        pg = dist

    def log(*a):
        if rank == 0:
            print(*a, file=sys.stderr, flush=True)

    shape = args.model
    prompt_len, W, K = args.prompt, args.warmup, args.steps
    max_seq = prompt_len + W + K + args.e2e_steps + args.profile_steps + 3
    cfg = synthetic.config(shape, max_seq)
    if args.layers:
        # truncated depth, for small profiler captures only (never a bench line)
        cfg.num_layers = args.layers
    # N > 1: one sequence, tensor parallel over the N GPUs (--replicas: N independent sequences)
    tpw = world if (world > 1 and not args.replicas) else 1
    t0 = time.time()
    eng = bt.TransformerEngine(cfg, device=local, rope_theta=synthetic.ROPE_THETA[shape],
                               tp_rank=rank if tpw > 1 else 0, tp_world=tpw)
    eng.generate(seed=0, sigma=0.02)
    if tpw > 1:
        from blocktensor_b200 import tp
        tp.connect(eng)
    kv = bt.KVCache(eng, max_seq, bt.BT_KV_FP16)
    log(f"[ours] {shape}: weights generated on device in {time.time() - t0:.1f} s")
    prompt = synthetic.tokens(rank if tpw == 1 else 0, prompt_len, cfg.vocab_size)
    t0 = time.time()
    prompt_info = None
    if tpw == 1 and not args.no_prefill:
        # the prompt's positions but the last as batched tensor-core GEMMs (bt_engine_prefill),
        # timed on the host around the call (it returns when done); the last prompt token is
        # the first decode step
        torch.cuda.synchronize()
        tp0 = time.perf_counter()
        eng.prefill(kv, prompt)
        pf_s = time.perf_counter() - tp0
        prompt_info = {"api": "bt_engine_prefill", "positions": prompt_len - 1, "seconds": pf_s,
                       "tokens_per_s": (prompt_len - 1) / pf_s}
        eng.steps(kv, 1)
    else:
        eng.begin(kv, prompt)
        eng.steps(kv, prompt_len)      # prompt, one position per step (untimed)
    eng.steps(kv, W)                   # warm-up decode steps
    torch.cuda.synchronize()
    log(f"[ours] prompt {prompt_len} + warm-up {W} steps in {time.time() - t0:.1f} s"
        + (f" (prefill {prompt_info['tokens_per_s']:.0f} tokens/s)" if prompt_info else ""))

    stream = torch.cuda.ExternalStream(eng.stream_handle, device=torch.device("cuda", local))
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    pos0 = prompt_len + W
    clocks = ClockSampler(local)
    if pg:
        pg.barrier()
    torch.cuda.synchronize()
    launches0 = bt.launch_count()
    clocks.start()
    ev0.record(stream)
    eng.steps(kv, K, stream=eng.stream_handle)
    ev1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    if pg:
        pg.barrier()
    launches = bt.launch_count() - launches0
    ms = ev0.elapsed_time(ev1)
    if pg:
        t = torch.tensor([ms], device="cuda")
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / K
    seqs = world if tpw == 1 else 1  # sequences decoded side by side
    value = seqs * K / (ms / 1000.0)

    # algorithmic bytes per step of this GPU (its share under tensor parallelism), over the timed contexts
    kvb = 2
    if tpw == 1:
        bytes_avg = sum(synthetic.step_bytes(cfg, pos0 + i + 1, kvb) for i in range(K)) / K
    else:
        bytes_avg = sum(kv.step_info(pos0 + i + 1)[1] for i in range(K)) / K
    peak, peak_kind = hbm_peak()
    achieved = bytes_avg / (ms_step / 1000.0) / 1e9

    # end to end through the reference-facing call with host buffers
    E = args.e2e_steps
    logits = torch.empty(cfg.vocab_size, dtype=torch.float32).pin_memory()
    tok_state = kv.state()[1]
    pos = pos0 + K
    import ctypes
    am = ctypes.c_uint32()
    lib = bt.load()
    torch.cuda.synchronize()
    if pg:
        pg.barrier()
    t0 = time.perf_counter()
    tok = tok_state
    for i in range(E):
        bt.native.check(lib.bt_engine_forward_token(eng.handle, kv.handle, tok, pos + i,
                                                    logits.data_ptr(), ctypes.byref(am)))
        tok = am.value
    e2e_s = time.perf_counter() - t0
    if pg:
        t = torch.tensor([e2e_s], device="cuda")
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e = seqs * E / e2e_s
    vocab_local = cfg.vocab_size
    if tpw > 1:
        from blocktensor_b200 import tp
        vocab_local = tp.shard(cfg.vocab_size, cfg.dim, cfg.hidden_dim, cfg.num_heads, cfg.num_kv_heads,
                               cfg.head_dim, rank, world).vocab  # this rank's logits come back

    # optional diagnostic: the same step as one launch per operation, events around every launch
    breakdown = None
    if args.profile_steps > 0:
        prof = eng.profile(kv, args.profile_steps)
        breakdown = {k: round(v / args.profile_steps * 1000.0, 1) for k, v in prof.items()}  # us per step

    # optional diagnostic: per-phase device timestamps of one more step (not timed)
    timeline = None
    if args.trace:
        eng.set_trace(True)
        eng.steps(kv, 1)
        torch.cuda.synchronize()
        timeline = trace_summary(eng.read_trace(), cfg.num_layers)
        eng.set_trace(False)
        log("[ours] phase timeline (us): " + json.dumps(timeline))

    diag = None
    if rank == 0 and world == 1 and not args.no_diagnostics and not args.layers:
        diag = {"prompt_prefill": prompt_info, "c1_gemv": c1_gemv(torch, bt, local, log),
                "c0_tiny_decode": c0_tiny(torch, bt, local, log)}

    # DRAM bytes per launch of the step kernel from an ncu capture (profiles/), scaled to this model
    traffic = None
    tfile = os.path.join(ROOT, "profiles", "decode_step_traffic.json")
    if os.path.exists(tfile) and not args.layers and tpw == 1:
        try:
            traffic = json.load(open(tfile))[shape]["dram_bytes_per_launch"]
        except Exception:
            traffic = None

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            tps, kind, done, p = cpu_reference_tokens_per_s(2, 1, budget_s=45.0, log=log, pos0=prompt_len)
            cpu = {"value": tps, "unit": "tokens/s", "cores": 1, "kind": kind,
                   "sample": f"{done} decode tokens of the same 7B-shaped model on one host thread "
                             f"(the reference engine is single-threaded), context {p - done + 1}-{p}"}
        except Exception as ex:  # the baseline is reported, never required
            cpu = {"value": None, "unit": "tokens/s", "cores": 1, "kind": "reference",
                   "sample": f"unavailable: {type(ex).__name__}: {ex}"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong" if tpw > 1 else "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": (f"{shape}-shaped int8 decode, batch 1, tensor parallel over {world} GPUs"
                                    if tpw > 1 else f"{shape}-shaped int8 decode, batch 1 per GPU"),
                       "model": shape, "global_batch": seqs, "seq_len": prompt_len, "prompt": prompt_len,
                       "decode_steps": K, "kv_cache": "fp16", "activations": "fp32",
                       "weights": "int8 Q8_0 (fp32 scale per 32)",
                       "parallelism": f"tp{world}" if tpw > 1 else (f"replicas{world}" if world > 1 else "single"),
                       "l2": "inputs larger than L2 (7.4 GB of weights per step)",
                       "truncated_layers": args.layers or None},
            # the persistent step kernel is the only kernel of the timed region: one launch per token
            "roofline": {"kernel": "decode_step_kernel (one launch per token)", "bound": "hbm",
                         "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_source": peak_kind, "bytes_per_launch": bytes_avg,
                         "us_per_launch": ms_step * 1000.0, "traffic": traffic,
                         "launch_per_op_breakdown_us": breakdown, "phase_timeline_us": timeline},
            "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": 32,
                    "d2h_bytes_per_step": vocab_local * 4 + 32,
                    "api": "bt_engine_forward_token(host token, host logits)"},
            "gpu_launches": launches,
            "diagnostics": diag,
            "clocks": clk,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    kv.close()
    eng.close()
    if pg:
        pg.barrier()
        pg.destroy_process_group()
    return 0


# ---------------------------------------------------------------- batched decode (TinyLlama, 64 sequences)

def run_batched(args):
    """TinyLlama-1.1B-shaped batched decode: 64 independent sequences with random prompts of
    uniform length in [128, 4096], 128 greedy steps each with an fp16 KV cache, sharded over
    the ranks (64 / N sequences per GPU, weights replicated, no collective on the data path).
    A step decodes one token of every sequence of the rank's batch (bt_batch_steps);
    value = all ranks' tokens / max over ranks of the device time."""
    import torch
    import blocktensor_b200 as bt
    from blocktensor_b200 import synthetic

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
        pg = dist

    def log(*a):
        if rank == 0:
            print(*a, file=sys.stderr, flush=True)

    n_total = args.sequences
    per = n_total // world
    seqs = list(range(rank * per, (rank + 1) * per))
    W, K = args.warmup, args.steps
    rng = np.random.default_rng(1234)
    ctx = rng.integers(128, 4097, n_total)  # the same draw on every rank
    max_seq = int(ctx.max()) + W + K + args.e2e_steps + 2
    cfg = synthetic.config("tinyllama-1.1b", max_seq)
    eng = bt.TransformerEngine(cfg, device=local, rope_theta=synthetic.ROPE_THETA["tinyllama-1.1b"])
    eng.generate(seed=0, sigma=0.02)
    P = args.page_tokens
    n_pages = sum(-(-(int(ctx[s]) + W + args.steps + args.e2e_steps + 2) // P) for s in seqs) if P else 0
    batch = bt.Batch(eng, per, max_seq, bt.BT_KV_FP16, page_tokens=P, n_pages=n_pages)
    t0 = time.time()
    n_prompt_tokens = 0
    for i, s in enumerate(seqs):
        p = synthetic.tokens(0, int(ctx[s]), cfg.vocab_size, stream=0xF100 + s)
        batch.prefill(i, p)
        n_prompt_tokens += len(p) - 1
    torch.cuda.synchronize()
    prefill_s = time.time() - t0
    log(f"[ours] c3: {per} sequences per GPU prefilled ({n_prompt_tokens} positions) in {prefill_s:.1f} s")
    batch.steps(W)
    stream = torch.cuda.ExternalStream(eng.stream_handle, device=torch.device("cuda", local))
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    bytes0 = batch.step_bytes()
    launches0 = bt.launch_count()
    clocks = ClockSampler(local)
    if pg:
        pg.barrier()
    torch.cuda.synchronize()
    clocks.start()
    ev0.record(stream)
    batch.steps(K, stream=eng.stream_handle)
    ev1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    launches = bt.launch_count() - launches0
    bytes1 = batch.step_bytes()
    ms = ev0.elapsed_time(ev1)
    if pg:
        t = torch.tensor([ms], device="cuda")
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms = float(t.item())
    value = n_total * K / (ms / 1000.0)
    bytes_avg = (bytes0 + bytes1) / 2.0 - 0.5 * 2 * cfg.num_layers * cfg.num_kv_heads * cfg.head_dim * 2 * per
    peak, peak_kind = hbm_peak()
    achieved = bytes_avg / (ms / K / 1000.0) / 1e9
    # end to end through the public API: each step's new token of every sequence read back to the host
    E = args.e2e_steps
    if pg:
        pg.barrier()
    torch.cuda.synchronize()
    te = time.perf_counter()
    for i in range(E):
        batch.steps(1)
        toks = batch.read_current()  # every sequence's new token, one copy per step
    e2e_s = time.perf_counter() - te
    if pg:
        t = torch.tensor([e2e_s], device="cuda")
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        e2e_s = float(t.item())
    if rank == 0:
        line = {
            "metric": "batched decode tokens/s and % HBM roofline (TinyLlama-1.1B shape, 64 sequences)",
            "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": ms / K, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "int8", "data": "synthetic",
            "config": {"workload": f"tinyllama-1.1b-shaped batched decode, {n_total} sequences, {per} per GPU",
                       "model": "tinyllama-1.1b", "global_batch": n_total, "contexts": "uniform [128, 4096]",
                       "kv_cache": f"fp16, paged ({P}-position pages)" if P else "fp16",
                       "parallelism": f"sequence-sharded x{world}",
                       "l2": "inputs larger than L2 (1.16 GB of weights + every sequence's KV per step)"},
            "roofline": {"kernel": "one batched step (GEMMs + attention), per GPU", "bound": "hbm",
                         "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_source": peak_kind, "bytes_per_step_per_gpu": bytes_avg},
            "e2e": {"value": n_total * E / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 4 * per, "api": "bt_batch_steps + bt_batch_read_current"},
            "prefill": {"positions_per_gpu": n_prompt_tokens, "seconds": prefill_s},
            "gpu_launches": launches, "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    batch.close()
    eng.close()
    if pg:
        pg.barrier()
        pg.destroy_process_group()
    return 0


def run_config_only(args):
    """One JSON line for the GEMV microbenchmark (--workload gemv: 4096 x 4096 int8, B in {1, 4,
    16}, HBM GB/s of the tile-layout GEMV at B = 1 as the value) or the tiny decoder (--workload
    tiny: 16-token prompt, 128 greedy steps, fp32 KV).  One GPU."""
    import torch
    import blocktensor_b200 as bt
    torch.cuda.set_device(0)

    def log(*a):
        print(*a, file=sys.stderr, flush=True)

    peak, peak_kind = hbm_peak()
    if args.workload == "gemv":
        res = c1_gemv(torch, bt, 0, log)
        head = next(r for r in res if r["B"] == 1 and r["kernel"].startswith("tcgen05 GEMV"))
        line = {"metric": "int8 dequant GEMV HBM GB/s (4096 x 4096, Q8_0 scales, B = 1; B = 4, 16 in rows)",
                "value": head["GBps"], "unit": "GB/s", "n_gpus": 1, "higher_is_better": True, "dtype": "int8",
                "data": "synthetic", "config": {"workload": "int8 GEMV 4096x4096, 16 weight copies cycled (302 MB)"},
                "roofline": {"bound": "hbm", "achieved": head["GBps"], "peak": peak, "unit": "GB/s",
                             "frac": head["GBps"] / peak, "peak_source": peak_kind}, "rows": res}
    else:
        res = c0_tiny(torch, bt, 0, log)
        line = {"metric": "decode tokens/s (tiny Llama-style decoder, batch 1)", "value": res["tokens_per_s"],
                "unit": "tokens/s", "n_gpus": 1, "higher_is_better": True, "dtype": "int8", "data": "synthetic",
                "config": {"workload": "tiny decoder D288 F768 L6 H6 V32000, 16-token prompt, 128 greedy steps, fp32 KV"},
                "roofline": {"bound": "hbm", "achieved": res["GBps"], "peak": peak, "unit": "GB/s",
                             "frac": res["frac_of_measured_hbm"], "peak_source": peak_kind}, "detail": res}
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--model", default="llama2-7b")
    ap.add_argument("--workload", choices=["decode", "batched", "gemv", "tiny"], default="decode",
                    help="decode: one sequence at batch 1 (the headline); batched: TinyLlama-shaped "
                         "batched decode of --sequences sequences sharded over the ranks")
    ap.add_argument("--sequences", type=int, default=64)
    ap.add_argument("--page-tokens", type=int, default=0,
                    help="batched workload: K/V in a page pool of pages of this many positions (0: contiguous)")
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--e2e-steps", type=int, default=64)
    ap.add_argument("--profile-steps", type=int, default=0,
                    help="also time the launch-per-operation step (per-kernel breakdown, diagnostic)")
    ap.add_argument("--no-prefill", action="store_true",
                    help="run the prompt one decode step per position instead of bt_engine_prefill")
    ap.add_argument("--no-diagnostics", action="store_true",
                    help="skip the GEMV microbenchmark and tiny-model lines of the diagnostics")
    ap.add_argument("--trace", action="store_true",
                    help="also record one step's per-phase device timestamps (diagnostic, untimed)")
    ap.add_argument("--replicas", action="store_true",
                    help="N > 1: N independent sequences (one per GPU) instead of tensor parallelism")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=0,
                    help="truncate the model to N layers (profiler captures; the JSON line is then marked)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "batched":
        return run_batched(args)
    if args.workload in ("gemv", "tiny"):
        return run_config_only(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())

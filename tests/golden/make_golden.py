"""Generates the golden fixtures in tests/golden/ from the reference's own code.

Run in a checkout where oracle/_ref/libbtref.so was built from the reference
sources (``make -C oracle``):

    python tests/golden/make_golden.py [--skip-7b]

* ref_kernels.npz  -- the deterministic ramps of the reference's tests
  (tests/test_stage3_kernels.cpp:49-204, test_stage4_quant.cpp:47-94,
  calc_numerical_errors.cpp:27-44, test_stage5_primitives.cpp:11-15,
  test_stage7_edge_cases.cpp:20-28) pushed through the reference library,
  plus bit-exact quantizer vectors (random and edge-case blocks).
* tiny_c0.npz      -- the tiny Llama-style config (D288 F768 L6 H6 hd48
  V32000, seed 0): 16 prompt ids and the greedy continuation, logits and
  per-layer residual taps, from the reference TransformerEngine (fp32 KV) and
  the bit-identical oracle restatement (fp16-KV variant, taps).
* llama7b_c2.npz   -- the 7B-shaped config (D4096 F11008 L32 H32 hd128 V32000,
  seed 0) with a short prompt: greedy tokens with fp32 KV (checked against
  the reference engine for the first steps) and with fp16 KV (restatement),
  top-2 logit margins, logits of one step and residual taps of a few layers.
* llama7b_c2_p512.npz -- the same model at the benchmarked configuration: a
  512-token prompt and 32 greedy tokens (contexts up to 544), fp16 and fp32 KV,
  with logits and taps of a few layers at the last prompt position and at the
  last generated position.  The restatement runs multithreaded (rows of each
  matvec split between threads, every row summed in the reference's order, so
  the results do not depend on the thread count) and is checked against the
  reference engine on the first positions.
"""
from __future__ import annotations

import argparse
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402

C = O.C


def _fp(a):
    return a.ctypes.data_as(C.c_void_p)


def ramp(n, mod, a, b):
    """static_cast<float>(i % mod) * a - b evaluated in float, as the reference tests do."""
    return (np.arange(n) % mod).astype(np.float32) * np.float32(a) - np.float32(b)


def ref_kernels(ref: O.RefLib):
    out = {}
    # rmsnorm 4x512 (test_stage3_kernels.cpp:51-58)
    x = ramp(4 * 512, 100, 0.1, 5.0)
    w = np.float32(1.0) + (np.arange(512) % 10).astype(np.float32) * np.float32(0.05)
    y = np.zeros_like(x)
    ref.btr_rmsnorm(_fp(x), _fp(w), _fp(y), 4, 512, 1e-5)
    out.update(rms_x=x, rms_w=w, rms_y=y)
    # rope seq 2 x 4 heads x hd 64 (test_stage3_kernels.cpp:93-103), pos 0 as in the
    # test and two later positions
    x = ramp(2 * 4 * 64, 30, 0.2, 3.0)
    out["rope_x"] = x
    for pos in (0, 7, 300):
        y = np.zeros_like(x)
        ref.btr_rope(_fp(x), _fp(y), 2, 4, 64, pos)
        out[f"rope_y_pos{pos}"] = y
    # softmax 4x256 (:134-141)
    x = ramp(4 * 256, 50, 0.1, 2.5)
    y = np.zeros_like(x)
    ref.btr_softmax(_fp(x), _fp(y), 4, 256)
    out.update(softmax_x=x, softmax_y=y)
    # silu 1024 (:171-177)
    x = ramp(1024, 100, 0.1, 5.0)
    y = np.zeros_like(x)
    ref.btr_silu(_fp(x), _fp(y), 1024)
    out.update(silu_x=x, silu_y=y)
    # Q8_0 matvec 16x256 (test_stage4_quant.cpp:49-66) and its error vs fp32
    # (calc_numerical_errors.cpp:27-44)
    raw = ramp(16 * 256, 50, 0.1, 2.5)
    xv = ramp(256, 20, 0.15, 1.5)
    blocks = ref.quantize_q8_0(raw)
    yq = ref.matvec_q8_0(blocks, xv, 16, 256)
    yf = np.zeros(16, np.float32)
    for r in range(16):  # float accumulation in the order of calc_numerical_errors.cpp:31-33
        acc = np.float32(0.0)
        for c in range(256):
            acc = np.float32(acc + np.float32(raw[r * 256 + c] * xv[c]))
        yf[r] = acc
    err = np.abs(yf - yq)
    out.update(mv_raw=raw, mv_x=xv, mv_blocks=blocks.view(np.uint8), mv_y=yq,
               mv_err_max=np.float32(err.max()), mv_err_mean=np.float32(err.sum(dtype=np.float32) / np.float32(16)))
    # greedy (test_stage5_primitives.cpp:11-15)
    lg = np.array([1.0, 2.5, 0.1, 10.0, -3.0], np.float32)
    out["greedy_logits"] = lg
    out["greedy_id"] = np.uint32(ref.btr_sample_greedy(_fp(lg), 5))
    # quantizer vectors: seeded normal data, uniform data, and edge-case blocks
    rng = np.random.default_rng(1234)
    qn = (rng.standard_normal(32 * 512) * 0.05).astype(np.float32)
    qu = rng.uniform(-3, 3, 32 * 256).astype(np.float32)
    s = np.float32(2.0 ** -6)
    half_way = np.array([127, 0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 3.5, 126.5, -126.5, 63.5, -63.5, 0.25, 0.75, -0.75, 1.0]
                        + [k + 0.5 for k in range(16)], np.float32) * s
    zeros = np.zeros(32, np.float32)
    neg_zero = -np.zeros(32, np.float32)
    tiny = np.full(32, 1e-39, np.float32)        # subnormal block: scale subnormal, inv = inf
    tiny[1] = 0.0
    tiny[2] = -1e-39
    big = np.linspace(-3e38, 3e38, 32).astype(np.float32)
    single = np.zeros(32, np.float32)
    single[5] = -7.25
    mixed = np.array([(-1) ** i * (i + 1) * 1e-3 for i in range(32)], np.float32)
    edge = np.concatenate([half_way, zeros, neg_zero, tiny, big, single, mixed])
    for name, v in (("qn", qn), ("qu", qu), ("qedge", edge)):
        out[f"{name}_x"] = v
        out[f"{name}_blocks"] = ref.quantize_q8_0(v).view(np.uint8)
        deq = np.zeros(v.size, np.float32)
        b = ref.quantize_q8_0(v)
        ref.btr_dequantize_q8_0(_fp(b), _fp(deq), v.size)
        out[f"{name}_deq"] = deq
    # zero-block edge case (test_stage7_edge_cases.cpp:20-28)
    zb = ref.quantize_q8_0(np.zeros(32, np.float32))
    out["zero_scale"] = np.float32(zb["scale"][0])
    return out


def tiny_c0(ref: O.RefLib, n_gen: int = 128):
    cfg = O.make_config(32000, 288, 768, 6, 6, 6, 48, 256)
    m = O.Model(cfg, seed=0)
    prompt = O.gen_tokens(0, O.STREAM_PROMPT, 16, cfg.vocab_size)
    eng = O.RefEngine(ref, m, kv_max_seq=256)
    kv32 = O.KV(cfg, 256, fp16=False)
    kv16 = O.KV(cfg, 256, fp16=True)
    toks = [int(prompt[0])]
    toks16 = [int(prompt[0])]
    logits_keep, taps_keep, taps16_keep, margins = {}, {}, {}, []
    keep_pos = (0, 15, 16, 47, 143)
    for p in range(16 + n_gen):
        t = toks[p]
        lr = eng.forward(t, p)
        lo, taps = O.forward_token(m, kv32, t, p, want_taps=True)
        assert np.array_equal(lr, lo), f"oracle restatement differs from reference at pos {p}"
        l16, taps16 = O.forward_token(m, kv16, toks16[p], p, want_taps=True)
        srt = np.sort(lr)
        margins.append(srt[-1] - srt[-2])
        if p in keep_pos:
            logits_keep[p] = lr
            taps_keep[p] = taps
            taps16_keep[p] = taps16
        nxt = int(prompt[p + 1]) if p + 1 < 16 else O.sample_greedy(lr)
        nxt16 = int(prompt[p + 1]) if p + 1 < 16 else O.sample_greedy(l16)
        toks.append(nxt)
        toks16.append(nxt16)
    k_l0, v_l0 = kv32.layer(0)
    out = dict(config=np.frombuffer(bytes(cfg), np.uint8), prompt=prompt, tokens=np.array(toks, np.uint32),
               tokens_kv16=np.array(toks16, np.uint32), margins=np.array(margins, np.float32),
               keep_pos=np.array(keep_pos, np.int32),
               kv_l0_k=k_l0[: (16 + n_gen) * 288], kv_l0_v=v_l0[: (16 + n_gen) * 288])
    for p in keep_pos:
        out[f"logits_p{p}"] = logits_keep[p]
        out[f"taps_p{p}"] = taps_keep[p]
        out[f"taps16_p{p}"] = taps16_keep[p]
    return out


def llama7b(ref: O.RefLib, n_prompt: int = 8, n_gen: int = 32, ref_steps: int = 2):
    cfg = O.make_config(32000, 4096, 11008, 32, 32, 32, 128, 1024)
    t0 = time.time()
    m = O.Model(cfg, seed=0)
    print(f"  7B model generated in {time.time() - t0:.1f} s", flush=True)
    prompt = O.gen_tokens(0, O.STREAM_PROMPT, n_prompt, cfg.vocab_size)
    max_seq = n_prompt + n_gen + 1
    out = dict(config=np.frombuffer(bytes(cfg), np.uint8), prompt=prompt)
    eng = O.RefEngine(ref, m, kv_max_seq=max_seq) if ref_steps else None
    for name, fp16 in (("kv32", False), ("kv16", True)):
        kv = O.KV(cfg, max_seq, fp16=fp16)
        toks = [int(prompt[0])]
        margins, top = [], []
        t0 = time.time()
        for p in range(n_prompt + n_gen):
            lo, taps = O.forward_token(m, kv, toks[p], p, want_taps=True)
            if eng is not None and not fp16 and p < ref_steps:
                lr = eng.forward(toks[p], p)
                assert np.array_equal(lr, lo), f"oracle differs from reference engine at 7B pos {p}"
            srt = np.argsort(lo)[::-1]
            margins.append(lo[srt[0]] - lo[srt[1]])
            top.append(srt[:8].astype(np.uint32))
            if p == n_prompt - 1:
                out[f"{name}_logits_last_prompt"] = lo
                out[f"{name}_taps_last_prompt"] = taps[[0, 1, 15, 31]]
                out[f"{name}_tap_norms_last_prompt"] = np.linalg.norm(taps, axis=1).astype(np.float32)
            nxt = int(prompt[p + 1]) if p + 1 < n_prompt else int(srt[0])
            toks.append(nxt)
        print(f"  7B {name}: {n_prompt + n_gen} steps in {time.time() - t0:.1f} s", flush=True)
        out[f"{name}_tokens"] = np.array(toks, np.uint32)
        out[f"{name}_margins"] = np.array(margins, np.float32)
        out[f"{name}_top8"] = np.stack(top)
        kv.close()
    if eng is not None:
        eng.close()
    m.close()
    return out


def llama7b_long(ref: O.RefLib, n_prompt: int = 512, n_gen: int = 32, ref_steps: int = 2):
    cfg = O.make_config(32000, 4096, 11008, 32, 32, 32, 128, 1024)
    t0 = time.time()
    m = O.Model(cfg, seed=0)
    print(f"  7B model generated in {time.time() - t0:.1f} s", flush=True)
    prompt = O.gen_tokens(0, O.STREAM_PROMPT, n_prompt, cfg.vocab_size)
    max_seq = n_prompt + n_gen + 1
    layers = [0, 1, 15, 31]
    out = dict(config=np.frombuffer(bytes(cfg), np.uint8), prompt=prompt, tap_layers=np.array(layers, np.int32))
    eng = O.RefEngine(ref, m, kv_max_seq=max_seq) if ref_steps else None
    for name, fp16 in (("kv16", True), ("kv32", False)):
        kv = O.KV(cfg, max_seq, fp16=fp16)
        toks = [int(prompt[0])]
        margins, top = [], []
        t0 = time.time()
        for p in range(n_prompt + n_gen):
            lo, taps = O.forward_token(m, kv, toks[p], p, want_taps=True)
            if eng is not None and not fp16 and p < ref_steps:
                lr = eng.forward(toks[p], p)
                assert np.array_equal(lr, lo), f"oracle differs from reference engine at 7B pos {p}"
            srt = np.argsort(lo)[::-1]
            margins.append(lo[srt[0]] - lo[srt[1]])
            top.append(srt[:8].astype(np.uint32))
            for tag, at in (("last_prompt", n_prompt - 1), ("last_gen", n_prompt + n_gen - 1)):
                if p == at:
                    out[f"{name}_logits_{tag}"] = lo
                    out[f"{name}_taps_{tag}"] = taps[layers]
                    out[f"{name}_tap_norms_{tag}"] = np.linalg.norm(taps, axis=1).astype(np.float32)
            nxt = int(prompt[p + 1]) if p + 1 < n_prompt else int(srt[0])
            toks.append(nxt)
            if p % 64 == 63:
                print(f"  7B {name}: {p + 1} steps, {time.time() - t0:.0f} s", flush=True)
        out[f"{name}_tokens"] = np.array(toks, np.uint32)
        out[f"{name}_margins"] = np.array(margins, np.float32)
        out[f"{name}_top8"] = np.stack(top)
        kv.close()
    if eng is not None:
        eng.close()
    m.close()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--skip-7b", action="store_true")
    ap.add_argument("--only-7b-long", action="store_true",
                    help="write only llama7b_c2_p512.npz (the benchmarked 512-token configuration)")
    a = ap.parse_args()
    ref = O.RefLib()
    if a.only_7b_long:
        np.savez_compressed(os.path.join(HERE, "llama7b_c2_p512.npz"), **llama7b_long(ref))
        print("llama7b_c2_p512.npz written")
        return
    np.savez_compressed(os.path.join(HERE, "ref_kernels.npz"), **ref_kernels(ref))
    print("ref_kernels.npz written")
    np.savez_compressed(os.path.join(HERE, "tiny_c0.npz"), **tiny_c0(ref))
    print("tiny_c0.npz written")
    if not a.skip_7b:
        np.savez_compressed(os.path.join(HERE, "llama7b_c2.npz"), **llama7b(ref))
        print("llama7b_c2.npz written")
        np.savez_compressed(os.path.join(HERE, "llama7b_c2_p512.npz"), **llama7b_long(ref))
        print("llama7b_c2_p512.npz written")


if __name__ == "__main__":
    main()

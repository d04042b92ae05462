"""Per-stage timeline of one decode step (a library built with BT_STAGE_TRACE).

``python -m blocktensor_b200.build --define BT_STAGE_TRACE`` builds the step
kernel with timestamps on every ring stage of every CTA (the first 2048 stages
of the step): [0] the producer issues the stage's copy, [1] issuer 1 sees it
landed, [4] issuer 1 has issued and committed its MMAs, [5] accumulator warp 5
starts waiting for the MMAs, [2] it sees them complete, [3] it has read the
sums and releases the stage, [7] it has formed the stage's digit sums, [6] it
has added them.  Then

    python -m blocktensor_b200.stage_trace [--model llama2-7b] [--layer 10] [--phase gateup] [--cta 0]

decodes a 512-token prompt's next tokens on the synthetic model and prints,
for one CTA and one GEMV phase, each stage's stamps relative to the phase
start and the medians of the intervals between them.  Rebuild without the
define afterwards: the stamps slow the step.
"""
from __future__ import annotations

import argparse

import numpy as np

STAGE_TRACE_MAX = 2048  # stages stamped per CTA (kStageTraceMax)
STAGE_SLOTS = 8         # stamps per stage (kStageSlots)
PHASES = ["qkv", "attention", "oproj", "gateup", "down"]


def capture(model: str = "llama2-7b", prompt: int = 512, warm: int = 6):
    import torch

    import blocktensor_b200 as bt
    from blocktensor_b200 import synthetic

    max_seq = prompt + warm + 8
    cfg = synthetic.config(model, max_seq)
    eng = bt.TransformerEngine(cfg, rope_theta=synthetic.ROPE_THETA[model])
    eng.generate(seed=0, sigma=0.02)
    kv = bt.KVCache(eng, max_seq, bt.BT_KV_FP16)
    eng.prefill(kv, synthetic.tokens(0, prompt, cfg.vocab_size))
    eng.steps(kv, warm)
    torch.cuda.synchronize()
    eng.set_trace(True)
    eng.steps(kv, 1)
    torch.cuda.synchronize()
    G = eng.num_sms
    P = 5 * cfg.num_layers + 1
    n = P * G * 8 + G * STAGE_TRACE_MAX * STAGE_SLOTS
    buf = np.zeros(n, np.uint64)
    bt.native.check(bt.load().bt_engine_read_trace(eng.handle, buf.ctypes.data, n))
    eng.set_trace(False)
    kv.close()
    eng.close()
    return buf[: P * G * 8].reshape(P, G, 8), buf[P * G * 8:].reshape(G, STAGE_TRACE_MAX, STAGE_SLOTS)


def summarize(phase: np.ndarray, stage: np.ndarray, layer: int, kind: str, cta: int) -> str:
    p = 5 * layer + PHASES.index(kind)
    ph = phase.astype(np.int64)
    st = stage[cta].astype(np.int64)
    a, e = ph[p, cta, 0], ph[p, cta, 3]
    idx = np.nonzero((st[:, 2] >= a) & (st[:, 2] <= e))[0]
    lines = [f"CTA {cta}, layer {layer} {kind}: {len(idx)} stages, phase {(e - a) / 1e3:.2f} us (us from the phase start)",
             "stage    copy   landed  issued  accwait  seen  released  sums  added"]
    for i in idx:
        cp, land, seen, rel, iss, w0, w1, w7 = (st[i] - a) / 1e3
        lines.append(f"{i:5d} {cp:8.2f} {land:7.2f} {iss:7.2f} {w0:7.2f} {seen:7.2f} {rel:7.2f} {w7:7.2f} {w1:7.2f}")
    if len(idx) > 2:
        s = st[idx]
        med = lambda v: float(np.median(v)) / 1e3  # noqa: E731
        lines.append(
            f"medians (us): release to release {med(np.diff(s[:, 3])):.2f}, copy to landed {med(s[:, 1] - s[:, 0]):.2f}, "
            f"landed to issued {med(s[:, 4] - s[:, 1]):.2f}, wait {med(s[:, 2] - s[:, 5]):.2f}, "
            f"read + release {med(s[:, 3] - s[:, 2]):.2f}, sums {med(s[:, 7] - s[:, 3]):.2f}, "
            f"adds {med(s[:, 6] - s[:, 7]):.2f}")
    return "\n".join(lines)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--model", default="llama2-7b")
    ap.add_argument("--layer", type=int, default=10)
    ap.add_argument("--phase", choices=[k for k in PHASES if k != "attention"], default="gateup")
    ap.add_argument("--cta", type=int, default=0)
    a = ap.parse_args()
    phase, stage = capture(a.model)
    print(summarize(phase, stage, a.layer, a.phase, a.cta))


if __name__ == "__main__":
    main()

"""CPU: host-side logic (synthetic workload spec, .btmodel format, byte accounting)."""
import numpy as np
import pytest

from blocktensor_b200 import btmodel, synthetic


def test_tokens_match_oracle_generator(oracle):
    for seed in (0, 1, 7):
        assert np.array_equal(synthetic.tokens(seed, 700, 32000), oracle.gen_tokens(seed, oracle.STREAM_PROMPT, 700, 32000))


def test_normal_matches_oracle_generator(oracle):
    a = synthetic.normal(3, 16 + 2, 5000, 0.02, offset=123)
    b = oracle.gen_normal(3, 16 + 2, 5000, 0.02, offset=123)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_step_bytes_7b():
    """7B int8: 6.607 G params -> 7.433 GB of weights; KV fp16 at c=640 adds 2*32*640*4096*2 B."""
    cfg = synthetic.config("llama2-7b", 1024)
    wb = synthetic.weight_bytes(cfg)
    assert abs(wb / 1e9 - 7.433) < 0.001
    b = synthetic.step_bytes(cfg, 640, 2)
    assert b - wb == 4 * 4096 * 65 + 4 * 4096 + 2 * 32 * 4096 * 2 * 641


def test_btmodel_roundtrip(tmp_path, oracle):
    cfg = oracle.make_config(50, 32, 64, 1, 2, 2, 16, 8)
    m = oracle.Model(cfg, seed=1)
    ts = [m.tensor_array(t).view(np.uint8) for t in m.tensors()]
    p = str(tmp_path / "a.btmodel")
    btmodel.write_btmodel(p, cfg, ts)
    r = btmodel.read_btmodel(p)
    assert bytes(r.config) == bytes(cfg)
    assert all(np.array_equal(a, b) for a, b in zip(r.tensors, ts))
    assert [t.nbytes for t in r.tensors] == r.expected_sizes()


def test_btmodel_truncated(tmp_path, oracle):
    cfg = oracle.make_config(50, 32, 64, 1, 2, 2, 16, 8)
    m = oracle.Model(cfg, seed=1)
    p = tmp_path / "t.btmodel"
    btmodel.write_btmodel(str(p), cfg, [m.tensor_array(t).view(np.uint8) for t in m.tensors()])
    data = p.read_bytes()
    p.write_bytes(data[:-10])
    with pytest.raises(RuntimeError):
        btmodel.read_btmodel(str(p))


def test_stage_trace_summary():
    """The stage-timeline summary picks the stages whose MMAs the accumulator saw inside the
    phase and reports the intervals between the stamps (synthetic stamps, no GPU)."""
    import numpy as np

    from blocktensor_b200 import stage_trace as st

    L, G = 12, 2
    phase = np.zeros((5 * L + 1, G, 8), np.uint64)
    stage = np.zeros((G, st.STAGE_TRACE_MAX, st.STAGE_SLOTS), np.uint64)
    p = 5 * 10 + st.PHASES.index("gateup")
    t0 = 1_000_000
    phase[p, 0, 0], phase[p, 0, 3] = t0, t0 + 10_000
    for i in range(4):  # stages 100..103, one every 700 ns
        b = t0 + 1_000 + 700 * i
        # copy, landed, seen, released, issued, wait start, added, sums
        stage[0, 100 + i] = [b - 2_000, b - 500, b + 130, b + 290, b - 240, b, b + 580, b + 450]
    stage[0, 99, 2] = t0 - 5  # seen before the phase: not one of its stages
    out = st.summarize(phase, stage, 10, "gateup", 0)
    lines = out.splitlines()
    assert lines[0].startswith("CTA 0, layer 10 gateup: 4 stages, phase 10.00 us")
    assert len(lines) == 2 + 4 + 1
    assert "release to release 0.70" in lines[-1]
    assert "wait 0.13" in lines[-1] and "adds 0.13" in lines[-1]


def test_phase_trace_summary():
    """bench.py's per-phase summary of a step trace: durations, counter waits and tails from
    synthetic stamps (every phase 10 us, CTAs passing their wait 1 us after the previous end,
    the last CTA ending 2 us after the median one)."""
    import importlib.util
    import os

    import numpy as np

    spec = importlib.util.spec_from_file_location("bench", os.path.join(os.path.dirname(__file__), "..", "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    L, G = 4, 3
    P = 5 * L + 1
    tr = np.zeros((P, G, 8), np.uint64)
    for p in range(P):
        base = 1_000_000 + 10_000 * p
        for c in range(G):
            tr[p, c, 0] = base + 1_000                # passed the counter wait
            tr[p, c, 1] = base + 2_000                # digits in shared memory
            tr[p, c, 2] = base + 3_000                # first row tile's sums
            tr[p, c, 3] = base + 8_000 + (2_000 if c == G - 1 else 0)  # end: the last CTA 2 us later
            tr[p, c, 4] = base - 20_000               # first copy of the phase
    res = bench.trace_summary(tr, L)
    for k in ("qkv", "oproj", "gateup", "down"):
        assert res[k]["dur"] == 10.0 and res[k]["wait"] == 1.0
        assert res[k]["digits"] == 1.0 and res[k]["first"] == 1.0 and res[k]["tail"] == 2.0
    assert res["step_us"] == round((float(tr[:, :, 3].max()) - float(tr[:, :, 0].min())) / 1000.0, 1)

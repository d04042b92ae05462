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

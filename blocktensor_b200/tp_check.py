"""Tensor-parallel decode against the single-GPU engine, one process per GPU.

Run under torchrun (``python -m torch.distributed.run --nproc-per-node W
--master-addr 127.0.0.1 --master-port P -m blocktensor_b200.tp_check OUT.json
[mha|gqa]``).
Every rank builds its share of the same synthetic model, the ranks exchange
their handles over a gloo process group and decode a prompt plus greedy
tokens; rank 0 then decodes the same sequence with the whole model on its
GPU and writes both token lists and the per-layer activation error of the
last step to OUT.json.
"""
from __future__ import annotations

import datetime
import json
import os
import sys

import numpy as np

# D 512, 8 heads of 64, FFN 1536, 4 layers, vocab 4096: every rank holds whole
# heads and whole 32-blocks at 2, 4 and 8 GPUs ("mha": 8 KV heads); "gqa": 4
# KV heads, 2 query heads per KV head on every rank (2 and 4 GPUs)
CONFIGS = {
    "mha": dict(vocab=4096, dim=512, hidden=1536, layers=4, heads=8, kv_heads=8, head_dim=64, max_seq=128),
    "gqa": dict(vocab=4096, dim=512, hidden=1536, layers=4, heads=8, kv_heads=4, head_dim=64, max_seq=128),
}
PROMPT = [17, 3051, 999, 2, 4000, 123, 77, 1024]
N_GEN = 40


def main(out_path: str, shape: str = "mha") -> int:
    import torch
    import torch.distributed as dist

    import blocktensor_b200 as bt
    from blocktensor_b200 import tp

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    c = CONFIGS[shape]
    cfg = bt.model_config(c["vocab"], c["dim"], c["hidden"], c["layers"], c["heads"], c["kv_heads"],
                          c["head_dim"], c["max_seq"])
    eng = bt.TransformerEngine(cfg, device=local, tp_rank=rank, tp_world=world)
    eng.generate(seed=0, sigma=0.02)
    tp.connect(eng)
    kv = bt.KVCache(eng, c["max_seq"], bt.BT_KV_FP32)
    eng.set_taps(True)
    got = eng.decode(kv, PROMPT, n_gen=N_GEN)
    taps = eng.read_taps()
    dist.barrier()
    rc = 0
    if rank == 0:
        ref = bt.TransformerEngine(cfg, device=local)
        ref.generate(seed=0, sigma=0.02)
        kv1 = bt.KVCache(ref, c["max_seq"], bt.BT_KV_FP32)
        ref.set_taps(True)
        want = ref.decode(kv1, PROMPT, n_gen=N_GEN)
        rtaps = ref.read_taps()
        err = np.abs(taps.astype(np.float64) - rtaps) / (1.0 + np.abs(rtaps))
        with open(out_path, "w") as f:
            json.dump({"world": world, "tokens": [int(t) for t in got], "want": [int(t) for t in want],
                       "tap_err_max": float(err.max())}, f)
        kv1.close()
        ref.close()
    dist.barrier()
    kv.close()
    eng.close()
    dist.destroy_process_group()
    return rc


if __name__ == "__main__":
    sys.exit(main(sys.argv[1], sys.argv[2] if len(sys.argv) > 2 else "mha"))

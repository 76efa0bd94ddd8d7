"""The small synthetic generation run shared by the scheduler's GPU tests
(tests/test_gpu_sched.py, tests/test_gpu_sched_ranks.py and their NCCL rank
worker): a 2-layer synthetic decoder with int8 KV, the default attribute
windows and the device lane streams and sampler.  With fixed attention
splits and the same number of batch rows on every shard, a lane's records
do not depend on which shard, stream or GPU runs it."""
from __future__ import annotations

COSTS = [300, 17, 1000, 64, 512, 5, 700, 128]
BUDGETS = [3, 5, 2, 4, 6, 1, 3, 5]
ROWS = 8
SPLIT = 128
SEED = 2024


def scheduler(pp, costs=COSTS, budgets=BUDGETS, rows=ROWS, split=SPLIT):
    D, sched = pp.decoder, pp.sched
    cfg = D.DecoderConfig(layers=2, width=256, heads=2, head_dim=128, ffn_hidden=512, max_context=1024)
    w = sched.default_windows()
    cap = max(costs) + max(budgets) + 4

    def make_model(shard, lanes, device):
        return sched.SyntheticPrimitiveModel(cfg, rows, lanes, [costs[ln] for ln in lanes], cap, device, w, seed=5,
                                             split_tokens=split)

    return sched.BranchScheduler(make_model, costs, SEED, budgets, w)

"""Worker for test_vocab_parallel_multi_gpu: one rank per GPU, NCCL, column slices of the rows.

Every rank builds the same full logits, keeps its contiguous column slice, samples through
sample_tokens_vocab_parallel, and checks the tokens against sample_tokens on the full rows.
Exit status 0 when every rank agrees with the full-row result.
"""

import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from pagedbatch_b200 import SamplingParams, sample_tokens, workloads  # noqa: E402
from pagedbatch_b200.vocab_parallel import sample_tokens_vocab_parallel  # noqa: E402


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=120))
    ok = True
    try:
        w = workloads.config3(rows=256)
        w1 = workloads.config1(rows=64)
        cases = [(w.logits, w.params), (w1.logits, w1.params)]
        # both shard kernels: the default choice for these sizes, and the streaming kernel forced
        for path in (None, "stream"):
            if path:
                os.environ["PB_PATH"] = path
            for logits, params in cases:
                V = logits.shape[1]
                lo, hi = V * rank // world, V * (rank + 1) // world
                x = logits.cuda()
                local = x[:, lo:hi].contiguous()
                gens = [torch.Generator().manual_seed(i) for i in range(len(params))]
                got = sample_tokens_vocab_parallel(local, params, gens)
                gens = [torch.Generator().manual_seed(i) for i in range(len(params))]
                want = sample_tokens(x, params, gens)
                if got != want:
                    bad = [i for i in range(len(got)) if got[i] != want[i]]
                    print(f"rank {rank} ({path}): {len(bad)} rows differ, first {bad[:5]}", flush=True)
                    ok = False
            os.environ.pop("PB_PATH", None)
        flag = torch.tensor([0 if ok else 1], device="cuda")
        dist.all_reduce(flag)
        ok = int(flag.item()) == 0
    finally:
        dist.destroy_process_group()
    if rank == 0:
        print("vocab-parallel", "OK" if ok else "MISMATCH", f"on {world} GPUs", flush=True)
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()

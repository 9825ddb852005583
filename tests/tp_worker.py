"""Two-GPU check of the tensor-parallel batched decoder, launched by
tests/test_batch_tp.py under torch.distributed.run (one process per GPU).

Both ranks build their shard of the same host model; rank 0 also runs the
unsharded batch on its GPU.  The sharded run's logits (gathered from the
ranks' vocabulary slices) must match the unsharded run's within the
reduction-order tolerance, step by step, and its ids must follow them."""
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import nutllm_b200 as nb  # noqa: E402
from nutllm_b200 import synthetic as syn  # noqa: E402


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    cfg = nb.Config(layers=2, heads=8, dim=256, head_dim=32, ffn_dim=512, vocab_size=1000,
                    max_seq=64, eos_token=1, kv_heads=2)
    w = syn.build_model(cfg, 1, 21)
    B, n, steps = 4, 5, 6
    prompts = np.stack([syn.prompt_ids(cfg, 300 + b, n) for b in range(B)])
    idb = [nb.tp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(idb, src=0)
    tp = nb.TPBatch(B, rank=rank, world=world, nccl_id=idb[0], weights=w, device=local)
    ids, logits, _ = tp.generate(prompts, steps, want_logits=True)
    parts = [None] * world
    dist.all_gather_object(parts, (tp.info()["vocab0"], logits))
    # the same run with the Wo / Wdown sums through peer memory, with and
    # without graph replay
    handles = [None] * world
    dist.all_gather_object(handles, tp.ipc_handle())
    tp.open_peers(handles)
    ids_p, logits_p, _ = tp.generate(prompts, steps, want_logits=True)
    ids_g, _, _ = tp.generate(prompts, steps)
    parts_p = [None] * world
    dist.all_gather_object(parts_p, (tp.info()["vocab0"], logits_p))
    tp.close()
    if rank == 0:
        full = np.concatenate([p[1] for p in sorted(parts, key=lambda x: x[0])], axis=2)
        one = nb.TPBatch(B, weights=w, device=local)
        ids1, logits1, _ = one.generate(prompts, steps, want_logits=True)
        one.close()
        d = np.abs(full - logits1)
        assert np.all(d <= 1e-3 + 1e-3 * np.abs(logits1)), float(d.max())
        assert ids.tolist() == [[int(np.argmax(full[k, b])) for k in range(steps)]
                                for b in range(B)]
        full_p = np.concatenate([p[1] for p in sorted(parts_p, key=lambda x: x[0])], axis=2)
        dp = np.abs(full_p - logits1)
        assert np.all(dp <= 1e-3 + 1e-3 * np.abs(logits1)), float(dp.max())
        assert ids_p.tolist() == ids_g.tolist() == [
            [int(np.argmax(full_p[k, b])) for k in range(steps)] for b in range(B)]
        print(f"peer all-reduce matches: max |diff| {float(dp.max()):.2e}")
        print(f"tensor parallel matches: max |diff| {float(d.max()):.2e}, "
              f"ids equal to one rank: {ids.tolist() == ids1.tolist()}")
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()

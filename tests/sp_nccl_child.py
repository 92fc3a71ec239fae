"""One rank of the two-GPU sequence-parallel check (launched by tests/test_sp_gpu.py through
torch.distributed.run): mk_forward_sp over NCCL (key split off) must give rank 0 the same bits as mk_forward
on one GPU."""
import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    from minicpm5_mk import mk_weights, sp
    from minicpm5_mk.mk_config import get_config
    from minicpm5_mk.mk_init import random_state_dict, synthetic_ids
    from minicpm5_mk.ops import MkEngine

    cfg = get_config("minicpm5-1b").replace(max_seq=8192)
    eng = MkEngine(cfg, mk_weights.prepare_mk_weights(random_state_dict(cfg, seed=1234, device=dev), cfg), dev)
    eng.set_sp_key_split(False)  # one attention CTA per query block: the same bits as the one-GPU forward
    ids = synthetic_ids(1, 8192, seed=1234).reshape(-1).contiguous().to(dev)
    h1, l1, t1 = eng.forward_sp(ids, 8192, rank, world, sp.nccl_allgather())
    torch.cuda.synchronize()
    ok = True
    if rank == 0:
        h1, l1, t1 = h1.clone(), l1.clone(), t1.clone()
        h0, l0, t0 = eng.forward(ids, 1, 8192)
        torch.cuda.synchronize()
        ok = torch.equal(t0, t1) and torch.equal(l0, l1) and torch.equal(h0, h1)
        print("rank0 top1", int(t0[0]), int(t1[0]), "max |dlogit|", float((l0 - l1).abs().max()), flush=True)
    flag = torch.tensor([1 if ok and eng.check_device_error() == 0 else 0], device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    all_ok = int(flag.item()) == 1
    dist.destroy_process_group()
    if rank == 0 and all_ok:
        print("SP_NCCL_OK", flush=True)
    sys.exit(0 if all_ok else 1)


if __name__ == "__main__":
    main()

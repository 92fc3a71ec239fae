import os, torch, torch.distributed as dist, torch.multiprocessing as mp
def run(rank):
    os.environ["MASTER_ADDR"]="127.0.0.1"; os.environ["MASTER_PORT"]="29533"
    dist.init_process_group("gloo", rank=rank, world_size=2)
    a = torch.full((4,), rank, dtype=torch.uint8); out = torch.empty(8, dtype=torch.uint8)
    dist.all_gather_into_tensor(out, a)
    print(rank, out.tolist())
    dist.destroy_process_group()
if __name__ == "__main__":
    mp.spawn(run, nprocs=2)

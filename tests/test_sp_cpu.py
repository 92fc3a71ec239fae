"""Sequence parallelism, host side: the zig-zag block arithmetic (Python mirror and the CUDA header's
sp_pos / sp_row compiled for the host) against the reference's `sp_global_block`, and the all-gather
callback with 2 gloo ranks on CPU."""
import os
import socket
import subprocess

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from minicpm5_mk import sp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "minicpm5-vllm-tpu_b200", "csrc")


def ref_sp_global_block(i, r):
    """Restatement of sp_global_block (plugin/minicpm5_mk/mk_attn.py:721-724): zig-zag over groups of
    4 blocks for the 2 TensorCores."""
    j = i % 2
    return 4 * (i // 2) + j * (3 - r) + (1 - j) * r


def test_world2_matches_reference_zigzag():
    nb = 8192 // 512
    for r in range(2):
        assert [sp.global_block(i, r, 2) for i in range(nb // 2)] == [ref_sp_global_block(i, r) for i in range(nb // 2)]


@pytest.mark.parametrize("seq,world", [(8192, 1), (8192, 2), (8192, 4), (8192, 8), (2048, 2), (1024, 4)])
def test_layout_partitions_and_round_trips(seq, world):
    blk = sp.sp_block(seq, world, 16, 2)
    assert blk > 0
    n = seq // world
    seen = torch.zeros(seq, dtype=torch.int64)
    work = []
    for r in range(world):
        pos = sp.local_positions(seq, blk, r, world)
        assert pos.tolist() == [sp.sp_pos(i, blk, r, world) for i in range(n)]
        assert torch.all(pos[1:] > pos[:-1])  # a rank's rows stay in sequence order
        seen[pos] += 1
        for i in range(0, n, 37):
            assert sp.sp_row(int(pos[i]), blk, world, n) == r * n + i
        work.append(int((pos + 1).sum()))  # causal attention work of the rank's queries
    assert torch.all(seen == 1)
    assert max(work) - min(work) <= blk * blk * world  # balanced up to one block pair


def test_sp_block_choice():
    assert sp.sp_block(8192, 2, 16, 2) == 512
    assert sp.sp_block(8192, 8, 16, 2) == 512
    assert sp.sp_block(1024, 2, 4, 2) == 256
    assert sp.sp_block(1024, 4, 4, 2) == 128
    assert sp.sp_block(1024, 8, 4, 2) == 0  # 64-token blocks cannot hold a 128-row query block at G = 2
    assert sp.sp_block(384, 2, 16, 2) == 0


def test_cuda_header_layout_matches_python(tmp_path):
    """sp_pos / sp_row of csrc/mk_common.cuh, compiled for the host with nvcc, give the Python mirror's
    values."""
    src = tmp_path / "sp_host.cu"
    src.write_text(f'''#include "{CSRC}/mk_common.cuh"
#include <cstdio>
int main() {{
  const int cases[][3] = {{{{8192, 2, 512}}, {{8192, 8, 512}}, {{2048, 2, 512}}, {{1024, 4, 128}}}};
  for (const auto& c : cases)
    for (int r = 0; r < c[1]; ++r) {{
      mk::SpLayout l; l.blk = c[2]; l.rank = r; l.world = c[1]; l.rows_per_rank = c[0] / c[1];
      for (int row = 0; row < l.rows_per_rank; row += 61) {{
        const int p = mk::sp_pos(l, row);
        std::printf("%d %d %d %d %d %d\\n", c[0], c[1], r, row, p, mk::sp_row(l, p));
      }}
    }}
  return 0;
}}
''')
    exe = tmp_path / "sp_host"
    nvcc = os.path.join("/usr/local/cuda/bin", "nvcc")
    if not os.path.exists(nvcc):
        pytest.skip("nvcc not installed")
    subprocess.run([nvcc, "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-o", str(exe), str(src)],
                   check=True, capture_output=True, timeout=300)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True, timeout=60).stdout.split("\n")
    rows = [list(map(int, line.split())) for line in out if line.strip()]
    assert len(rows) > 100
    for seq, world, r, row, p, back in rows:
        blk = {(8192, 2): 512, (8192, 8): 512, (2048, 2): 512, (1024, 4): 128}[(seq, world)]
        assert p == sp.sp_pos(row, blk, r, world)
        assert back == sp.sp_row(p, blk, world, seq // world) == r * (seq // world) + row


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ws = torch.zeros(4096, dtype=torch.uint8)
        send, recv, nbytes = 256, 1024, 100
        ws[send:send + nbytes] = rank + 1
        gather = sp.nccl_allgather()(ws)
        assert gather(ws.data_ptr() + send, ws.data_ptr() + recv, nbytes, 0) == 0
        q.put((rank, ws[recv:recv + world * nbytes].tolist(), int(ws[recv + world * nbytes:].sum())))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_allgather_callback_two_gloo_ranks():
    """The callback the library calls gathers rank r's bytes to offset r * bytes_per_rank of every
    rank's receive rows and touches nothing else of the workspace."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict((r, (g, rest)) for r, g, rest in (q.get(timeout=120) for _ in procs))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(2):
        gathered, rest = res[r]
        assert gathered == [1] * 100 + [2] * 100
        assert rest == 0


def _worker_dead_peer(rank, world, port, q):
    """Rank 1 leaves before the gather; rank 0's gather must fail within the group timeout, not hang."""
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    if rank == 1:
        q.put((1, "left"))
        q.close()
        q.join_thread()  # the message is out before the process vanishes
        os._exit(0)  # no destroy, no gather: the peer just disappears
    ws = torch.zeros(1024, dtype=torch.uint8)
    gather = sp.nccl_allgather()(ws)
    try:
        gather(ws.data_ptr(), ws.data_ptr() + 256, 100, 0)
        q.put((0, "returned"))
    except Exception as e:  # noqa: BLE001 - any error is the expected outcome
        q.put((0, "error: " + type(e).__name__))


def test_allgather_with_a_dead_peer_errors_out():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_dead_peer, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res[1] == "left"
    assert res[0].startswith("error"), res


def test_allgather_rejects_buffers_outside_the_workspace():
    ws = torch.zeros(64, dtype=torch.uint8)
    with pytest.raises(ValueError):
        sp._slice(ws, ws.data_ptr() + 60, 16)

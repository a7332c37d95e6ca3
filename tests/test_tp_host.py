"""Host side of tensor parallelism on CPU with two gloo ranks (world size 2, 127.0.0.1):
each rank computes the slices it would load with jinf_tp_shard (the engine's loader rule:
q/k/v, gate/up and the vocabulary split by rows, attn_output and ffn_down by whole
32-element column blocks, everything else replicated), the slices are exchanged, and
together they must tile every tensor of the Llama-3-8B and tiny shapes exactly once. The
NCCL unique id crosses the same gloo channel that bench.py uses."""
import ctypes as C
import os
import queue
import socket

import pytest

WORLD = 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _shard(name, rows, cols, rank, size):
    import jinf
    out = [C.c_int64() for _ in range(4)]
    rc = jinf.lib.jinf_tp_shard(name.encode(), rows, cols, rank, size, *[C.byref(o) for o in out])
    return (rc,) + tuple(o.value for o in out)


def _rank_main(rank, world, port, tensors, id_bytes, out_q):
    import sys
    import datetime
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "jetson-inference_b200"))
    import torch.distributed as dist
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        mine = {name: _shard(name, rows, cols, rank, world) for name, rows, cols in tensors}
        gathered = [None] * world
        dist.all_gather_object(gathered, mine)
        buf = [id_bytes if rank == 0 else None]
        dist.broadcast_object_list(buf, src=0)
        dist.barrier()
        dist.destroy_process_group()
        out_q.put((rank, "ok", gathered, buf[0]))
    except Exception as e:
        out_q.put((rank, "error", repr(e), None))


def _tensors(shape):
    import jinf
    syn = jinf.SynthModel(shape, seed=0)
    out = []
    for name in syn.tensor_names():
        _, dims, _ = syn.tensor_info(name)
        cols = dims[0]
        rows = dims[1] if len(dims) > 1 else 1
        out.append((name, rows, cols))
    syn.close()
    return out


@pytest.mark.parametrize("which", ["8b", "tiny"])
def test_gloo_ranks_tile_every_tensor(which):
    import jinf
    import torch.multiprocessing as mp
    shape = jinf.LLAMA3_8B if which == "8b" else jinf.TINY
    tensors = _tensors(shape)
    id_bytes = bytes(range(128))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, WORLD, port, tensors, id_bytes, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(WORLD):
            rank, status, gathered, got_id = q.get(timeout=180)
            assert status == "ok", f"rank {rank}: {gathered}"
            results[rank] = (gathered, got_id)
    except queue.Empty:
        pytest.fail("a gloo rank did not report")
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert results[1][1] == id_bytes  # the NCCL id as rank 1 receives it
    gathered = results[0][0]
    assert gathered == results[1][0]
    roles = {0: "replicated", 1: "column", 2: "row"}
    for name, rows, cols in tensors:
        per_rank = [gathered[r][name] for r in range(WORLD)]
        assert all(p[0] == 0 for p in per_rank), name
        role = roles[jinf.lib.jinf_split_tp_role(name.encode())]
        if role == "replicated":
            assert all(p[1:] == (0, rows, 0, cols) for p in per_rank), name
            continue
        covered = []
        for _, r0, nr, c0, nc in per_rank:
            if role == "column":
                assert (c0, nc) == (0, cols), name
                covered.append((r0, r0 + nr))
            else:
                assert (r0, nr) == (0, rows) and c0 % 32 == 0 and nc % 32 == 0, name
                covered.append((c0, c0 + nc))
        covered.sort()
        total = rows if role == "column" else cols
        assert covered[0][0] == 0 and covered[-1][1] == total, name
        assert all(a[1] == b[0] for a, b in zip(covered, covered[1:])), name


def test_shard_rejects_uneven_splits():
    assert _shard("blk.0.attn_q.weight", 100, 4096, 0, 3)[0] != 0        # rows not divisible
    assert _shard("blk.0.ffn_down.weight", 4096, 1408, 0, 8)[0] != 0     # 176 columns: not whole blocks
    assert _shard("blk.0.ffn_down.weight", 4096, 1408, 0, 2)[0] == 0
    assert _shard("token_embd.weight", 4096, 512, 1, 8)[1:] == (0, 4096, 0, 512)

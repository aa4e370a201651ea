"""The row-sharded LM head over NCCL on real GPUs (one process per GPU).

Each rank holds its contiguous vocabulary slice of a Q6_K head 2048 ->
262,144, runs the fused GEMV + top-40 with its first row as the id offset,
the ranks all-gather the 64-bit keys over NCCL and every rank merges them
(heliopause_b200/sharded_head.py: the stripe + merge of
webgpu/segment-runner.ts:3208-3248 and mergeTopCandidates :3773-3794 with the
stripes on different GPUs).  Every rank's merged ids and values must equal
the unsharded hpc_lm_head_topk on the whole head, bit for bit, at 1, 5 and
64 columns.  Needs two GPUs; the ranks are spawned child processes with a
short process-group timeout.
"""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int):
    from datetime import timedelta

    import torch.distributed as dist

    from heliopause_b200 import kernels as hk
    from heliopause_b200 import sharded_head as sh
    from heliopause_b200 import synthetic as syn
    torch.cuda.set_device(rank)
    hk.init_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=torch.device("cuda", rank))
    try:
        K, V, k = 2048, 262144, 40
        full = syn.q6_k_weight(V, K, seed=77)
        first, n = sh.shard_rows(V, world)[rank]
        rb = syn.row_bytes(syn.Q6_K, K)
        backend = sh.CudaShardBackend("Q6_K", full[first * rb:(first + n) * rb], K, n, first, 64, k)
        whole = hk.create_quantized_weight_handle("Q6_K", full, K, V)
        head = sh.ShardedLmHead(backend, k)
        for m in (1, 5, 64):
            x = torch.from_numpy(syn.activations(m, K, seed=100 + m)).cuda()
            ids, vals = head.topk(x, m)
            rid, rval = hk.lm_head_topk(whole, x, m, k)
            assert torch.equal(ids.reshape(m, k), rid.reshape(m, k)), f"rank {rank} m={m}: ids differ"
            assert torch.equal(vals.reshape(m, k), rval.reshape(m, k)), f"rank {rank} m={m}: values differ"
        torch.cuda.synchronize()
        dist.barrier()
        hk.release_quantized_weight_handle(whole)
        backend.release()
    finally:
        dist.destroy_process_group()


def test_sharded_lm_head_two_gpus_equals_unsharded():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")
    import torch.multiprocessing as mp
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.spawn(_rank_main, args=(2, _free_port()), nprocs=2, join=True)

"""Row-sharded LM head + top-k (heliopause_b200/sharded_head.py).

CPU: two gloo ranks (spawned processes) run ShardedLmHead with an
oracle-backed backend (C restatement of lib.rs for the slice logits, the
same 64-bit key encoding and merge order as the kernels) and must reproduce
the oracle's top-k of the whole head (topK, runtime.ts:514-527) with the
softcap applied after selection (mergeTopCandidates,
webgpu/segment-runner.ts:3773-3794).

GPU (one device): the shards of 2, 4 and 8 ranks are emulated on one GPU --
each slice's fused GEMV + top-k keys (hpc_lm_head_topk_q8 with its id
offset), concatenated in rank order as the all-gather lays them out, then
hpc_topk_merge_keys -- and must equal the unsharded hpc_lm_head_topk.
"""
import math
import os
import socket

import numpy as np
import pytest
import torch

from heliopause_b200 import sharded_head as sh
from heliopause_b200 import synthetic as syn

K_DIM, ROWS, TOPK, COLS = 512, 3001, 12, 2


def _orderable(v: np.float32) -> int:
    b = int(np.float32(v).view(np.uint32))
    if v == 0:
        b = 0
    if v != v:
        return 0
    return (~b & 0xFFFFFFFF) if b & 0x80000000 else (b | 0x80000000)


def _key(v, i) -> int:
    return (_orderable(v) << 32) | (0xFFFFFFFF - int(i))


def _decode(key: int):
    o = key >> 32
    b = (o & 0x7FFFFFFF) if o & 0x80000000 else (~o & 0xFFFFFFFF)
    return 0xFFFFFFFF - (key & 0xFFFFFFFF), float(np.uint32(b).view(np.float32))


class OracleShardBackend:
    """Test-only backend: slice logits from the C oracle, keys in Python."""

    def __init__(self, weight, first_row, rows, k):
        from oracle import oracle
        self.o, self.first_row, self.rows, self.k = oracle, first_row, rows, k
        rb = oracle.row_bytes(oracle.Q6_K, K_DIM)
        self.w = weight[first_row * rb:(first_row + rows) * rb]
        self.s = oracle.prepare_scales(oracle.Q6_K, self.w, K_DIM, rows)

    def local_keys(self, hidden, columns):
        lg = self.o.matmul_prepared(self.o.Q6_K, self.w, self.s, hidden.numpy(), K_DIM, self.rows, columns)
        keys = []
        for c in range(columns):
            row = lg[c * self.rows:(c + 1) * self.rows]
            ks = sorted((_key(v, self.first_row + i) for i, v in enumerate(row)), reverse=True)[:self.k]
            keys += ks
        return torch.tensor(np.array(keys, dtype=np.uint64).view(np.int64))

    def merge(self, gathered, groups, columns, softcap):
        g = gathered.numpy().view(np.uint64).reshape(groups, columns, self.k)
        ids = np.zeros((columns, self.k), np.int32)
        vals = np.zeros((columns, self.k), np.float32)
        for c in range(columns):
            best = sorted((int(x) for x in g[:, c, :].reshape(-1)), reverse=True)[:self.k]
            for j, key in enumerate(best):
                i, v = _decode(key)
                ids[c, j] = i
                vals[c, j] = np.float32(math.tanh(v / softcap) * softcap) if softcap > 0 else v
        return torch.from_numpy(ids), torch.from_numpy(vals)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, softcap, out_dir):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = syn.q6_k_weight(ROWS, K_DIM, seed=31)
        first, n = sh.shard_rows(ROWS, world)[rank]
        head = sh.ShardedLmHead(OracleShardBackend(w, first, n, TOPK), TOPK)
        x = torch.from_numpy(syn.activations(COLS, K_DIM, seed=32))
        ids, vals = head.topk(x, COLS, softcap)
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), ids=ids.numpy(), vals=vals.numpy())
    finally:
        dist.destroy_process_group()


def test_shard_rows_matches_split_rule(oracle):
    for rows, world in ((262144, 8), (3001, 2), (10, 4), (7, 7)):
        parts = sh.shard_rows(rows, world)
        assert parts == oracle.split_rows(rows, world)
        assert sum(n for _, n in parts) == rows


@pytest.mark.parametrize("softcap", [0.0, 0.5])
def test_two_gloo_ranks_equal_unsharded_oracle(oracle, tmp_path, softcap):
    import torch.multiprocessing as mp
    mp.start_processes(_rank_main, args=(2, _free_port(), softcap, str(tmp_path)), nprocs=2, start_method="spawn")
    w = syn.q6_k_weight(ROWS, K_DIM, seed=31)
    x = syn.activations(COLS, K_DIM, seed=32)
    lg = oracle.matmul_prepared(oracle.Q6_K, w, oracle.prepare_scales(oracle.Q6_K, w, K_DIM, ROWS), x, K_DIM, ROWS,
                                COLS)
    for rank in range(2):
        got = np.load(tmp_path / f"rank{rank}.npz")
        for c in range(COLS):
            ids, vals = oracle.topk(lg[c * ROWS:(c + 1) * ROWS], TOPK)
            if softcap > 0:
                vals = oracle.softcap(vals, softcap)
            assert np.array_equal(got["ids"][c], ids)
            assert np.allclose(got["vals"][c], vals, rtol=1e-6, atol=1e-7)


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4, 8])
def test_emulated_shards_equal_unsharded_head_on_gpu(world):
    from heliopause_b200 import kernels as hk
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    hk.init_device(0)
    kdim, rows, k, cols = 2048, 262144, 40, 3
    w = syn.q6_k_weight(rows, kdim, seed=33)
    x = torch.from_numpy(syn.activations(cols, kdim, seed=34)).cuda()
    rb = syn.row_bytes(syn.Q6_K, kdim)
    full = hk.create_quantized_weight_handle("Q6_K", w, kdim, rows)
    backends = []
    try:
        for softcap in (0.0, 30.0):
            ref_ids, ref_vals = hk.lm_head_topk(full, x, cols, k, softcap=softcap)
            if not backends:
                backends = [sh.CudaShardBackend("Q6_K", w[first * rb:(first + n) * rb], kdim, n, first, cols, k)
                            for first, n in sh.shard_rows(rows, world)]
            gathered = torch.cat([b.local_keys(x, cols) for b in backends])
            ids, vals = backends[0].merge(gathered, world, cols, softcap)
            assert torch.equal(ids.cpu(), ref_ids.cpu())
            assert torch.equal(vals.cpu(), ref_vals.cpu())
    finally:
        for b in backends:
            b.release()
        hk.release_quantized_weight_handle(full)

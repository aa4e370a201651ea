"""Row-sharded LM head + top-k over several GPUs (one process per GPU).

The vocabulary rows are split contiguously over the ranks (the row split of
splitRows, runner/wasm/thread-pool.ts:410-424: the first `rows % world`
ranks take one extra row).  Each rank runs the fused GEMV + top-k on its
slice with its first row as `id_offset`, producing k 64-bit keys per column
(orderable(value) << 32 | 0xFFFFFFFF - id, larger = better); the ranks
all-gather the keys (NCCL) and every rank merges them into the global top-k,
value descending then id ascending, with the softcap applied after selection.
This is the stripe + merge of the WebGPU output path
(webgpu/segment-runner.ts:3208-3248, mergeTopCandidates :3773-3794) with the
stripes on different GPUs.

`ShardedLmHead` holds the orchestration (split, offsets, gather, merge); the
per-rank compute is a backend object.  `CudaShardBackend` is the product
backend (C-ABI kernels); tests substitute a CPU backend to exercise the
orchestration over gloo.
"""
from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as dist


def shard_rows(rows: int, world: int) -> list[tuple[int, int]]:
    """(first row, row count) per rank."""
    base, extra = divmod(rows, world)
    out, start = [], 0
    for r in range(world):
        n = base + (1 if r < extra else 0)
        out.append((start, n))
        start += n
    return out


class CudaShardBackend:
    """One rank's slice of the head, resident on the current CUDA device."""

    def __init__(self, type_name: str, slice_bytes, input_size: int, rows: int, first_row: int, max_columns: int,
                 k: int):
        from . import _lib
        from . import kernels as hk
        self.hk, self.L = hk, _lib.lib()
        self.input_size, self.rows, self.first_row, self.k = input_size, rows, first_row, k
        self.handle = hk.create_quantized_weight_handle(type_name, slice_bytes, input_size, rows)
        self.max_columns = max_columns
        nb = C.c_size_t()
        hk.assert_cuda_ok(self.L.hpc_q8_workspace_bytes(input_size, max_columns, C.byref(nb)), "workspace bytes")
        self.ws_bytes = nb.value
        self.ws = torch.empty(self.ws_bytes, dtype=torch.uint8, device="cuda")
        hk.assert_cuda_ok(self.L.hpc_lm_head_candidates_bytes(self.handle.handle, max_columns, k, C.byref(nb)),
                          "candidate bytes")
        self.cand_bytes = nb.value
        self.cand = torch.empty(self.cand_bytes, dtype=torch.uint8, device="cuda")
        self.ids = torch.empty(max_columns * k, dtype=torch.int32, device="cuda")
        self.vals = torch.empty(max_columns * k, dtype=torch.float32, device="cuda")

    def _stream(self):
        return C.c_void_p(torch.cuda.current_stream().cuda_stream)

    def local_keys(self, hidden: torch.Tensor, columns: int) -> torch.Tensor:
        """[columns * k] int64 (the uint64 keys' bits) of this slice."""
        if columns > self.max_columns:
            raise ValueError(f"{columns} columns > {self.max_columns}")
        keys = torch.empty(columns * self.k, dtype=torch.int64, device="cuda")
        hk, L, st = self.hk, self.L, self._stream()
        hk.assert_cuda_ok(L.hpc_q8_quantize(C.c_void_p(hidden.data_ptr()), hidden.numel(), self.input_size, columns,
                                            C.c_void_p(self.ws.data_ptr()), self.ws_bytes, st), "q8")
        hk.assert_cuda_ok(L.hpc_lm_head_topk_q8(self.handle.handle, C.c_void_p(self.ws.data_ptr()), self.ws_bytes,
                                                self.input_size, columns, self.k, self.first_row,
                                                C.c_void_p(self.cand.data_ptr()), self.cand_bytes, C.c_float(0.0),
                                                C.c_void_p(self.ids.data_ptr()), C.c_void_p(self.vals.data_ptr()),
                                                C.c_void_p(keys.data_ptr()), st), "lm head shard")
        return keys

    def merge(self, gathered: torch.Tensor, groups: int, columns: int, softcap: float):
        ids = torch.empty((columns, self.k), dtype=torch.int32, device="cuda")
        vals = torch.empty((columns, self.k), dtype=torch.float32, device="cuda")
        self.hk.assert_cuda_ok(self.L.hpc_topk_merge_keys(C.c_void_p(gathered.data_ptr()), groups, columns, self.k,
                                                          C.c_float(softcap), C.c_void_p(ids.data_ptr()),
                                                          C.c_void_p(vals.data_ptr()), self._stream()), "merge")
        return ids, vals

    def release(self):
        self.hk.release_quantized_weight_handle(self.handle)


class ShardedLmHead:
    """Top-k of the full head from row slices spread over the process group."""

    def __init__(self, backend, k: int, group=None):
        self.backend, self.k, self.group = backend, k, group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1

    def topk(self, hidden: torch.Tensor, columns: int, softcap: float = 0.0):
        """(ids, values), each [columns, k], identical on every rank."""
        keys = self.backend.local_keys(hidden, columns)
        if self.world > 1:
            gathered = torch.empty(self.world * keys.numel(), dtype=keys.dtype, device=keys.device)
            dist.all_gather_into_tensor(gathered, keys, group=self.group)
        else:
            gathered = keys
        return self.backend.merge(gathered, self.world, columns, softcap)

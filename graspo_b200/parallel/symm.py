"""Symmetric device buffers and the in-kernel tensor-parallel all-reduce.

``SymmetricBuffer`` allocates one equally sized buffer per rank of a process
group and maps every peer's buffer into this process (CUDA IPC handles
exchanged over the group), so kernels can store into a peer's memory over
NVLink and signal it with system-scope atomics.

``PeerReduce`` is one all-reduce site of the decode loop (the o_proj or
down_proj output).  The producing swap-AB split-K GEMM pushes every finished
fp32 output tile into each peer's receive slot for this rank and adds the
tile's element count to the peer's arrival counter; the consuming residual-add
+ RMSNorm kernel waits (bounded) until all peers' elements have arrived and
sums the partials in rank order -- so every rank holds bit-identical results
and no NCCL call is left on the decode path.  Layout of each rank's buffer::

    [0:4)   arrival counter (int32, written by peers)
    [4:8)   finished-CTA counter of the consumer (int32, local)
    [256:)  tp receive slots of rows x width fp32 (slot q: rank q's partial)

This replaces the per-layer NCCL all-reduce after o_proj / down_proj in the
reference's decode loop (reference: backends/graspoflow/tensor_utils.py:146-164
via models/common/layers_qwen3.py:264, 335).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from graspo_b200.ops._ext import err_word, ext

_HEADER = 256


class SymmetricBuffer:
    def __init__(self, nbytes: int, group, device: torch.device) -> None:
        C = ext()
        self.device = device
        self.buf, handle = C.symm_alloc(int(nbytes), device.index)
        self.rank = dist.get_rank(group)
        self.size = dist.get_world_size(group)
        handles: list = [None] * self.size
        dist.all_gather_object(handles, bytes(handle.tolist()), group=group)
        self.ptrs: list[int] = []
        for q, h in enumerate(handles):
            if q == self.rank:
                self.ptrs.append(self.buf.data_ptr())
            else:
                self.ptrs.append(C.symm_open(torch.tensor(list(h), dtype=torch.uint8), device.index))

    def close(self) -> None:
        C = ext()
        for q, p in enumerate(self.ptrs):
            if q != self.rank:
                C.symm_close(p, self.device.index)
        self.ptrs = []


class PeerReduce:
    """One fused all-reduce site: ``rows`` x ``width`` fp32 partials per rank."""

    def __init__(self, rows: int, width: int, group, device: torch.device) -> None:
        self.rows, self.width = int(rows), int(width)
        slot = self.rows * self.width * 4
        tp = dist.get_world_size(group)
        self.sym = SymmetricBuffer(_HEADER + tp * slot, group, device)
        r, p = self.sym.rank, self.sym.ptrs
        self.tp = tp
        self.push_dst = torch.tensor([0 if q == r else p[q] + _HEADER + r * slot for q in range(tp)],
                                     dtype=torch.int64)
        self.push_flag = torch.tensor([0 if q == r else p[q] for q in range(tp)], dtype=torch.int64)
        self.recv_src = torch.tensor([0 if q == r else p[r] + _HEADER + q * slot for q in range(tp)],
                                     dtype=torch.int64)
        self.sync = torch.tensor([p[r], p[r] + 4], dtype=torch.int64)
        self.expected = self.rows * self.width * (tp - 1)
        self.tile_ctr = torch.zeros(8192, dtype=torch.int32, device=device)
        self.err = err_word(device)

    def gemm_kwargs(self) -> dict:
        return {"push_dst": self.push_dst, "push_flag": self.push_flag, "tile_ctr": self.tile_ctr}

    def norm_kwargs(self) -> dict:
        return {"peer_src": self.recv_src, "peer_sync": self.sync, "peer_expected": self.expected,
                "err": self.err}

    def close(self) -> None:
        self.sym.close()

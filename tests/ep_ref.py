"""Reference (torch) implementation of the expert-parallel exchange steps, for tests.

Same contract as ``hydranet_b200.ep.CudaExchange``: ``pack`` writes W blocks of
T fixed rows (activations, k local ids with -1 for picks owned elsewhere, k
float32 weights), ``unpack`` splits received rows back into those three
arrays, ``combine`` sums per token, in rank order in float32, the partial rows
of the ranks that hold one of its picks.
"""

from __future__ import annotations

import torch


class TorchExchange:
    def __init__(self, row_align: int = 16):
        self.align = row_align

    def row_bytes(self, H: int, k: int, itemsize: int) -> int:
        n = H * itemsize + 8 * k
        return (n + self.align - 1) // self.align * self.align

    def pack(self, x, idx, w, num_experts, world):
        T, H = x.shape
        k = idx.shape[1]
        per = num_experts // world
        rb = self.row_bytes(H, k, x.element_size())
        send = torch.zeros(world, T, rb, dtype=torch.uint8)
        xb = x.contiguous().view(torch.uint8).view(T, -1)
        for d in range(world):
            local = (idx >= d * per) & (idx < (d + 1) * per)
            ids = torch.where(local, idx - d * per, torch.full_like(idx, -1)).to(torch.int32)
            wts = torch.where(local, w.to(torch.float32), torch.zeros_like(w, dtype=torch.float32))
            send[d, :, :xb.shape[1]] = torch.where(local.any(1, keepdim=True), xb, torch.zeros_like(xb))
            send[d, :, xb.shape[1]:xb.shape[1] + 4 * k] = ids.contiguous().view(torch.uint8).view(T, -1)
            send[d, :, xb.shape[1] + 4 * k:xb.shape[1] + 8 * k] = wts.contiguous().view(torch.uint8).view(T, -1)
        return send.view(world * T, rb)

    def unpack(self, recv, H, k, dtype):
        n = recv.shape[0]
        xs = torch.empty((), dtype=dtype).element_size() * H
        rows = recv[:, :xs].contiguous().view(dtype).view(n, H)
        ids = recv[:, xs:xs + 4 * k].contiguous().view(torch.int32).view(n, k)
        wts = recv[:, xs + 4 * k:xs + 8 * k].contiguous().view(torch.float32).view(n, k)
        return rows, ids, wts

    def combine(self, back, idx, num_experts, world):
        T, k = idx.shape
        per = num_experts // world
        out = torch.zeros(T, back.shape[-1], dtype=torch.float32)
        for d in range(world):
            has = ((idx >= d * per) & (idx < (d + 1) * per)).any(1)
            out += torch.where(has[:, None], back[d].to(torch.float32), torch.zeros_like(out))
        return out.to(back.dtype)

"""Out-feature (column) split of W4G64 linears across GPUs, gathered over NCCL.

The reference runs on one device; this is the multi-GPU layer the B200
build adds for large prefill GEMMs (the M = 4096 Qwen2-1.5B MLP). A linear's output
features are split into contiguous row ranges, one per rank. In the canonical
layout (src/qwen_int4/linear.py:39-44) row n of qweight is the K/2 bytes at
n*K/2, its scales are row n of ``scales`` and its zero points are nibbles
n*G .. n*G+G-1 of ``zeros`` (G = K/64), so a row range is a contiguous byte
range of every buffer (for even G; odd G is repacked on the host).

Each rank computes ``x @ W_r^T`` for its rows with the b200 kernels and the
shards are joined with one ``all_gather_into_tensor`` over NCCL (NVLink /
NVSwitch on one node). For the SwiGLU MLP (src/qwen_int4/model.py:125-136)
gate and up shards line up element-wise, so ``silu(gate) * up`` is formed on
the shard and gathered once before ``down_proj``, whose output is gathered
again: two collectives per MLP.

The per-shard compute is pluggable (``linear_fn``) so that the sharding and
gathering logic can be tested on CPU ranks (gloo) against the oracle; the
default is the CUDA backend, with no CPU fallback.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch
import torch.distributed as dist

GROUP = 64


def shard_bounds(n: int, world: int, rank: int) -> tuple[int, int]:
    """Row range of ``rank``: as even as possible, earlier ranks take the remainder."""
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def _unpack_nibbles(packed: torch.Tensor, count: int) -> torch.Tensor:
    b = packed.reshape(-1).to(torch.int16)
    return torch.stack((b & 0xF, b >> 4), dim=-1).reshape(-1)[:count]


def _pack_nibbles(nibbles: torch.Tensor) -> torch.Tensor:
    if nibbles.numel() % 2:
        nibbles = torch.cat((nibbles, nibbles.new_zeros(1)))
    pairs = nibbles.reshape(-1, 2)
    return (pairs[:, 0] | (pairs[:, 1] << 4)).to(torch.uint8).reshape(-1, 1)


@dataclass
class W4G64Shard:
    """The buffers of one rank's output rows, in the canonical layout."""

    qweight: torch.Tensor
    scales: torch.Tensor
    zeros: torch.Tensor
    bias: torch.Tensor | None
    rows: tuple[int, int]
    in_features: int

    @property
    def out_features(self) -> int:
        return self.rows[1] - self.rows[0]


def shard_rows(qweight, scales, zeros, bias, *, in_features: int, start: int, stop: int) -> W4G64Shard:
    """Rows [start, stop) of a canonical W4G64 linear (no copy when byte-aligned)."""
    k = in_features
    g = k // GROUP
    q = qweight.reshape(-1)[start * k // 2: stop * k // 2].reshape(-1, 1)
    s = scales[start:stop]
    if g % 2 == 0:
        z = zeros.reshape(-1)[start * g // 2: stop * g // 2].reshape(-1, 1)
    else:  # zero points of the shard straddle bytes: repack
        total = scales.shape[0] * g
        z = _pack_nibbles(_unpack_nibbles(zeros, total)[start * g: stop * g]).to(zeros.device)
    b = None if bias is None else bias[start:stop]
    return W4G64Shard(q.contiguous(), s.contiguous(), z.contiguous(),
                      None if b is None else b.contiguous(), (start, stop), k)


def _default_linear(x, shard: W4G64Shard) -> torch.Tensor:
    from .backends import b200_w4g64_linear

    return b200_w4g64_linear(x, shard.qweight, shard.scales, shard.zeros, shard.bias,
                             out_features=shard.out_features, in_features=shard.in_features,
                             group_size=GROUP, packing="canonical")


def gather_columns(local: torch.Tensor, n_total: int, group=None) -> torch.Tensor:
    """All-gather ``[M, N_r]`` shards (contiguous row ranges) into ``[M, N]``."""
    world = dist.get_world_size(group)
    m = local.shape[0]
    sizes = [shard_bounds(n_total, world, r) for r in range(world)]
    width = max(b - a for a, b in sizes)
    if local.shape[1] != width:  # uneven split: pad to a common width
        local = torch.nn.functional.pad(local, (0, width - local.shape[1]))
    buf = torch.empty((world * m, width), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(buf, local.contiguous(), group=group)  # rank r -> rows [r*M, (r+1)*M)
    buf = buf.view(world, m, width)
    parts = [buf[r, :, : b - a] for r, (a, b) in enumerate(sizes)]
    return torch.cat(parts, dim=1)


class ColumnParallelW4G64:
    """One W4G64 linear split by output features over the ranks of ``group``."""

    def __init__(self, qweight, scales, zeros, bias, *, in_features: int, out_features: int,
                 group=None, linear_fn: Callable | None = None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.out_features = out_features
        self.in_features = in_features
        a, b = shard_bounds(out_features, self.world, self.rank)
        self.shard = shard_rows(qweight, scales, zeros, bias, in_features=in_features, start=a, stop=b)
        self.linear_fn = linear_fn or _default_linear

    @classmethod
    def from_quant_linear(cls, layer, group=None, linear_fn=None):
        return cls(layer.qweight, layer.scales, layer.zeros, layer.bias, in_features=layer.in_features,
                   out_features=layer.out_features, group=group, linear_fn=linear_fn)

    def local(self, x: torch.Tensor) -> torch.Tensor:
        return self.linear_fn(x.reshape(-1, self.in_features), self.shard)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        y = gather_columns(self.local(x), self.out_features, self.group)
        return y.reshape(*x.shape[:-1], self.out_features)


class ColumnParallelMLP:
    """SwiGLU MLP (src/qwen_int4/model.py:125-136) with gate/up/down column-split.

    ``silu(gate) * up`` is computed in FP32 on the aligned gate/up shards and
    gathered once; ``down_proj`` receives the FP32 intermediate, as in the
    reference, and its output shards are gathered and cast to ``x.dtype``.
    """

    def __init__(self, mlp, group=None, linear_fn=None):
        self.gate = ColumnParallelW4G64.from_quant_linear(mlp.gate_proj, group, linear_fn)
        self.up = ColumnParallelW4G64.from_quant_linear(mlp.up_proj, group, linear_fn)
        self.down = ColumnParallelW4G64.from_quant_linear(mlp.down_proj, group, linear_fn)
        self.group = group

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-1]
        g = self.gate.local(x).to(torch.float32)
        u = self.up.local(x).to(torch.float32)
        h = torch.nn.functional.silu(g) * u
        full_h = gather_columns(h, self.gate.out_features, self.group)
        y = self.down(full_h)
        return y.reshape(*lead, self.down.out_features).to(x.dtype)

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
the shard by the fused gate/up call; ``ColumnParallelMLP`` then either
gathers it for a column-split ``down_proj`` (two all-gathers per MLP) or
feeds it to a ``down_proj`` split by input features on the same boundaries
(one all-reduce of the output, the intermediate never leaves the GPU), or, in
``column_fused`` mode, has the SwiGLU pass store its shard straight into
every rank's gathered intermediate over CUDA IPC peer mappings and publish a
per-call epoch flag (``qi4_w4g64_gate_up_silu_scatter``), which each rank
waits for on the GPU (``qi4_peer_flag_wait``) before its ``down_proj``.

The per-shard compute is pluggable (``linear_fn``) so that the sharding and
gathering logic can be tested on CPU ranks (gloo) against the oracle; the
default is the CUDA backend, with no CPU fallback.
"""

from __future__ import annotations

import ctypes
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


def group_bounds(n: int, world: int, rank: int, unit: int = GROUP) -> tuple[int, int]:
    """Range of ``rank`` with every boundary on a multiple of ``unit`` (whole
    quantisation groups): ``n`` in ``unit`` blocks split as evenly as possible."""
    a, b = shard_bounds(-(-n // unit), world, rank)
    return min(a * unit, n), min(b * unit, n)


def shard_cols(qweight, scales, zeros, *, out_features: int, in_features: int, start: int,
               stop: int) -> W4G64Shard:
    """Input features [start, stop) of a canonical W4G64 linear (whole groups):
    the packed bytes, scales and zero points of those groups of every row."""
    n, k = out_features, in_features
    if start % GROUP or (stop % GROUP and stop != k) or not 0 <= start <= stop <= k:
        raise ValueError(f"column shard [{start}, {stop}) must fall on group boundaries of K={k}")
    g, g0, g1 = k // GROUP, start // GROUP, stop // GROUP
    q = qweight.reshape(n, k // 2)[:, start // 2: stop // 2]
    s = scales.reshape(n, g)[:, g0:g1]
    z = _pack_nibbles(_unpack_nibbles(zeros, n * g).reshape(n, g)[:, g0:g1].reshape(-1)).to(zeros.device)
    return W4G64Shard(q.contiguous().reshape(-1, 1), s.contiguous(), z.contiguous(), None, (0, n), stop - start)


def _default_linear(x, shard: W4G64Shard) -> torch.Tensor:
    from .backends import b200_w4g64_linear

    return b200_w4g64_linear(x, shard.qweight, shard.scales, shard.zeros, shard.bias,
                             out_features=shard.out_features, in_features=shard.in_features,
                             group_size=GROUP, packing="canonical")


def _default_swiglu(x, gate: W4G64Shard, up: W4G64Shard) -> torch.Tensor:
    from .backends import b200_w4g64_gate_up_silu

    return b200_w4g64_gate_up_silu(x, gate, up)


def _world(group) -> tuple[int, int]:
    if not dist.is_available() or not dist.is_initialized():
        return 1, 0  # one process: no collectives
    return dist.get_world_size(group), dist.get_rank(group)


def gather_columns(local: torch.Tensor, n_total: int, group=None, bounds=None) -> torch.Tensor:
    """All-gather ``[M, N_r]`` shards (contiguous column ranges, rank order)
    into ``[M, N]``. ``bounds`` lists every rank's range (default: ``shard_bounds``)."""
    world, _ = _world(group)
    if world == 1:
        return local
    m = local.shape[0]
    sizes = bounds or [shard_bounds(n_total, world, r) for r in range(world)]
    width = max(b - a for a, b in sizes)
    if local.shape[1] != width:  # uneven split: pad to a common width
        local = torch.nn.functional.pad(local, (0, width - local.shape[1]))
    buf = torch.empty((world * m, width), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(buf, local.contiguous(), group=group)  # rank r -> rows [r*M, (r+1)*M)
    buf = buf.view(world, m, width)
    out = torch.empty((m, n_total), dtype=local.dtype, device=local.device)
    for r, (a, b) in enumerate(sizes):  # one strided copy per rank, no intermediate concatenation
        out[:, a:b].copy_(buf[r, :, : b - a])
    return out


class _DevArray:
    """A device buffer given as a raw pointer, viewable as a torch tensor."""

    def __init__(self, ptr: int, shape: tuple, typestr: str = "<f4"):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False), "version": 3,
                                         "strides": None}


class PeerGatherBuffers:
    """Every rank's gathered FP32 intermediate [rows, width] and its flag words
    (world flags + one CTA counter), in one buffer per rank shared over CUDA
    IPC (plain peer mappings, no multicast); with one process, a local buffer.
    Collective: every rank of ``group`` constructs it with the same sizes."""

    def __init__(self, lib, rows: int, width: int, group, device):
        from . import _lib

        self.lib, self.rows, self.width = lib, rows, width
        self.world, self.rank = _world(group)
        data_bytes = (rows * width * 4 + 255) // 256 * 256
        total = data_bytes + 256
        self._opened, self._owned, self._tensor = [], None, None
        if self.world == 1:
            self._tensor = torch.zeros(total // 4, dtype=torch.float32, device=device)
            bases = [self._tensor.data_ptr()]
        else:
            ptr, handle = ctypes.c_void_p(), (ctypes.c_char * 64)()
            _lib.check(lib.qi4_ipc_alloc(total, ctypes.byref(ptr), handle), "qi4_ipc_alloc")
            self._owned = ptr.value
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=group)
            bases = []
            for p, h in enumerate(handles):
                if p == self.rank:
                    bases.append(self._owned)
                    continue
                peer = ctypes.c_void_p()
                _lib.check(lib.qi4_ipc_open((ctypes.c_char * 64).from_buffer_copy(h), ctypes.byref(peer)),
                           "qi4_ipc_open")
                self._opened.append(peer.value)
                bases.append(peer.value)
        self.data = [b for b in bases]
        self.flags = [b + data_bytes for b in bases]
        self.local = torch.as_tensor(_DevArray(self.data[self.rank], (rows, width)), device=device)

    def close(self):
        for p in self._opened:
            self.lib.qi4_ipc_close(p)
        if self._owned is not None:
            self.lib.qi4_ipc_free(self._owned)
        self._opened, self._owned, self._tensor = [], None, None


class ColumnParallelW4G64:
    """One W4G64 linear split by output features over the ranks of ``group``."""

    def __init__(self, qweight, scales, zeros, bias, *, in_features: int, out_features: int,
                 group=None, linear_fn: Callable | None = None):
        self.group = group
        self.world, self.rank = _world(group)
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
    """SwiGLU MLP (src/qwen_int4/model.py:125-136) split over the ranks of ``group``.

    gate_proj / up_proj are split by output features on whole-group
    boundaries (64 columns), and each rank forms ``silu(gate) * up`` in FP32
    on its shard with one fused call (the FP32 tensor the reference passes to
    ``down_proj``). Then, by ``mode``:

    * ``"column"`` - the intermediate is all-gathered (FP32, M x 8960),
      ``down_proj`` is split by output features, and its output, cast to
      ``x.dtype`` first, is all-gathered: two all-gathers per MLP.
    * ``"column_row"`` - ``down_proj`` is split by input features on the same
      boundaries, so each rank's intermediate shard is exactly the input its
      ``down_proj`` shard needs; the FP32 partial outputs are summed with one
      all-reduce (M x 1536 FP32) and cast. Nothing of the intermediate
      crosses the link. The sum over ranks changes the FP32 summation order
      only.
    * ``"column_fused"`` - as ``"column"``, but the intermediate's gather is
      fused into the SwiGLU pass: each value is stored into every rank's
      gathered buffer (peer stores over NVLink) as it is produced, and a
      per-call epoch flag, waited for on the GPU with a time limit
      (``flag_timeout_s``; a time-out is reported by ``qi4_device_status``),
      replaces the collective. The down_proj output is gathered over NCCL,
      which also keeps a rank from overwriting a peer's intermediate before
      that peer's down_proj has read it. CUDA backend only.

    With one process (no process group) both modes are the unsplit MLP.
    """

    MODES = ("column", "column_row", "column_fused")

    def __init__(self, mlp, group=None, linear_fn=None, mode: str = "column", swiglu_fn=None,
                 flag_timeout_s: float = 2.0):
        if mode not in self.MODES:
            raise ValueError(f"mode must be one of {self.MODES}, got {mode!r}")
        self.group, self.mode = group, mode
        self.world, self.rank = _world(group)
        gate, up, down = mlp.gate_proj, mlp.up_proj, mlp.down_proj
        self.hidden, self.inter = gate.in_features, gate.out_features
        self.bounds = [group_bounds(self.inter, self.world, r) for r in range(self.world)]
        a, b = self.bounds[self.rank]
        self.gate = shard_rows(gate.qweight, gate.scales, gate.zeros, None, in_features=self.hidden, start=a, stop=b)
        self.up = shard_rows(up.qweight, up.scales, up.zeros, None, in_features=self.hidden, start=a, stop=b)
        if mode == "column_fused" and (linear_fn is not None or swiglu_fn is not None
                                       or gate.qweight.device.type != "cuda"):
            raise ValueError("mode 'column_fused' runs the CUDA kernels only (no linear_fn / swiglu_fn, CUDA weights)")
        self.flag_timeout_ns = int(flag_timeout_s * 1e9)
        self._peer, self._epoch = None, 0
        if mode in ("column", "column_fused"):
            ra, rb = shard_bounds(self.hidden, self.world, self.rank)
            self.down = shard_rows(down.qweight, down.scales, down.zeros, down.bias, in_features=self.inter,
                                   start=ra, stop=rb)
        else:
            self.down = shard_cols(down.qweight, down.scales, down.zeros, out_features=self.hidden,
                                   in_features=self.inter, start=a, stop=b)
            self.down_bias = down.bias
        self.linear_fn = linear_fn or _default_linear
        if swiglu_fn is None and linear_fn is not None:
            swiglu_fn = lambda x, g, u: (torch.nn.functional.silu(self.linear_fn(x, g).float())  # noqa: E731
                                         * self.linear_fn(x, u).float())
        self.swiglu_fn = swiglu_fn or _default_swiglu

    def _fused_intermediate(self, x2: torch.Tensor) -> torch.Tensor:
        from . import _lib

        lib = _lib.load()
        m = x2.shape[0]
        if self._peer is None or self._peer.rows < m:  # collective: every rank sees the same M
            if self._peer is not None:
                self.close()
            self._peer = PeerGatherBuffers(lib, m, self.inter, self.group, x2.device)
            self._epoch = 0
        self._epoch = (self._epoch + 1) & 0xFFFFFFFF
        pb, w = self._peer, self.world
        codes = {torch.float16: _lib.DTYPE_F16, torch.bfloat16: _lib.DTYPE_BF16, torch.float32: _lib.DTYPE_F32}
        x2 = x2.contiguous()
        g, u = self.gate, self.up
        stream = torch.cuda.current_stream(x2.device).cuda_stream
        rc = lib.qi4_w4g64_gate_up_silu_scatter(
            x2.data_ptr(), codes[x2.dtype], m, self.hidden, g.qweight.data_ptr(), g.scales.data_ptr(),
            g.zeros.data_ptr(), u.qweight.data_ptr(), u.scales.data_ptr(), u.zeros.data_ptr(), g.out_features,
            (ctypes.c_void_p * w)(*pb.data), self.inter, self.bounds[self.rank][0], (ctypes.c_void_p * w)(*pb.flags),
            w, self.rank, self._epoch, stream)
        _lib.check(rc, "qi4_w4g64_gate_up_silu_scatter")
        _lib.check(lib.qi4_peer_flag_wait(pb.flags[self.rank], w, self._epoch, self.flag_timeout_ns, stream),
                   "qi4_peer_flag_wait")
        return pb.local[:m]

    def close(self):
        """Releases the peer buffers of ``column_fused`` mode (collective)."""
        if self._peer is not None:
            torch.cuda.synchronize()
            if self.world > 1:
                dist.barrier(group=self.group)  # no peer still stores into or reads these buffers
            self._peer.close()
            self._peer = None

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-1]
        x2 = x.reshape(-1, self.hidden)
        if self.mode == "column_fused":
            y = self.linear_fn(self._fused_intermediate(x2), self.down).to(x.dtype)
            return gather_columns(y, self.hidden, self.group).reshape(*lead, self.hidden)
        if self.gate.out_features:
            h = self.swiglu_fn(x2, self.gate, self.up)
        else:
            h = torch.zeros((x2.shape[0], 0), dtype=torch.float32, device=x.device)
        if self.mode == "column":
            full_h = gather_columns(h, self.inter, self.group, self.bounds)
            y = self.linear_fn(full_h, self.down).to(x.dtype)
            y = gather_columns(y, self.hidden, self.group)
        else:
            if self.down.in_features:
                y = self.linear_fn(h, self.down).float()
            else:
                y = torch.zeros((x2.shape[0], self.hidden), dtype=torch.float32, device=x.device)
            if self.world > 1:
                dist.all_reduce(y, group=self.group)
            if self.down_bias is not None:
                y = y + self.down_bias.float()
            y = y.to(x.dtype)
        return y.reshape(*lead, self.hidden)

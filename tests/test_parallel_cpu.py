"""Column-split W4G64 over 2 CPU ranks (gloo): sharding and gathering logic.

The per-shard compute is the oracle here (the CUDA kernels need a GPU); the
gathered result must equal the unsplit oracle linear up to the summation
order BLAS picks for different matrix widths (1e-6 relative): every output
element comes from the same weight row and the same activations.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import w4g64 as orc


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_linear(x, shard):
    out = orc.linear(x.float().numpy(), shard.qweight.numpy(), shard.scales.numpy(), shard.zeros.numpy(),
                     None if shard.bias is None else shard.bias.float().numpy(),
                     out_features=shard.out_features, in_features=shard.in_features)
    return torch.from_numpy(out)


def _worker(rank, world, port, n, k, g_odd, result_path):
    import importlib
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    par = importlib.import_module("qwen2-int4-systems_b200.parallel")
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(5)
        w = rng.standard_normal((n, k), dtype=np.float32) * 0.05
        qw, sc, z = orc.quantize_asymmetric_rtn(w)
        bias = torch.from_numpy(rng.standard_normal(n, dtype=np.float32) * 0.1)
        x = torch.from_numpy(rng.standard_normal((3, k), dtype=np.float32))
        lin = par.ColumnParallelW4G64(torch.from_numpy(qw), torch.from_numpy(sc), torch.from_numpy(z), bias,
                                      in_features=k, out_features=n, linear_fn=_oracle_linear)
        got = lin(x)
        ref = orc.linear(x.numpy(), qw, sc, z, bias.numpy(), out_features=n, in_features=k)
        ok = got.shape == ref.shape and np.allclose(got.numpy(), ref, rtol=1e-6, atol=1e-6)
        flag = torch.tensor([1 if ok else 0])
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        if rank == 0:
            with open(result_path, "w") as f:
                f.write(str(int(flag.item())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize(("n", "k", "world"), [(96, 128, 2), (7, 192, 2), (100, 64, 3)])
def test_column_split_gather_equals_unsplit(tmp_path, n, k, world):
    result = tmp_path / "ok"
    mp.start_processes(_worker, args=(world, _free_port(), n, k, (k // 64) % 2, str(result)), nprocs=world,
                       join=True, start_method="spawn")
    assert result.read_text() == "1"


def test_shard_bounds_cover_exactly():
    import importlib

    par = importlib.import_module("qwen2-int4-systems_b200.parallel")
    for n in (1, 7, 8960, 1536):
        for world in (1, 2, 3, 8):
            spans = [par.shard_bounds(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert max(b - a for a, b in spans) - min(b - a for a, b in spans) <= 1


def test_odd_group_count_zero_points_are_repacked():
    import importlib

    par = importlib.import_module("qwen2-int4-systems_b200.parallel")
    rng = np.random.default_rng(2)
    n, k = 5, 192  # G = 3: shard boundaries fall inside zero-point bytes
    qw, sc, z = orc.quantize_asymmetric_rtn(rng.standard_normal((n, k), dtype=np.float32))
    full = orc.dequantize_groupwise(qw, sc, out_features=n, in_features=k, zeros=z)
    for a, b in ((0, 2), (2, 5), (1, 4)):
        sh = par.shard_rows(torch.from_numpy(qw), torch.from_numpy(sc), torch.from_numpy(z), None,
                            in_features=k, start=a, stop=b)
        part = orc.dequantize_groupwise(sh.qweight.numpy(), sh.scales.numpy(), out_features=b - a,
                                        in_features=k, zeros=sh.zeros.numpy())
        np.testing.assert_array_equal(part, full[a:b])


def _mlp_worker(rank, world, port, result_path, mode="column"):
    import importlib
    import sys
    from types import SimpleNamespace

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    par = importlib.import_module("qwen2-int4-systems_b200.parallel")
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(9)
        hidden, inter = 128, 320

        def qlinear(n, k):
            qw, sc, z = orc.quantize_asymmetric_rtn(rng.standard_normal((n, k), dtype=np.float32) * 0.05)
            return SimpleNamespace(qweight=torch.from_numpy(qw), scales=torch.from_numpy(sc),
                                   zeros=torch.from_numpy(z), bias=None, in_features=k, out_features=n)

        mlp = SimpleNamespace(gate_proj=qlinear(inter, hidden), up_proj=qlinear(inter, hidden),
                              down_proj=qlinear(hidden, inter))
        x = torch.from_numpy(rng.standard_normal((4, hidden), dtype=np.float32)).to(torch.bfloat16)
        got = par.ColumnParallelMLP(mlp, linear_fn=_oracle_linear, mode=mode)(x)

        def full(layer, inp):
            return orc.linear(inp, layer.qweight.numpy(), layer.scales.numpy(), layer.zeros.numpy(), None,
                              out_features=layer.out_features, in_features=layer.in_features)

        xf = x.float().numpy()
        g, u = full(mlp.gate_proj, xf), full(mlp.up_proj, xf)
        h = (torch.nn.functional.silu(torch.from_numpy(g)) * torch.from_numpy(u)).numpy()
        ref = torch.from_numpy(full(mlp.down_proj, h)).to(torch.bfloat16)
        ok = got.dtype == torch.bfloat16 and got.shape == ref.shape and torch.allclose(
            got.float(), ref.float(), rtol=1e-2, atol=1e-3)
        flag = torch.tensor([1 if ok else 0])
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        if rank == 0:
            with open(result_path, "w") as f:
                f.write(str(int(flag.item())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize(("mode", "world"), [("column", 2), ("column_row", 2), ("column_row", 3)])
def test_column_split_swiglu_mlp_matches_unsplit(tmp_path, mode, world):
    """Both split modes give the unsplit MLP (intermediate 320 = 5 groups, so
    3 ranks get uneven group-aligned shards)."""
    result = tmp_path / "ok"
    mp.start_processes(_mlp_worker, args=(world, _free_port(), str(result), mode), nprocs=world, join=True,
                       start_method="spawn")
    assert result.read_text() == "1"


def test_single_process_mlp_is_the_unsplit_mlp():
    """Without a process group both modes run the whole MLP on one rank."""
    import importlib
    from types import SimpleNamespace

    par = importlib.import_module("qwen2-int4-systems_b200.parallel")
    rng = np.random.default_rng(3)

    def qlinear(n, k):
        qw, sc, z = orc.quantize_asymmetric_rtn(rng.standard_normal((n, k), dtype=np.float32) * 0.05)
        return SimpleNamespace(qweight=torch.from_numpy(qw), scales=torch.from_numpy(sc),
                               zeros=torch.from_numpy(z), bias=None, in_features=k, out_features=n)

    mlp = SimpleNamespace(gate_proj=qlinear(192, 64), up_proj=qlinear(192, 64), down_proj=qlinear(64, 192))
    x = torch.from_numpy(rng.standard_normal((2, 64), dtype=np.float32)).to(torch.bfloat16)
    a = par.ColumnParallelMLP(mlp, linear_fn=_oracle_linear, mode="column")(x)
    b = par.ColumnParallelMLP(mlp, linear_fn=_oracle_linear, mode="column_row")(x)
    assert torch.equal(a, b)
    # The fused exchange is the CUDA kernels' own (peer stores over CUDA IPC):
    # CPU weights or a pluggable shard compute are refused, never emulated.
    with pytest.raises(ValueError, match="column_fused"):
        par.ColumnParallelMLP(mlp, mode="column_fused")
    with pytest.raises(ValueError, match="column_fused"):
        par.ColumnParallelMLP(mlp, linear_fn=_oracle_linear, mode="column_fused")
    with pytest.raises(ValueError, match="mode must be one of"):
        par.ColumnParallelMLP(mlp, mode="row")


def test_group_bounds_and_column_shards():
    """Group-aligned ranges cover the features exactly, and a column shard
    dequantises to the matching columns of the full weight (odd G: zero
    points repacked)."""
    import importlib

    par = importlib.import_module("qwen2-int4-systems_b200.parallel")
    for n, world in ((8960, 8), (8960, 3), (320, 3), (64, 2), (1536, 8)):
        spans = [par.group_bounds(n, world, r) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
        assert all(a % 64 == 0 for a, _ in spans)
    rng = np.random.default_rng(4)
    n, k = 5, 320  # G = 5
    qw, sc, z = orc.quantize_asymmetric_rtn(rng.standard_normal((n, k), dtype=np.float32))
    full = orc.dequantize_groupwise(qw, sc, out_features=n, in_features=k, zeros=z)
    for a, b in ((0, 128), (128, 320), (64, 192)):
        sh = par.shard_cols(torch.from_numpy(qw), torch.from_numpy(sc), torch.from_numpy(z),
                            out_features=n, in_features=k, start=a, stop=b)
        part = orc.dequantize_groupwise(sh.qweight.numpy(), sh.scales.numpy(), out_features=n,
                                        in_features=b - a, zeros=sh.zeros.numpy())
        np.testing.assert_array_equal(part, full[:, a:b])
    with pytest.raises(ValueError):
        par.shard_cols(torch.from_numpy(qw), torch.from_numpy(sc), torch.from_numpy(z),
                       out_features=n, in_features=k, start=32, stop=128)


def _dead_peer_worker(rank, world, port, result_path):
    """Rank 1 leaves before the collective; rank 0 must get an error, not hang."""
    import datetime
    import importlib
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    par = importlib.import_module("qwen2-int4-systems_b200.parallel")
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        return  # exits without joining the gather
    try:
        par.gather_columns(torch.zeros(2, 4), 8)
        outcome = "no-error"
    except Exception:
        outcome = "error"
    with open(result_path, "w") as f:
        f.write(outcome)


def test_gather_with_a_lost_rank_fails_instead_of_hanging(tmp_path):
    result = tmp_path / "outcome"
    try:
        mp.start_processes(_dead_peer_worker, args=(2, _free_port(), str(result)), nprocs=2, join=True,
                           start_method="spawn")
    except Exception:
        pass  # a rank may also exit with an error; what matters is rank 0's outcome
    assert result.read_text() == "error"


def test_torch_asymmetric_quantizer_matches_the_oracle_bytes():
    """The device-agnostic torch quantiser used to build synthetic asymmetric
    weights gives the oracle's (reference-pinned) bytes on CPU."""
    import importlib

    q2 = importlib.import_module("qwen2-int4-systems_b200.qwen2")
    rng = np.random.default_rng(11)
    for n, k in ((8, 128), (3, 192), (16, 64)):
        w = rng.standard_normal((n, k), dtype=np.float32) * 0.05
        w[0, :64] = 0.0  # an all-zero group
        qw, sc, z = q2.quantize_asymmetric_rtn_torch(torch.from_numpy(w))
        oq, osc, oz = orc.quantize_asymmetric_rtn(w)
        np.testing.assert_array_equal(qw.numpy(), oq)
        np.testing.assert_array_equal(sc.numpy(), osc)
        np.testing.assert_array_equal(z.numpy(), oz)

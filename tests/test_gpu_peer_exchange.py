"""The column-split gather fused into the SwiGLU pass, on one GPU.

qi4_w4g64_gate_up_silu_scatter stores a rank's shard of silu(gate) * up into
every rank's gathered buffer and publishes the call's epoch on every rank's
flag array; qi4_peer_flag_wait waits for all of a rank's flags. Here the
ranks are emulated on one GPU: all "ranks" run their scatter in one stream
before any wait, so no kernel waits on another that has not run (the flags
are already set when the waits start). Checked: every gathered buffer equals
each shard computed by qi4_w4g64_gate_up_silu on the shard's weights (bit for
bit on the tensor-core route; within one bf16 rounding of the projections on
the GEMV route, whose fused kernel sums in another order); flags hold the
epoch and the CTA counters are re-armed; a second call reuses the buffers;
an empty shard still publishes; and a flag nobody
sets ends the wait at its time limit with QI4_DEVICE_WAIT_TIMEOUT while the
GPU context stays usable. The multi-GPU path itself is tested in
test_gpu_multi.py (two GPUs, CUDA IPC peer mappings).
"""

import ctypes
import importlib

import numpy as np
import pytest
import torch

from oracle import w4g64 as orc

pytestmark = pytest.mark.gpu

BF16, F32 = 1, 2


def _lib(b200):
    mod = importlib.import_module(b200.__name__ + "._lib")
    return mod, mod.load()


def _par(b200):
    return importlib.import_module(b200.__name__ + ".parallel")


def _weights(n, k, seed, dev):
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(2):  # gate, up
        qw, sc, z = orc.quantize_asymmetric_rtn(rng.standard_normal((n, k), dtype=np.float32) * 0.02)
        out.append((torch.from_numpy(qw).to(dev), torch.from_numpy(sc).to(dev), torch.from_numpy(z).to(dev)))
    return out


def _run_emulated(b200, dev, m, n, k, world, x_dtype, epochs=(1,), seed=0):
    mod, lib = _lib(b200)
    par = _par(b200)
    (gq, gs, gz), (uq, us, uz) = _weights(n, k, seed, dev)
    bounds = [par.group_bounds(n, world, r) for r in range(world)]
    shards = []
    for a, b in bounds:
        g = par.shard_rows(gq, gs, gz, None, in_features=k, start=a, stop=b)
        u = par.shard_rows(uq, us, uz, None, in_features=k, start=a, stop=b)
        shards.append((g, u))
    bufs = [torch.full((m, n), float("nan"), dtype=torch.float32, device=dev) for _ in range(world)]
    flags = [torch.zeros(world + 1, dtype=torch.int32, device=dev) for _ in range(world)]
    outs = (ctypes.c_void_p * world)(*[t.data_ptr() for t in bufs])
    fl = (ctypes.c_void_p * world)(*[t.data_ptr() for t in flags])
    stream = torch.cuda.current_stream().cuda_stream
    code = BF16 if x_dtype == torch.bfloat16 else F32
    for call, epoch in enumerate(epochs):
        g = torch.Generator().manual_seed(seed * 10 + call)
        x = torch.randn(m, k, generator=g).to(x_dtype).to(dev)
        for r, ((a, b), (gsh, ush)) in enumerate(zip(bounds, shards)):
            rc = lib.qi4_w4g64_gate_up_silu_scatter(
                x.data_ptr(), code, m, k, gsh.qweight.data_ptr(), gsh.scales.data_ptr(), gsh.zeros.data_ptr(),
                ush.qweight.data_ptr(), ush.scales.data_ptr(), ush.zeros.data_ptr(), b - a, outs, n, a, fl, world,
                r, epoch, stream)
            mod.check(rc, "qi4_w4g64_gate_up_silu_scatter")
        for p in range(world):
            mod.check(lib.qi4_peer_flag_wait(flags[p].data_ptr(), world, epoch, 10_000_000, stream),
                      "qi4_peer_flag_wait")
        torch.cuda.synchronize()
        # Reference: each shard through the unsplit fused entry point.
        ref = torch.empty(m, n, dtype=torch.float32, device=dev)
        for (a, b), (gsh, ush) in zip(bounds, shards):
            if b == a:
                continue
            part = torch.empty(m, b - a, dtype=torch.float32, device=dev)
            rc = lib.qi4_w4g64_gate_up_silu(x.data_ptr(), code, m, k, gsh.qweight.data_ptr(), gsh.scales.data_ptr(),
                                            gsh.zeros.data_ptr(), ush.qweight.data_ptr(), ush.scales.data_ptr(),
                                            ush.zeros.data_ptr(), part.data_ptr(), b - a, stream)
            mod.check(rc, "qi4_w4g64_gate_up_silu")
            ref[:, a:b] = part
        torch.cuda.synchronize()
        for p in range(world):
            if m > 16:  # the same tensor-core launch per shard: bit-identical
                assert torch.equal(bufs[p], ref), f"epoch {epoch}: rank {p}'s gathered buffer differs"
            else:  # grouped GEMV against the fused GEMV: projections may round one bf16 step apart
                d = (bufs[p] - ref).abs()
                assert bool((d <= 1e-3 + 2 ** -6 * ref.abs()).all()), float(d.max())
            assert torch.equal(bufs[p], bufs[0])
            assert flags[p][:world].tolist() == [epoch] * world
            assert int(flags[p][world]) == 0  # CTA counter re-armed
        # The gathered intermediate against the oracle (tensor-core tolerance).
        xo = x.float().cpu().numpy()
        gref = orc.linear(xo, gq.cpu().numpy(), gs.cpu().numpy(), gz.cpu().numpy(), None, out_features=n,
                          in_features=k, accumulate="f64")
        uref = orc.linear(xo, uq.cpu().numpy(), us.cpu().numpy(), uz.cpu().numpy(), None, out_features=n,
                          in_features=k, accumulate="f64")
        exp = gref / (1 + np.exp(-gref)) * uref
        got = bufs[0].cpu().numpy()
        assert np.all(np.abs(got - exp) <= 3e-2 + 2 ** -6 * np.abs(exp)), float(np.abs(got - exp).max())
    assert lib.qi4_device_status(torch.cuda.current_stream().cuda_stream) == 0


@pytest.mark.parametrize(("m", "world"), [(256, 2), (64, 3), (5, 2)])
def test_scatter_gathers_every_shard_into_every_rank(b200, cuda_device, m, world):
    """Tensor-core route (M > 16) and the grouped GEMV route (M <= 16); two
    and three emulated ranks, two calls on the same buffers."""
    _run_emulated(b200, cuda_device, m, 1280, 1536, world, torch.bfloat16, epochs=(1, 2), seed=m + world)


def test_scatter_fp32_activations_and_an_empty_shard(b200, cuda_device):
    """FP32 activations; 128 columns over three ranks on whole groups leave
    the third rank without columns: it still publishes its epoch."""
    _run_emulated(b200, cuda_device, 40, 128, 512, 3, torch.float32, epochs=(7,), seed=5)


def test_flag_wait_time_limit_reports_and_leaves_the_context_usable(b200, cuda_device):
    mod, lib = _lib(b200)
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.qi4_device_status(stream) == 0
    flags = torch.zeros(3, dtype=torch.int32, device=cuda_device)  # nobody will set these
    mod.check(lib.qi4_peer_flag_wait(flags.data_ptr(), 2, 1, 2_000_000, stream), "qi4_peer_flag_wait")
    torch.cuda.synchronize()
    assert lib.qi4_device_status(stream) == 1  # QI4_DEVICE_WAIT_TIMEOUT, read and cleared
    assert lib.qi4_device_status(stream) == 0
    assert float((torch.ones(4, device=cuda_device) * 2).sum()) == 8.0
    # Arguments are checked before any launch.
    assert lib.qi4_peer_flag_wait(flags.data_ptr(), 9, 1, 2_000_000, stream) == -1
    assert lib.qi4_peer_flag_wait(flags.data_ptr(), 2, 1, 10, stream) == -1


def test_column_fused_mlp_in_one_process_equals_the_unsplit_mlp(b200, cuda_device):
    """With one process the fused mode runs the same path with world = 1 (a
    local buffer, its own flag): equal to the fused gate/up + down_proj."""
    from types import SimpleNamespace

    par = _par(b200)
    rng = np.random.default_rng(3)

    def qlinear(n, k):
        qw, sc, z = orc.quantize_asymmetric_rtn(rng.standard_normal((n, k), dtype=np.float32) * 0.02)
        return SimpleNamespace(qweight=torch.from_numpy(qw).to(cuda_device), scales=torch.from_numpy(sc).to(cuda_device),
                               zeros=torch.from_numpy(z).to(cuda_device), bias=None, in_features=k, out_features=n)

    mlp = SimpleNamespace(gate_proj=qlinear(1280, 1536), up_proj=qlinear(1280, 1536), down_proj=qlinear(1536, 1280))
    x = torch.from_numpy(rng.standard_normal((96, 1536), dtype=np.float32)).to(torch.bfloat16).to(cuda_device)
    hm = b200.b200_w4g64_gate_up_silu(x, mlp.gate_proj, mlp.up_proj)
    d = mlp.down_proj
    ref = b200.b200_w4g64_linear(hm, d.qweight, d.scales, d.zeros, None, out_features=1536, in_features=1280,
                                 group_size=64, packing="canonical").to(torch.bfloat16)
    split = par.ColumnParallelMLP(mlp, mode="column_fused")
    for _ in range(2):
        assert torch.equal(split(x), ref)
    split.close()
    with pytest.raises(ValueError, match="column_fused"):
        par.ColumnParallelMLP(mlp, mode="column_fused", linear_fn=lambda x, s: x)

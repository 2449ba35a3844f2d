"""Column-split W4G64 on 2 GPUs over NCCL (skipped on a single-GPU host).

A split linear against the oracle, and the Qwen2 MLP in the three split
modes (two NCCL collectives; one all-reduce; the intermediate's gather fused
into the SwiGLU pass over CUDA IPC peer memory, called twice on the same
buffers) against the same MLP unsplit on one GPU (the b200 kernels either
way).
"""

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import w4g64 as orc

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_path):
    import importlib
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    par = importlib.import_module("qwen2-int4-systems_b200.parallel")
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    ok = True
    try:
        rng = np.random.default_rng(11)
        for m, n, k, dt in ((4, 1000, 1536, torch.bfloat16), (256, 8960, 1536, torch.bfloat16),
                            (64, 1536, 8960, torch.float16)):
            qw, sc, z = orc.quantize_asymmetric_rtn(rng.standard_normal((n, k), dtype=np.float32) * 0.02)
            x = torch.from_numpy(rng.standard_normal((m, k), dtype=np.float32)).to(dt)
            lin = par.ColumnParallelW4G64(torch.from_numpy(qw).to(dev), torch.from_numpy(sc).to(dev),
                                          torch.from_numpy(z).to(dev), None, in_features=k, out_features=n)
            got = lin(x.to(dev)).float().cpu().numpy()
            ref = orc.linear(x.float().numpy(), qw, sc, z, None, out_features=n, in_features=k, accumulate="f64")
            ok = ok and got.shape == ref.shape and bool(np.all(np.abs(got - ref) <= 2e-2 + np.abs(ref) * 2 ** -7))
        from types import SimpleNamespace

        def qlinear(n, k):
            qw, sc = orc.quantize_symmetric_rtn(rng.standard_normal((n, k), dtype=np.float32) * 0.02)
            z = np.zeros(((n * (k // 64) + 1) // 2, 1), dtype=np.uint8)
            return SimpleNamespace(qweight=torch.from_numpy(qw).to(dev), scales=torch.from_numpy(sc).to(dev),
                                   zeros=torch.from_numpy(z).to(dev), bias=None, in_features=k, out_features=n)

        mlp = SimpleNamespace(gate_proj=qlinear(8960, 1536), up_proj=qlinear(8960, 1536),
                              down_proj=qlinear(1536, 8960))
        x = torch.from_numpy(rng.standard_normal((512, 1536), dtype=np.float32)).to(torch.bfloat16).to(dev)
        b200 = importlib.import_module("qwen2-int4-systems_b200")
        hm = b200.b200_w4g64_gate_up_silu(x, mlp.gate_proj, mlp.up_proj)
        d = mlp.down_proj
        ref = b200.b200_w4g64_linear(hm, d.qweight, d.scales, d.zeros, None, out_features=1536, in_features=8960,
                                     group_size=64, packing="canonical").to(torch.bfloat16).float()
        for mode in ("column", "column_row", "column_fused"):
            split = par.ColumnParallelMLP(mlp, mode=mode)
            got = split(x).float()
            cos = torch.nn.functional.cosine_similarity(got.flatten(), ref.flatten(), dim=0)
            ok = ok and bool((got - ref).abs().max() <= 2e-2 + 2 ** -7 * ref.abs().max()) and float(cos) > 0.99999
            if mode == "column_fused":
                # A second call reuses the peer buffers with the next epoch;
                # a shorter input reuses them too.
                x2 = torch.flip(x, dims=(0,))[:300].contiguous()
                ref2 = torch.flip(ref, dims=(0,))[:300]
                got2 = split(x2).float()
                ok = ok and bool((got2 - ref2).abs().max() <= 2e-2 + 2 ** -7 * ref2.abs().max())
                lib = importlib.import_module("qwen2-int4-systems_b200._lib").load()
                ok = ok and lib.qi4_device_status(torch.cuda.current_stream().cuda_stream) == 0
                split.close()
        flag = torch.tensor([1 if ok else 0], device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        if rank == 0:
            with open(result_path, "w") as f:
                f.write(str(int(flag.item())))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_column_split_over_two_gpus_matches_oracle(tmp_path):
    result = tmp_path / "ok"
    mp.start_processes(_worker, args=(2, _free_port(), str(result)), nprocs=2, join=True, start_method="spawn")
    assert result.read_text() == "1"

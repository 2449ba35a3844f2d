"""Column-split W4G64 on 2 GPUs over NCCL (skipped on a single-GPU host)."""

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

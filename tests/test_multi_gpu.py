"""Two-GPU paths over NCCL (skipped with fewer than two GPUs).

* token-sharded calibration: each rank accumulates its own tokens on its own
  GPU, one all-reduce merges the fp32 accumulators; the statistics match a
  single GPU that saw every token (different summation order: max error
  1e-6 of the largest magnitude);
* row-sharded quantization: each rank quantizes its own rows with no
  communication; its bytes equal the same rows quantized on one GPU;
* full X^T X with tokens split over ranks and summed with one all-reduce.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

WIDTH, TOKENS, ROWS = 1024, 3000, 1000


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    from mxwave_b200 import synthetic as syn

    x = torch.from_numpy(syn.bf16_bits_to_f32(syn.det_activations(TOKENS, WIDTH, seed=41)))
    w = torch.from_numpy(syn.det_dense_weight(ROWS, WIDTH, 42, outlier_fraction=0.01).view("int16").copy())
    return x.to(torch.bfloat16), w.view(torch.bfloat16)


def _worker(rank: int, world: int, port: int, out_dir: str) -> None:
    from datetime import timedelta

    import torch.distributed as dist

    from mxwave_b200 import _lib
    from mxwave_b200.calibration import ActivationCollector
    from mxwave_b200.core import quantize_mxfp4

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        x, w = _inputs()
        lo, hi = TOKENS * rank // world, TOKENS * (rank + 1) // world
        col = ActivationCollector({"p.weight": WIDTH}, ("mean-abs", "rms", "block-hessian"), hessian_damp=1e-6)
        col.update("p.weight", x[lo:hi].to(dev))
        col.all_reduce()
        stats = col.finalize()
        r0, r1 = ROWS * rank // world, ROWS * (rank + 1) // world
        packed, scales = quantize_mxfp4(w[r0:r1].to(dev), gamma=stats["rms"]["p.weight"].to(dev))
        lib = _lib.load()
        xs = x[lo:hi].to(dev).contiguous()
        gram = torch.zeros(WIDTH, WIDTH, device=dev)
        stream = torch.cuda.current_stream(dev)
        _lib.check(lib.mxw_accumulate_xtx(xs.data_ptr(), hi - lo, WIDTH, WIDTH, gram.data_ptr(), WIDTH, None,
                                          stream.cuda_stream), "xtx")
        dist.all_reduce(gram)
        torch.cuda.synchronize(dev)
        torch.save({"stats": stats, "counts": col.observation_counts, "packed": packed.cpu(),
                    "scales": scales.cpu(), "gram": gram.cpu()}, os.path.join(out_dir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_two_gpu_token_and_row_sharding(tmp_path, cuda_device) -> None:
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from mxwave_b200 import _lib
    from mxwave_b200.calibration import ActivationCollector
    from mxwave_b200.core import quantize_mxfp4

    mp.start_processes(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    x, w = _inputs()
    col = ActivationCollector({"p.weight": WIDTH}, ("mean-abs", "rms", "block-hessian"), hessian_damp=1e-6)
    col.update("p.weight", x.to(cuda_device))
    want = col.finalize()
    lib = _lib.load()
    xd = x.to(cuda_device).contiguous()
    gram = torch.zeros(WIDTH, WIDTH, device=cuda_device)
    _lib.check(lib.mxw_accumulate_xtx(xd.data_ptr(), TOKENS, WIDTH, WIDTH, gram.data_ptr(), WIDTH, None,
                                      torch.cuda.current_stream().cuda_stream), "xtx")
    ranks = [torch.load(tmp_path / f"rank{r}.pt") for r in range(2)]

    def assert_near(got: torch.Tensor, expected: torch.Tensor, tol: float) -> None:
        # Relative to the largest magnitude: summation order differs between
        # one GPU and two shards plus an all-reduce.
        err = (got.double() - expected.double()).abs().max().item()
        assert err <= tol * expected.double().abs().max().item(), err

    for r in ranks:
        assert r["counts"] == {"p.weight": TOKENS}
        for objective in ("mean-abs", "rms", "block-hessian"):
            assert_near(r["stats"][objective]["p.weight"], want[objective]["p.weight"], 1e-6)
        assert_near(r["gram"], gram.cpu(), 1e-6)
    # Each rank's row shard, quantized on its own GPU with its all-reduced
    # rms, is byte-identical to the same rows quantized here with that rms.
    for rank, r in enumerate(ranks):
        a, b = ROWS * rank // 2, ROWS * (rank + 1) // 2
        g = r["stats"]["rms"]["p.weight"].to(cuda_device)
        p_all, s_all = quantize_mxfp4(w.to(cuda_device), gamma=g)
        assert torch.equal(r["packed"], p_all[a:b].cpu()) and torch.equal(r["scales"], s_all[a:b].cpu())

"""The sharded segment engine on 2 GPUs over NCCL (one process per GPU): one
track split across the ranks, overlap strips exchanged, compared with the
reference's apply_model output (golden fixture). Skipped with fewer than two
GPUs."""

from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, key: str, shifts: int, q) -> None:
    import sys

    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import torch.distributed as dist

    from conftest import golden, rel_err
    from unblend_b200.distributed import apply_model_sharded
    from unblend_b200.htdemucs import HTDemucsCuda
    from unblend_b200.synth import htdemucs_state_dict

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        g = golden("apply_small.pt")
        m = HTDemucsCuda(g["config"], htdemucs_state_dict(g["config"], g["seed"]), precision="fp32").cuda()
        out = apply_model_sharded(m, g["mix"][0].cuda(), overlap=g["overlap"], chunk_batch_size=1, shifts=shifts,
                                  shift_offsets=g[key].get("offsets"))
        err = rel_err(out[None].cpu()[..., :: g["decimate"]], g[key]["out"])
        lo, hi, own = apply_model_sharded(m, g["mix"][0].cuda(), overlap=g["overlap"], gather=False)
        # A host track: copied in by the engine, result back in page-locked host memory.
        host = apply_model_sharded(m, g["mix"][0].clone(), overlap=g["overlap"], chunk_batch_size=1, shifts=shifts,
                                   shift_offsets=g[key].get("offsets"), device=torch.device("cuda", rank))
        assert host.device.type == "cpu" and host.is_pinned()
        # Not bit-equal: the DConv statistics accumulate with float64 atomics, in any order.
        assert rel_err(host, out.cpu()) < 1e-6
        q.put((rank, err, lo, hi, tuple(own.shape)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("key,shifts", [("shifts0", 0), ("shifts1", 1)])
def test_sharded_apply_matches_reference_on_two_gpus(key, shifts):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, key, shifts, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err, lo, hi, shape in results:
        assert err < 1e-4, (rank, err)
        assert shape[-1] == hi - lo
    assert results[0][2] == 0 and results[0][3] == results[1][2]

"""FSDP peer-memory collectives on 2 GPUs (NCCL ranks): the fused reduce-scatter and AdamW+all-gather
kernels agree with the NCCL baseline path, including gradient accumulation across two backward passes."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import datetime

    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    from vlmrl import ops
    from vlmrl.core.optim import AdamWConfig
    from vlmrl.models.qwen3vl.config import get_preset
    from vlmrl.models.qwen3vl.params import all_layouts, init_params, text_layouts
    from vlmrl.parallel.fsdp import FSDPOptimizer, FSDPParams

    dev = torch.device("cuda", rank)
    spec = get_preset("tiny")
    units = init_params(spec, seed=0, device=dev)
    cfg = AdamWConfig(lr=1e-3, weight_decay=0.01, max_grad_norm=1.0)
    engines = {}
    for comm in ("p2p", "nccl"):
        fp = FSDPParams(all_layouts(spec), {k: v.clone() for k, v in units.items()}, dtype=torch.bfloat16,
                        trainable=[l.name for l in text_layouts(spec)], replicate=["visual"], comm=comm)
        engines[comm] = (fp, FSDPOptimizer(fp, cfg))
    assert engines["p2p"][0].comm == "p2p", "peer access unavailable between the two GPUs"
    results = {}
    for comm, (fp, opt) in engines.items():
        for step in range(1, 4):
            for acc in range(1 if step != 2 else 2):       # step 2 accumulates two backward passes
                for u in reversed(fp.order):
                    g = fp.grad(u)
                    gen = torch.Generator(device=dev).manual_seed(1000 * step + 100 * acc + 10 * rank + fp.slot[u])
                    g.copy_(torch.randn(g.shape, generator=gen, device=dev) * 1e-2)
                    fp.grad_done(u)
            opt.step(step)
            if comm == "p2p":
                ops.check_errors(rank)
                fp.verify_signals()          # every peer counter exactly where the protocol puts it
        ops.check_errors(rank)
        gathered = {u: fp.get(u).float().clone() for u in fp.order}
        master = opt.master_units()
        results[comm] = (gathered, master)
        torch.cuda.synchronize()
    if rank == 0:
        torch.save({c: ({k: v.cpu() for k, v in g.items()}, {k: v.cpu() for k, v in m.items()})
                    for c, (g, m) in results.items()}, out_path)
    engines["p2p"][0].close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_p2p_fsdp_matches_nccl(tmp_path):
    out = str(tmp_path / "p2p.pt")
    mp.start_processes(_worker, args=(2, _free_port(), out), nprocs=2, join=True, start_method="spawn")
    res = torch.load(out)
    g_p2p, m_p2p = res["p2p"]
    g_nccl, m_nccl = res["nccl"]
    for u in m_nccl:
        torch.testing.assert_close(m_p2p[u], m_nccl[u], atol=1e-6, rtol=1e-5, msg=lambda s: f"master {u}: {s}")
        # the gathered bf16 copy is the rounded fp32 master, on every rank
        torch.testing.assert_close(g_p2p[u][:m_p2p[u].numel()], m_p2p[u].bfloat16().float(), atol=0, rtol=0,
                                   msg=lambda s: f"gathered {u}: {s}")
        torch.testing.assert_close(g_p2p[u], g_nccl[u], atol=1e-2, rtol=1e-2)
